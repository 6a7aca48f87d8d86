"""The harness executable, the sm_100a backend, the evaluator and the vendor
columns on a B200: real nvcc builds of candidates with both ABIs, real runs."""

from __future__ import annotations

import json
import math
import subprocess

import pytest

from kernel_mcts_b200 import build as native_build
from kernel_mcts_b200.backend import CudaSm100Backend, CudaSm100Config, schedule_program
from kernel_mcts_b200.domain import InvalidReason, KernelProgram, ProposalStatus
from kernel_mcts_b200.evaluation import BackendKernelEvaluator, EvaluationContext
from kernel_mcts_b200.vendor_baselines import VendorBaselineSuite
from kernel_mcts_b200.workloads import gemm_workload

pytestmark = pytest.mark.gpu

# A deliberately simple candidate with the reference ABI (one thread per output).
NAIVE_ROOT = r"""
#include <cuda_bf16.h>
extern "C" __global__ void bf16_gemm_root(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                          __nv_bfloat16* C, int M, int N, int K) {
    int row = blockIdx.y * blockDim.y + threadIdx.y, col = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= M || col >= N) return;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) acc += __bfloat162float(A[row * K + k]) * __bfloat162float(B[col * K + k]);
    C[row * N + col] = __float2bfloat16(acc);
}
"""
# The same kernel but it forgets the last k: wrong results.
WRONG_ROOT = NAIVE_ROOT.replace("k < K;", "k < K - 1;")
# A host-launcher candidate that owns its launch: the library's tcgen05 kernel.
LAUNCHER = r"""
#include <cuda_runtime.h>
#include "kmcts_gemm.h"
extern "C" int bf16_gemm_launch(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
    return kmcts_bf16_gemm_ex(A, B, C, M, N, K, KMCTS_B_COL, nullptr, s, nullptr);
}
"""
FAILING_LAUNCHER = LAUNCHER.replace("return kmcts_bf16_gemm_ex", "(void)kmcts_bf16_gemm_ex; return 1; //")

WORKLOAD = gemm_workload("bf16_gemm_512_test", 512, 512, 512)
CONTEXT = EvaluationContext("test-worker", "test-manifest", {}, {"gpu": "B200"})


@pytest.fixture(scope="module")
def backend(tmp_path_factory, cuda_device):
    native_build.build_all()
    return CudaSm100Backend(CudaSm100Config(artifact_root=tmp_path_factory.mktemp("artifacts"),
                                            warmup_count=2, measurement_count=5))


@pytest.fixture(scope="module")
def evaluator(backend):
    root = backend.compile(KernelProgram(NAIVE_ROOT), WORKLOAD)
    assert root.success, root.stderr
    root_bench = backend.benchmark(root.artifact, WORKLOAD)
    return BackendKernelEvaluator(backend=backend, root_benchmark=root_bench, context=CONTEXT)


def run_harness(*args: str) -> dict:
    out = subprocess.run([str(native_build.HARNESS), *args], capture_output=True, text=True, timeout=300)
    payload = json.loads(out.stdout.strip().splitlines()[-1])
    payload["_returncode"] = out.returncode
    return payload


def test_harness_correctness_and_benchmark_modes(backend):
    ok = run_harness("--mode=correctness", "--M=512", "--N=384", "--K=1024", "--seed=3")
    assert ok["status"] == "ok" and ok["success"] is True and ok["_returncode"] == 0
    assert ok["reference_metadata"]["implementation"] == "cuBLAS" and ok["max_ulp"] <= 1
    bench = run_harness("--mode=benchmark", "--M=512", "--N=384", "--K=1024", "--warmups=3", "--measurements=7")
    assert bench["status"] == "ok" and len(bench["timings_us"]) == 7 and all(t > 0 for t in bench["timings_us"])
    bad = run_harness("--mode=nonsense", "--M=1", "--N=1", "--K=1")
    assert bad == {"status": "infrastructure_failure", "operation": "arguments", "_returncode": 2}


def test_harness_integer_inputs_match_cublas_bit_for_bit(backend):
    for layout in ("col", "row"):
        res = run_harness("--mode=correctness", "--M=1024", "--N=1024", "--K=2048", "--inputs=int",
                          f"--b-layout={layout}")
        assert res["success"] and res["max_ulp"] == 0 and res["maximum_error"] == 0.0, res


def test_vendor_columns_under_the_same_protocol(backend):
    results = VendorBaselineSuite(backend).run(gemm_workload("vendor_1024", 1024, 1024, 1024))
    assert set(results) == {"cublas", "cutlass"}
    for name in ("cublas", "cutlass"):
        column = results[name]
        assert column["correctness"]["success"] is True, column
        assert column["benchmark"].median_us > 0


def test_root_abi_candidate_is_valid(evaluator):
    result = evaluator.evaluate(KernelProgram(NAIVE_ROOT + "\n// same kernel, new text\n"), WORKLOAD)
    assert result.status == ProposalStatus.VALID, result
    assert abs(result.reward) < 1.0  # the same kernel as the root


def test_launcher_candidate_owns_its_launch_and_is_much_faster(evaluator):
    result = evaluator.evaluate(KernelProgram(LAUNCHER), WORKLOAD)
    assert result.status == ProposalStatus.VALID, result
    assert result.reward > math.log(3.0), result.reward


def test_wrong_candidate_fails_correctness(evaluator):
    result = evaluator.evaluate(KernelProgram(WRONG_ROOT), WORKLOAD)
    assert result.status == ProposalStatus.INVALID
    assert result.invalid_reason == InvalidReason.CORRECTNESS_FAILURE


def test_launch_failure_is_reported(evaluator):
    result = evaluator.evaluate(KernelProgram(FAILING_LAUNCHER), WORKLOAD)
    assert result.invalid_reason == InvalidReason.LAUNCH_FAILURE


def test_compile_error_is_reported(evaluator):
    result = evaluator.evaluate(KernelProgram(NAIVE_ROOT.replace("float acc", "flot acc")), WORKLOAD)
    assert result.invalid_reason == InvalidReason.COMPILE_FAILURE


def test_schedule_programs_evaluate_without_nvcc(evaluator):
    good = evaluator.evaluate(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3), WORKLOAD)
    assert good.status == ProposalStatus.VALID and good.reward > 0
    one_cta = evaluator.evaluate(schedule_program(tile_m=128, cluster_m=1, tile_n=128, tile_k=64, stages=4), WORKLOAD)
    assert one_cta.status == ProposalStatus.VALID
    rejected = evaluator.evaluate(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=5), WORKLOAD)
    assert rejected.invalid_reason == InvalidReason.COMPILE_FAILURE


def test_inprocess_schedule_evaluation_matches_the_harness_path(backend):
    """Schedule programs evaluated in process see the harness's inputs (the
    library generator) and its acceptance test; results agree."""
    from kernel_mcts_b200.domain import BenchmarkResult
    from kernel_mcts_b200.inprocess import HybridSm100Backend, InProcessSm100Backend

    workload = gemm_workload("inproc_1024", 1024, 768, 512)
    hybrid = HybridSm100Backend(backend, InProcessSm100Backend(warmup_count=2, measurement_count=5))
    ev_in = BackendKernelEvaluator(backend=hybrid, root_benchmark=BenchmarkResult((100.0,), 100.0), context=CONTEXT)
    ev_sub = BackendKernelEvaluator(backend=backend, root_benchmark=BenchmarkResult((100.0,), 100.0), context=CONTEXT)
    program = schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3)
    fast = ev_in.evaluate(program, workload)
    slow = ev_sub.evaluate(program, workload)
    assert fast.status == slow.status == ProposalStatus.VALID
    assert fast.correctness.maximum_error == slow.correctness.maximum_error
    assert fast.correctness.reference_metadata["max_ulp"] <= 1
    assert 0.5 < fast.benchmark.median_us / slow.benchmark.median_us < 2.0
    cand = ev_in.evaluate(KernelProgram(LAUNCHER), workload)  # candidate sources still go through nvcc
    assert cand.status == ProposalStatus.VALID


def test_pool_sweep_on_one_gpu_in_process(backend, tmp_path):
    from kernel_mcts_b200.pool import EvaluationPool, WorkerSpec
    from kernel_mcts_b200.sweep import run_schedule_sweep, schedule_grid

    workload = gemm_workload("sweep_2048", 2048, 2048, 2048, b_layout="row", inputs="randn")
    spec = WorkerSpec("kernel_mcts_b200.pool:sm100_evaluator",
                      {"artifact_root": str(tmp_path), "root_us": 100.0, "warmup_count": 2, "measurement_count": 5})
    with EvaluationPool([0], spec) as pool:
        report = run_schedule_sweep(pool, workload, {"benchmark": {"median_us": 50.0}}, schedules=schedule_grid(24, 3))
    assert report["status"] == "ok" and report["evaluations"] > 0
    assert all(t["status"] in ("VALID", "STATICALLY_REJECTED") for t in report["trials"]), report["trials"]


def test_multi_shape_workload_in_process_and_through_the_harness(backend):
    """A weighted two-shape workload: both backends evaluate every shape and
    report per-shape medians; the reward weights the per-shape speed-ups."""
    from kernel_mcts_b200.domain import BenchmarkResult
    from kernel_mcts_b200.inprocess import HybridSm100Backend, InProcessSm100Backend
    from kernel_mcts_b200.workloads import multi_shape_gemm_workload

    workload = multi_shape_gemm_workload("mix_small", [(1024, 1024, 1024, 0.5), (2048, 512, 1536, 0.5)],
                                         b_layout="row", inputs="randn")
    keys = {"K=1024,M=1024,N=1024", "K=1536,M=2048,N=512"}
    root = BenchmarkResult((100.0,), 100.0, per_shape_median_us={k: 100.0 for k in keys})
    program = schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3)
    hybrid = HybridSm100Backend(backend, InProcessSm100Backend(warmup_count=2, measurement_count=5))
    for be in (hybrid, backend):
        result = BackendKernelEvaluator(backend=be, root_benchmark=root, context=CONTEXT).evaluate(program, workload)
        assert result.status == ProposalStatus.VALID, result
        assert set(result.benchmark.per_shape_median_us) == keys
        expect = sum(0.5 * math.log(100.0 / t) for t in result.benchmark.per_shape_median_us.values())
        assert result.reward == pytest.approx(expect)
        assert set(result.correctness.reference_metadata["per_shape"]) == keys


def test_pool_autotuner_on_one_gpu(tmp_path):
    """The post-search autotuner over the in-process pool: every schedule
    trial is evaluated (or statically rejected) and the best reward kept."""
    from kernel_mcts_b200.autotune import PoolAutotuner, TuningConfig
    from kernel_mcts_b200.pool import EvaluationPool, WorkerSpec

    workload = gemm_workload("tune_2048", 2048, 2048, 2048, b_layout="row", inputs="randn")
    spec = WorkerSpec("kernel_mcts_b200.pool:sm100_evaluator",
                      {"artifact_root": str(tmp_path), "root_us": 100.0, "warmup_count": 2, "measurement_count": 5})
    program = schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3)
    with EvaluationPool([0], spec) as pool:
        baseline = pool.evaluate(program, workload)
        assert baseline.status == ProposalStatus.VALID
        result = PoolAutotuner(pool, workload, TuningConfig(budget=8, method="random", seed=1)).run(baseline)
    assert result.used == 8
    statuses = {t.evaluation.status for t in result.trials}
    assert statuses <= {ProposalStatus.VALID, ProposalStatus.INVALID}, statuses
    assert any(t.evaluation.status == ProposalStatus.VALID for t in result.trials)
    assert result.best is not None and result.best.reward >= baseline.reward


def test_sm100_metric_set_profiles_a_schedule_on_b200(backend):
    """The worker's /profile path on a B200: the sm100_v1 metric set is
    validated against this GPU's ncu (--query-metrics-mode all), then one
    launch of a 256^3 schedule program is profiled through
    lightweight_profile (one kernel, one launch, --clock-control none).  The
    same harness command runs once without ncu first and must exit 0."""
    import shutil

    if shutil.which("ncu") is None:
        pytest.skip("ncu not installed")
    workload = gemm_workload("bf16_gemm_256_profile", 256, 256, 256)
    compiled = backend.compile(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3), workload)
    assert compiled.success, compiled.stderr
    target = backend.profile_target_command(compiled.artifact, workload)
    plain = subprocess.run(target, capture_output=True, text=True, timeout=120,
                           env=dict(backend.config.subprocess_environment))
    assert plain.returncode == 0, plain.stdout[-2000:] + plain.stderr[-2000:]
    profile = backend.lightweight_profile(compiled.artifact, workload, "sm100_v1")
    assert profile["metric_set"] == "sm100_v1" and profile["profiler"] == "ncu"
    summary = profile["summary"]
    assert summary["tensor_pipe_active_pct_of_elapsed"] > 0.0
    assert summary["duration"] > 0.0 and summary["sm_cycles_active"] > 0.0
