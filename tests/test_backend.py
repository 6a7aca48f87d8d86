"""CudaSm100Backend against a fake command runner (no GPU, no nvcc), in the
manner of the reference's CUDA-backend tests (tests/test_cuda_backend.py)."""

from __future__ import annotations

import json
import subprocess
from pathlib import Path

import pytest

from kernel_mcts_b200 import build as native_build
from kernel_mcts_b200.backend import (
    CudaSm100Backend,
    CudaSm100Config,
    Sm100Artifact,
    detect_candidate_abi,
    parse_payload,
    parse_ptxas_resources,
    schedule_program,
)
from kernel_mcts_b200.domain import KernelProgram
from kernel_mcts_b200.evaluation import (
    CandidateBenchmarkError,
    CandidateLaunchError,
    CandidateTimeoutError,
    EvaluationInfrastructureError,
)
from kernel_mcts_b200.profiling import LIGHTWEIGHT_V1_METRICS, SM100_V1_METRICS, parse_ncu_csv
from kernel_mcts_b200.workloads import (
    BF16_GEMM_4096_B200,
    BF16_GEMM_4096_RANDN,
    gemm_workload,
    multi_shape_gemm_workload,
)

ROOT_SOURCE = """
#include <cuda_bf16.h>
// a candidate with the reference ABI
extern "C" __global__ void bf16_gemm_root(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                          __nv_bfloat16* C, int M, int N, int K) {}
"""
LAUNCHER_SOURCE = """
#include <cuda_runtime.h>
extern "C" int bf16_gemm_launch(const void* A, const void* B, void* C, int M, int N, int K,
                                cudaStream_t stream) { return 0; }
"""
OK_CORRECTNESS = json.dumps({
    "status": "ok", "success": True, "maximum_error": 0.01, "mean_error": 0.001, "failed_test_id": None,
    "reference_metadata": {"implementation": "cuBLAS"}, "max_ulp": 1, "n_gt_1ulp": 0,
    "ulp_hist": [10, 2, 0, 0], "n_nonfinite": 0, "kernel": "candidate:bf16_gemm_root",
})


class FakeRunner:
    def __init__(self) -> None:
        self.calls: list[tuple[list[str], float, dict]] = []
        self.compile_returncode = 0
        self.compile_stderr = "ptxas info    : Compiling entry function 'bf16_gemm_root' for 'sm_100a'\n" \
                              "ptxas info    : Function properties for bf16_gemm_root\n" \
                              "    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads\n" \
                              "ptxas info    : Used 40 registers, used 1 barriers, 2048 bytes smem\n"
        self.correctness_stdout = OK_CORRECTNESS
        self.benchmark_stdout = json.dumps({"status": "ok", "timings_us": [10.0, 12.0, 11.0]})
        self.returncode = 0
        self.timeout_stage: str | None = None
        self.ncu_stdout = ""
        self.by_m: dict[tuple[str, str], str] = {}  # (mode, "--M=...") -> stdout for that shape

    def __call__(self, command, *, timeout, env):
        command = list(command)
        self.calls.append((command, timeout, dict(env)))
        if "-o" in command and command[0].endswith("nvcc"):
            # The candidate's own compile step is the one a test makes fail;
            # the harness object and the link always succeed here.
            candidate = "-c" in command and any(Path(part).name.startswith("candidate.") for part in command)
            if self.timeout_stage == "compile" and candidate:
                raise subprocess.TimeoutExpired(command, timeout)
            returncode = self.compile_returncode if candidate else 0
            if returncode == 0:
                Path(command[command.index("-o") + 1]).write_bytes(b"executable bytes")
            return subprocess.CompletedProcess(command, returncode, "", self.compile_stderr if candidate else "")
        if command[0].endswith("nvidia-smi"):
            return subprocess.CompletedProcess(command, 0, "40, 1965, 3996, 500.0, 1000.0, P0, 99, 20, 0x0000000000000000\n", "")
        if command[0].endswith("ncu"):
            return subprocess.CompletedProcess(command, 0, self.ncu_stdout, "")
        if self.timeout_stage == "execute":
            raise subprocess.TimeoutExpired(command, timeout)
        out = self.benchmark_stdout if "--mode=benchmark" in command else self.correctness_stdout
        mode = "benchmark" if "--mode=benchmark" in command else "correctness"
        for arg in command:
            out = self.by_m.get((mode, arg), out)
        return subprocess.CompletedProcess(command, self.returncode, "some log line\n" + out + "\n", "")


def make_backend(tmp_path, runner, **changes) -> CudaSm100Backend:
    cfg = {"artifact_root": tmp_path, "nvcc": "/opt/cuda/bin/nvcc", "ncu": "/opt/cuda/bin/ncu",
           "warmup_count": 2, "measurement_count": 3, **changes}
    return CudaSm100Backend(CudaSm100Config(**cfg), runner=runner)


def test_candidate_compile_command_targets_sm100a_and_links_the_library(tmp_path):
    """The harness is compiled once per ABI (relocatable device code); each
    candidate is compiled alone with ptxas resource output, then linked to it
    and to the library."""
    runner = FakeRunner()
    result = make_backend(tmp_path, runner).compile(KernelProgram(ROOT_SOURCE), BF16_GEMM_4096_B200)
    assert result.success and result.artifact is not None
    harness, compile_step, link = (c[0] for c in runner.calls[:3])
    assert "-c" in harness and any(p.endswith("harness.cu") for p in harness)
    assert "-DKMCTS_CANDIDATE_ROOT" in harness and "-rdc=true" in harness
    command, timeout, env = runner.calls[1]
    assert command[0] == "/opt/cuda/bin/nvcc"
    for step in (harness, compile_step, link):
        assert "arch=compute_100a,code=sm_100a" in step
        assert not any("--keep" in part for part in step)  # no PTX kept: nothing reads it
    assert "-c" in compile_step and "-rdc=true" in compile_step and "-Xptxas=-v" in compile_step
    assert "-lkmcts_gemm_sm100" in link and "-lcublas" in link and "-rdc=true" in link
    assert any(p.startswith(str(tmp_path / "harness-root-")) for p in link)
    assert set(env) <= {"PATH", "LANG", "LC_ALL", "LD_LIBRARY_PATH", "CUDA_VISIBLE_DEVICES", "HOME"}
    assert result.compiler_context["ptxas"] == [
        {"function": "bf16_gemm_root", "stack_bytes": 0, "spill_store_bytes": 0, "spill_load_bytes": 0,
         "registers": 40, "barriers": 1, "static_smem_bytes": 2048}
    ]


def test_candidate_builds_are_cached_on_disk_across_backends(tmp_path):
    """A backend sharing the candidate cache (another process, e.g. a host
    compile pool ahead of the GPU workers) reuses a build and its compiler
    output; the harness object is built once per ABI."""
    first = FakeRunner()
    built = make_backend(tmp_path / "a", first, candidate_cache=tmp_path / "cache").compile(
        KernelProgram(ROOT_SOURCE), BF16_GEMM_4096_B200)
    second = FakeRunner()
    reused = make_backend(tmp_path / "b", second, candidate_cache=tmp_path / "cache").compile(
        KernelProgram(ROOT_SOURCE + "\n// a comment only"), BF16_GEMM_4096_B200)
    assert built.success and reused.success and second.calls == []
    assert reused.artifact.executable == built.artifact.executable
    assert reused.compiler_context["ptxas"] == built.compiler_context["ptxas"]
    other = make_backend(tmp_path / "b", second, candidate_cache=tmp_path / "cache").compile(
        KernelProgram(ROOT_SOURCE.replace("int K) {}", "int K) { (void)M; }")), BF16_GEMM_4096_B200)
    assert other.success and len(second.calls) == 2  # compile + link; the harness object is reused


def test_launcher_abi_is_detected_and_compiled_with_its_macro(tmp_path):
    runner = FakeRunner()
    make_backend(tmp_path, runner).compile(KernelProgram(LAUNCHER_SOURCE), BF16_GEMM_4096_B200)
    assert "-DKMCTS_CANDIDATE_LAUNCHER" in runner.calls[0][0] and "-DKMCTS_CANDIDATE_LAUNCHER" in runner.calls[1][0]
    assert detect_candidate_abi(LAUNCHER_SOURCE) == "launcher"
    assert detect_candidate_abi("// bf16_gemm_launch(\n" + ROOT_SOURCE) == "root"  # comments ignored
    with pytest.raises(ValueError):
        detect_candidate_abi("__global__ void other() {}")


def test_compile_failure_and_timeout_are_reported_not_raised(tmp_path):
    runner = FakeRunner()
    runner.compile_returncode = 1
    failed = make_backend(tmp_path, runner).compile(KernelProgram(ROOT_SOURCE), BF16_GEMM_4096_B200)
    assert not failed.success and not failed.timed_out and failed.artifact is None
    runner = FakeRunner()
    runner.timeout_stage = "compile"
    timed = make_backend(tmp_path / "t", runner).compile(KernelProgram(ROOT_SOURCE), BF16_GEMM_4096_B200)
    assert not timed.success and timed.timed_out


def test_execute_builds_the_reference_harness_command(tmp_path):
    runner = FakeRunner()
    backend = make_backend(tmp_path, runner)
    artifact = Sm100Artifact("id", tmp_path / "evaluate", ("--kernel=candidate",), "root")
    checked = backend.check_correctness(artifact, BF16_GEMM_4096_B200)
    assert checked.success and checked.maximum_error == 0.01 and checked.mean_error == 0.001
    assert checked.reference_metadata["max_ulp"] == 1
    command = runner.calls[-1][0]
    for flag in ("--mode=correctness", "--M=4096", "--N=4096", "--K=4096", "--rtol=0.02", "--atol=0.02",
                 "--seed=0", "--warmups=2", "--measurements=3", "--b-layout=col", "--inputs=uniform",
                 "--kernel=candidate"):
        assert flag in command, flag


def test_benchmark_statistics_and_operating_state(tmp_path):
    runner = FakeRunner()
    backend = make_backend(tmp_path, runner)
    result = backend.benchmark(Sm100Artifact("id", tmp_path / "e"), BF16_GEMM_4096_RANDN)
    assert result.timings_us == (10.0, 12.0, 11.0)
    assert result.median_us == 11.0 and result.mean_us == 11.0 and result.min_us == 10.0 and result.max_us == 12.0
    assert result.stddev_us == pytest.approx((2 / 3) ** 0.5)
    assert result.warmup_count == 2
    assert result.gpu_operating_state["before"]["clocks.sm"] == 1965.0
    assert "--inputs=randn" in runner.calls[-2][0] and "--b-layout=row" in runner.calls[-2][0]


def test_timing_count_mismatch_is_an_infrastructure_failure(tmp_path):
    runner = FakeRunner()
    runner.benchmark_stdout = json.dumps({"status": "ok", "timings_us": [1.0]})
    with pytest.raises(EvaluationInfrastructureError):
        make_backend(tmp_path, runner).benchmark(Sm100Artifact("id", tmp_path / "e"), BF16_GEMM_4096_B200)


@pytest.mark.parametrize(
    "stdout,returncode,error",
    [
        ('{"status":"launch_failure","reason":"device_wait_timeout"}', 1, CandidateLaunchError),
        ('{"status":"benchmark_failure"}', 1, CandidateBenchmarkError),
        ('{"status":"infrastructure_failure","operation":"cudaMalloc_A"}', 2, EvaluationInfrastructureError),
        ("not json", 0, EvaluationInfrastructureError),
        ("[1, 2]", 0, EvaluationInfrastructureError),
    ],
)
def test_harness_statuses_map_to_the_evaluation_taxonomy(tmp_path, stdout, returncode, error):
    runner = FakeRunner()
    runner.correctness_stdout = stdout
    runner.returncode = returncode
    with pytest.raises(error):
        make_backend(tmp_path, runner).check_correctness(Sm100Artifact("id", tmp_path / "e"), BF16_GEMM_4096_B200)


def test_execution_timeout_is_a_candidate_timeout(tmp_path):
    runner = FakeRunner()
    runner.timeout_stage = "execute"
    with pytest.raises(CandidateTimeoutError):
        make_backend(tmp_path, runner).check_correctness(Sm100Artifact("id", tmp_path / "e"), BF16_GEMM_4096_B200)


def test_payload_is_the_last_stdout_line():
    assert parse_payload('warning: x\n{"status": "ok"}\n') == {"status": "ok"}
    assert parse_payload('{"status":"ok","maximum_error":NaN}')["status"] == "ok"  # NaN token accepted


def test_schedule_programs_select_prebuilt_kernels_without_nvcc(tmp_path):
    runner = FakeRunner()
    backend = make_backend(tmp_path, runner)
    ok = backend.compile(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3),
                         BF16_GEMM_4096_B200)
    assert ok.success and runner.calls == []  # no compiler invocation
    assert "--tile-m=256" in ok.artifact.extra_args and "--kernel=tcgen05" in ok.artifact.extra_args
    assert ok.artifact.executable == native_build.HARNESS
    too_big = backend.compile(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=6),
                              BF16_GEMM_4096_B200)
    assert not too_big.success and "shared memory" in too_big.stderr
    quad = backend.compile(schedule_program(tile_m=256, cluster_m=2, cluster_n=2), BF16_GEMM_4096_B200)
    assert quad.success and "--cluster-n=2" in quad.artifact.extra_args
    multicast = backend.compile(schedule_program(tile_m=128, cluster_m=1, cluster_n=2), BF16_GEMM_4096_B200)
    assert not multicast.success and "multicast" in multicast.stderr
    with pytest.raises(ValueError):
        backend.normalize_program(KernelProgram('{"warp_size": 7}', "kmcts_sm100"))


def test_contract_validation(tmp_path):
    backend = make_backend(tmp_path, FakeRunner())
    with pytest.raises(ValueError):
        backend.compile(KernelProgram(ROOT_SOURCE, "cute_dsl"), BF16_GEMM_4096_B200)
    bad = gemm_workload("x", 64, 64, 64)
    object.__setattr__(bad, "dtype", "float16")
    with pytest.raises(ValueError):
        backend.compile(KernelProgram(ROOT_SOURCE), bad)


def test_fingerprint_hashes_bytes_and_schedule(tmp_path):
    exe = tmp_path / "e"
    exe.write_bytes(b"abc")
    backend = make_backend(tmp_path, FakeRunner())
    a = backend.binary_fingerprint(Sm100Artifact("1", exe, ("--tile-n=256",)), {})
    b = backend.binary_fingerprint(Sm100Artifact("1", exe, ("--tile-n=128",)), {})
    assert a != b and len(a) == 64


def test_normalize_strips_comments_and_whitespace(tmp_path):
    backend = make_backend(tmp_path, FakeRunner())
    assert backend.normalize_program(KernelProgram("a  // x\n/* y */ b\n")) == "a b"


def test_ptxas_parse_multiple_kernels():
    text = ("ptxas info    : Compiling entry function 'k1' for 'sm_100a'\n"
            "ptxas info    : Used 94 registers, used 1 barriers\n"
            "ptxas info    : Compiling entry function 'k2' for 'sm_100a'\n"
            "    32 bytes stack frame, 4 bytes spill stores, 8 bytes spill loads\n"
            "ptxas info    : Used 40 registers\n")
    got = parse_ptxas_resources(text)
    assert [k["function"] for k in got] == ["k1", "k2"]
    assert got[0]["registers"] == 94 and got[1]["spill_load_bytes"] == 8


def test_ncu_csv_long_and_wide_layouts():
    long_rows = ['"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"']
    for i, m in enumerate(SM100_V1_METRICS):
        long_rows.append(f'"0","gemm","{m}","u","{i},000.5"')
    parsed = parse_ncu_csv("\n".join(long_rows), SM100_V1_METRICS)
    assert parsed[SM100_V1_METRICS[1]]["value"] == 1000.5
    wide = ",".join(f'"{m}"' for m in SM100_V1_METRICS) + "\n" + ",".join('"u"' for _ in SM100_V1_METRICS) + "\n" + \
        ",".join(f'"{i}"' for i, _ in enumerate(SM100_V1_METRICS))
    assert parse_ncu_csv(wide, SM100_V1_METRICS)[SM100_V1_METRICS[2]]["value"] == 2.0
    with pytest.raises(ValueError):
        parse_ncu_csv("garbage", SM100_V1_METRICS)


MIX = multi_shape_gemm_workload("mix", [(512, 256, 128, 0.75), (1024, 512, 256, 0.25)], b_layout="row",
                                inputs="randn")


def test_multi_shape_benchmark_reports_each_shape_and_the_weighted_median(tmp_path):
    runner = FakeRunner()
    runner.by_m[("benchmark", "--M=512")] = json.dumps({"status": "ok", "timings_us": [10.0, 12.0, 11.0]})
    runner.by_m[("benchmark", "--M=1024")] = json.dumps({"status": "ok", "timings_us": [40.0, 44.0, 42.0]})
    result = make_backend(tmp_path, runner).benchmark(Sm100Artifact("id", tmp_path / "e"), MIX)
    assert result.per_shape_median_us == {"K=128,M=512,N=256": 11.0, "K=256,M=1024,N=512": 42.0}
    assert result.median_us == pytest.approx(0.75 * 11.0 + 0.25 * 42.0)
    assert len(result.timings_us) == 6 and result.min_us == 10.0 and result.max_us == 44.0
    runs = [c[0] for c in runner.calls if "--mode=benchmark" in c[0]]
    assert [next(a for a in r if a.startswith("--M=")) for r in runs] == ["--M=512", "--M=1024"]


def test_multi_shape_correctness_fails_on_any_shape_and_names_it(tmp_path):
    runner = FakeRunner()
    bad = json.loads(OK_CORRECTNESS)
    bad.update(success=False, maximum_error=0.5, mean_error=0.01)
    runner.by_m[("correctness", "--M=1024")] = json.dumps(bad)
    result = make_backend(tmp_path, runner).check_correctness(Sm100Artifact("id", tmp_path / "e"), MIX)
    assert not result.success and result.failed_test_id == "K=256,M=1024,N=512"
    assert result.maximum_error == 0.5
    assert set(result.reference_metadata["per_shape"]) == {"K=128,M=512,N=256", "K=256,M=1024,N=512"}
    good = make_backend(tmp_path, FakeRunner()).check_correctness(Sm100Artifact("id", tmp_path / "e"), MIX)
    assert good.success and good.failed_test_id is None


def test_multi_shape_schedule_must_be_legal_on_every_shape(tmp_path):
    backend = make_backend(tmp_path, FakeRunner())
    ok = backend.compile(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3), MIX)
    assert ok.success
    ragged = multi_shape_gemm_workload("r", [(512, 256, 128, 0.5), (512, 256, 100, 0.5)], b_layout="row")
    rejected = backend.compile(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3), ragged)
    assert not rejected.success and "statically rejected" in rejected.stderr


def test_multi_shape_reward_through_the_evaluator(tmp_path):
    from kernel_mcts_b200.domain import BenchmarkResult
    from kernel_mcts_b200.evaluation import BackendKernelEvaluator, EvaluationContext
    import math

    runner = FakeRunner()
    runner.by_m[("benchmark", "--M=512")] = json.dumps({"status": "ok", "timings_us": [10.0, 10.0, 10.0]})
    runner.by_m[("benchmark", "--M=1024")] = json.dumps({"status": "ok", "timings_us": [40.0, 40.0, 40.0]})
    root = BenchmarkResult(timings_us=(1.0,), median_us=1.0, warmup_count=0,
                           per_shape_median_us={"K=128,M=512,N=256": 20.0, "K=256,M=1024,N=512": 40.0})
    context = EvaluationContext("w0", "env", {}, {})
    evaluator = BackendKernelEvaluator(backend=make_backend(tmp_path, runner), root_benchmark=root, context=context)
    result = evaluator.evaluate(schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3), MIX)
    assert result.status.value == "VALID", result
    assert result.reward == pytest.approx(0.75 * math.log(2.0) + 0.25 * math.log(1.0))


# ------------------------------------------------------- profile metric sets


def _query_listing(metrics):
    rows = ["Metric Name  Metric Type  Metric Unit  Metric Description"]
    rows += [f"{m}  Counter  byte  something" for m in metrics]
    return "\n".join(rows)


def _wide_csv(metrics):
    return (",".join(f'"{m}"' for m in metrics) + "\n" + ",".join('"u"' for _ in metrics) + "\n"
            + ",".join(f'"{i + 1}"' for i, _ in enumerate(metrics)))


def test_sm100_metric_set_is_validated_against_ncu_before_profiling(tmp_path):
    """As src/kernel_mcts/cuda_backend.py:413-461: a non-default metric set is
    checked against `ncu --query-metrics-mode all` once, and a set the GPU's
    ncu does not offer is refused with the missing names."""
    from kernel_mcts_b200.evaluation import EvaluationInfrastructureError

    class QueryRunner(FakeRunner):
        def __init__(self, listing):
            super().__init__()
            self.listing = listing

        def __call__(self, command, *, timeout, env):
            if command[0].endswith("ncu") and "--query-metrics-mode" in command:
                self.calls.append((list(command), timeout, dict(env)))
                return subprocess.CompletedProcess(command, 0, self.listing, "")
            return super().__call__(command, timeout=timeout, env=env)

    artifact = Sm100Artifact("id", tmp_path / "exe", abi="schedule")
    # One metric missing (the exempt launch attribute does not count).
    partial = [m for m in SM100_V1_METRICS if m not in ("launch__registers_per_thread", "dram__bytes_read.sum")]
    runner = QueryRunner(_query_listing(partial))
    with pytest.raises(EvaluationInfrastructureError, match="dram__bytes_read.sum"):
        make_backend(tmp_path, runner).lightweight_profile(artifact, BF16_GEMM_4096_B200, "sm100_v1")
    assert not any("--metrics" in c[0] for c in runner.calls)  # refused before profiling
    # Complete listing: validated once, then profiled; the second call skips the query.
    runner = QueryRunner(_query_listing([m for m in SM100_V1_METRICS if m != "launch__registers_per_thread"]))
    runner.ncu_stdout = _wide_csv(SM100_V1_METRICS)
    backend = make_backend(tmp_path, runner)
    for _ in range(2):
        profile = backend.lightweight_profile(artifact, BF16_GEMM_4096_B200, "sm100_v1")
        assert profile["metric_set"] == "sm100_v1"
        assert profile["summary"]["tensor_pipe_active_pct_of_elapsed"] == 3.0
    queries = [c[0] for c in runner.calls if "--query-metrics-mode" in c[0]]
    assert queries == [["/opt/cuda/bin/ncu", "--query-metrics-mode", "all", "--devices", "0"]]
    profiled = [c[0] for c in runner.calls if "--metrics" in c[0]]
    assert len(profiled) == 2 and "--clock-control" in profiled[0] and "none" in profiled[0]
    # The default set is never queried (the reference skips it too).
    runner = QueryRunner("")
    runner.ncu_stdout = _wide_csv(LIGHTWEIGHT_V1_METRICS)
    make_backend(tmp_path, runner).lightweight_profile(artifact, BF16_GEMM_4096_B200, "lightweight_v1")
    assert not any("--query-metrics-mode" in c[0] for c in runner.calls)


def test_sm100_metric_set_is_offered_by_this_ncu_for_b200():
    """The installed ncu lists every sm100_v1 metric for the B200 chip (gb100);
    `--chips` answers without a GPU."""
    import shutil

    from kernel_mcts_b200.profiling import metrics_missing_from_query, resolve_metric_set

    ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
    if not Path(ncu).exists():
        pytest.skip("ncu not installed")
    out = subprocess.run([ncu, "--query-metrics-mode", "all", "--chips", "gb100"], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    for metric_set in ("sm100_v1", "lightweight_v1"):
        assert metrics_missing_from_query(resolve_metric_set(metric_set, "sm_100a"), out.stdout) == []
