"""The tier-0 evaluator's state machine, reward and state key (CPU, fake
backend), in the manner of the reference's tests/test_evaluation.py."""

from __future__ import annotations

import math
import sys
from dataclasses import dataclass, field
from pathlib import Path

import pytest

from kernel_mcts_b200.domain import (
    BenchmarkResult,
    CompileStatus,
    CorrectnessStatus,
    InvalidReason,
    KernelProgram,
    ProposalStatus,
    ShapeCase,
    WorkloadContract,
)
from kernel_mcts_b200.evaluation import (
    BackendKernelEvaluator,
    CandidateBenchmarkError,
    CandidateLaunchError,
    CandidateTimeoutError,
    EvaluationContext,
    EvaluationInfrastructureError,
    root_normalized_reward,
    state_key,
)
from kernel_mcts_b200.serialization import deserialize_evaluation, serialize_evaluation
from kernel_mcts_b200.workloads import BF16_GEMM_4096_B200

CONTEXT = EvaluationContext("worker-0", "manifest-0", {"block": [16, 16, 1]}, {"gpu": "B200", "nvcc": "12.9"})
ROOT = BenchmarkResult((100.0,), 100.0)


@dataclass
class Artifact:
    artifact_id: str = "artifact-1"


@dataclass
class Compiled:
    success: bool = True
    artifact: Artifact | None = field(default_factory=Artifact)
    stdout: str = ""
    stderr: str = ""
    duration_seconds: float = 0.5
    timed_out: bool = False
    artifact_paths: tuple[str, ...] = ("/tmp/x",)
    compiler_context: dict | None = None


@dataclass
class Checked:
    success: bool = True
    maximum_error: float = 0.01
    mean_error: float = 0.001
    failed_test_id: str | None = None
    reference_metadata: dict = field(default_factory=lambda: {"implementation": "cuBLAS"})


class FakeBackend:
    name = "fake"

    def __init__(self, *, compiled=None, checked=None, bench=None, fail_at=None, error=None):
        self.calls: list[str] = []
        self.compiled = compiled or Compiled()
        self.checked = checked or Checked()
        self.bench = bench or BenchmarkResult((50.0, 50.0), 50.0)
        self.fail_at, self.error = fail_at, error

    def _step(self, name):
        self.calls.append(name)
        if self.fail_at == name:
            raise self.error

    def normalize_program(self, program):
        self.calls.append("normalize")
        return program.source.strip()

    def compile(self, program, workload):
        self._step("compile")
        return self.compiled

    def check_correctness(self, artifact, workload):
        self._step("correctness")
        return self.checked

    def benchmark(self, artifact, workload):
        self._step("benchmark")
        return self.bench

    def binary_fingerprint(self, artifact, launch_config):
        self._step("fingerprint")
        return "binary-hash"

    def lightweight_profile(self, artifact, workload, metric_set="lightweight_v1"):
        return {"metric_set": metric_set}


def evaluate(backend, source="kernel"):
    evaluator = BackendKernelEvaluator(backend=backend, root_benchmark=ROOT, context=CONTEXT)
    return evaluator.evaluate(KernelProgram(source), BF16_GEMM_4096_B200)


def test_valid_evaluation_runs_stages_in_order_and_rewards_log_speedup():
    backend = FakeBackend()
    result = evaluate(backend)
    assert backend.calls == ["normalize", "compile", "correctness", "benchmark", "fingerprint"]
    assert result.status == ProposalStatus.VALID
    assert result.reward == pytest.approx(math.log(100.0 / 50.0))
    assert result.compile_status == CompileStatus.SUCCESS and result.correctness_status == CorrectnessStatus.PASS
    assert result.binary_hash == "binary-hash" and result.state_key and result.source_hash
    assert result.worker_id == "worker-0" and result.compiled_artifact.artifact_id == "artifact-1"


def test_compile_failure_stops_before_correctness():
    backend = FakeBackend(compiled=Compiled(success=False, artifact=None, stderr="error"))
    result = evaluate(backend)
    assert backend.calls == ["normalize", "compile"]
    assert result.status == ProposalStatus.INVALID and result.invalid_reason == InvalidReason.COMPILE_FAILURE
    assert result.compile_status == CompileStatus.FAIL


def test_compile_timeout_is_a_timeout():
    result = evaluate(FakeBackend(compiled=Compiled(success=False, artifact=None, timed_out=True)))
    assert result.invalid_reason == InvalidReason.TIMEOUT


def test_correctness_failure_stops_before_benchmark():
    backend = FakeBackend(checked=Checked(success=False, failed_test_id="fixed_shape"))
    result = evaluate(backend)
    assert "benchmark" not in backend.calls
    assert result.invalid_reason == InvalidReason.CORRECTNESS_FAILURE
    assert result.correctness_status == CorrectnessStatus.FAIL
    assert result.correctness.failed_test_id == "fixed_shape"


@pytest.mark.parametrize(
    "stage,error,reason",
    [
        ("correctness", CandidateLaunchError("x"), InvalidReason.LAUNCH_FAILURE),
        ("benchmark", CandidateTimeoutError("x"), InvalidReason.TIMEOUT),
        ("benchmark", CandidateBenchmarkError("x"), InvalidReason.BENCHMARK_FAILURE),
    ],
)
def test_candidate_errors_become_invalid_reasons(stage, error, reason):
    result = evaluate(FakeBackend(fail_at=stage, error=error))
    assert result.status == ProposalStatus.INVALID and result.invalid_reason == reason
    assert result.metadata["error_type"] == type(error).__name__


def test_infrastructure_errors_are_not_blamed_on_the_candidate():
    result = evaluate(FakeBackend(fail_at="benchmark", error=EvaluationInfrastructureError("gpu gone")))
    assert result.status == ProposalStatus.INFRASTRUCTURE_FAILURE and result.invalid_reason is None
    assert result.correctness_status == CorrectnessStatus.PASS


@pytest.mark.parametrize("timings", [(), (0.0,), (float("nan"),), (-1.0,)])
def test_invalid_timings_are_benchmark_failures(timings):
    bench = BenchmarkResult(timings, 1.0)
    result = evaluate(FakeBackend(bench=bench))
    assert result.invalid_reason == InvalidReason.BENCHMARK_FAILURE


def test_weighted_multi_shape_reward():
    workload = WorkloadContract("multi", "gemm", "bfloat16",
                                (ShapeCase({"M": 1, "N": 1, "K": 1}, 0.25), ShapeCase({"M": 2, "N": 2, "K": 2}, 0.75)),
                                0.02, 0.02)
    root = BenchmarkResult((1.0,), 1.0, {"K=1,M=1,N=1": 10.0, "K=2,M=2,N=2": 40.0})
    cand = BenchmarkResult((1.0,), 1.0, {"K=1,M=1,N=1": 5.0, "K=2,M=2,N=2": 10.0})
    assert root_normalized_reward(root, cand, workload) == pytest.approx(0.25 * math.log(2) + 0.75 * math.log(4))


def test_state_key_identity():
    key = state_key(binary_hash="b", workload=BF16_GEMM_4096_B200, context=CONTEXT)
    assert key == state_key(binary_hash="b", workload=BF16_GEMM_4096_B200, context=CONTEXT)
    assert key != state_key(binary_hash="c", workload=BF16_GEMM_4096_B200, context=CONTEXT)
    other = EvaluationContext("w", "m", {"block": [32, 8, 1]}, CONTEXT.hardware_toolchain)
    assert key != state_key(binary_hash="b", workload=BF16_GEMM_4096_B200, context=other)


def test_evaluation_round_trips_through_wire_json():
    result = evaluate(FakeBackend())
    wire = serialize_evaluation(result)
    assert set(wire) >= {"status", "program", "state_key", "reward", "benchmark", "invalid_reason", "compile_status",
                         "correctness_status", "worker_id", "environment_manifest_id", "source_hash", "binary_hash",
                         "launch_config", "compilation", "correctness", "metadata"}
    back = deserialize_evaluation(wire)
    assert back.status == result.status and back.reward == result.reward and back.state_key == result.state_key
    assert back.benchmark.median_us == result.benchmark.median_us


REFERENCE_SRC = Path("/root/reference/src")


@pytest.mark.skipif(not (REFERENCE_SRC / "kernel_mcts" / "evaluation.py").exists(),
                    reason="reference tree not present")
def test_backend_plugs_into_the_reference_evaluator(tmp_path):
    """The reference's own BackendKernelEvaluator drives CudaSm100Backend
    (fake runner, no GPU): the result objects carry the attributes it reads."""
    sys.path.insert(0, str(REFERENCE_SRC))
    try:
        from kernel_mcts import domain as ref_domain
        from kernel_mcts.evaluation import BackendKernelEvaluator as RefEvaluator
        from kernel_mcts.evaluation import EvaluationContext as RefContext
    finally:
        sys.path.remove(str(REFERENCE_SRC))
    from test_backend import FakeRunner, ROOT_SOURCE, make_backend

    backend = make_backend(tmp_path, FakeRunner())
    ref_workload = ref_domain.WorkloadContract(
        benchmark_id="bf16_gemm_4096_b200", operation="gemm", dtype="bfloat16",
        shapes=(ref_domain.ShapeCase({"M": 4096, "N": 4096, "K": 4096}, 1.0),), rtol=0.02, atol=0.02,
        metadata=dict(BF16_GEMM_4096_B200.metadata),
    )
    evaluator = RefEvaluator(backend=backend, root_benchmark=ref_domain.BenchmarkResult((100.0,), 100.0),
                             context=RefContext("w", "m", {}, {}))
    result = evaluator.evaluate(ref_domain.KernelProgram(ROOT_SOURCE), ref_workload)
    assert result.status.value == "VALID", result
    assert result.reward == pytest.approx(math.log(100.0 / 11.0))
