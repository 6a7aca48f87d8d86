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


from reference_tree import REFERENCE_SRC  # noqa: E402


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


def test_reference_sequential_loop_runs_on_the_b200_backend(tmp_path):
    """The reference's own sequential refinement loop
    (src/kernel_mcts/sequential.py:77-288) runs unchanged with its own
    BackendKernelEvaluator over CudaSm100Backend (fake runner: no GPU, no
    nvcc, no ncu) and a scripted generator: it evaluates, profiles and
    accepts candidates, and the best node is the fastest one."""
    if not REFERENCE_SRC.exists():
        pytest.skip("reference source tree not present")
    sys.path.insert(0, str(REFERENCE_SRC))
    try:
        from kernel_mcts import domain as ref_domain
        from kernel_mcts.evaluation import BackendKernelEvaluator as RefEvaluator
        from kernel_mcts.evaluation import EvaluationContext as RefContext
        from kernel_mcts.generation import GenerationResult
        from kernel_mcts.sequential import SequentialConfig, run_sequential_loop
    except Exception as error:  # the reference needs packages this image may lack
        pytest.skip(f"reference sequential loop not importable: {error}")
    finally:
        sys.path.remove(str(REFERENCE_SRC))
    import json

    from kernel_mcts_b200.profiling import resolve_metric_set
    from test_backend import FakeRunner, LAUNCHER_SOURCE, ROOT_SOURCE, make_backend

    class Runner(FakeRunner):
        """Compiles each candidate into distinct executable bytes (its source)."""

        def __call__(self, command, *, timeout, env):
            out = super().__call__(command, timeout=timeout, env=env)
            command = list(command)
            if "-o" in command and command[0].endswith("nvcc"):
                # Compile: the object is the source; link: the executable is the object.
                inputs = [c for c in command if Path(c).name.startswith("candidate.") and c.endswith((".cu", ".o"))]
                if inputs:
                    Path(command[command.index("-o") + 1]).write_bytes(Path(inputs[0]).read_bytes())
            return out

    runner = Runner()
    metrics = resolve_metric_set("lightweight_v1", "sm_100a").metrics
    runner.ncu_stdout = "\n".join(['"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"'] +
                                  [f'"0","bf16_gemm_launch","{m}","u","{i + 1}"' for i, m in enumerate(metrics)])
    backend = make_backend(tmp_path, runner)
    # The root times 11 us; each candidate the generator proposes is faster.
    speeds = iter([11.0, 8.0, 6.0, 5.0])
    real_execute = backend._execute

    def execute(artifact, workload, mode, dimensions=None):
        if mode == "benchmark" and "candidate" in " ".join(artifact.extra_args):
            t = next(speeds, 5.0)
            runner.benchmark_stdout = json.dumps({"status": "ok", "timings_us": [t, t, t]})
        return real_execute(artifact, workload, mode, dimensions)

    backend._execute = execute
    ref_workload = ref_domain.WorkloadContract(
        benchmark_id="bf16_gemm_4096_b200", operation="gemm", dtype="bfloat16",
        shapes=(ref_domain.ShapeCase({"M": 4096, "N": 4096, "K": 4096}, 1.0),), rtol=0.02, atol=0.02,
        metadata=dict(BF16_GEMM_4096_B200.metadata),
    )
    evaluator = RefEvaluator(backend=backend, root_benchmark=ref_domain.BenchmarkResult((11.0,), 11.0),
                             context=RefContext("w", "m", {}, {}))
    root = evaluator.evaluate(ref_domain.KernelProgram(ROOT_SOURCE), ref_workload)
    assert root.status.value == "VALID", root

    class Generator:
        def __init__(self):
            self.calls = 0

        def generate(self, request):
            self.calls += 1
            source = LAUNCHER_SOURCE + f"\nstatic const int kCandidate = {self.calls};\n"
            return GenerationResult(f"g{self.calls}", source, ref_domain.KernelProgram(source), f"h{self.calls}")

    class Trace:
        def __init__(self):
            self.events = []

        def emit(self, kind, payload):
            self.events.append(kind)

        def start_run(self, *args, **kwargs):
            pass

        def store_compiler_artifact(self, sha256, content):
            pass

        def get_node_dataflow(self, node_id):
            return None

    trace = Trace()
    result = run_sequential_loop(
        root_evaluation=root, workload=ref_workload, hardware={"gpu": "B200"}, generator=Generator(),
        evaluator=evaluator, profiler=evaluator, trace=trace, generation_budget=3,
        config=SequentialConfig(compiler_detail="none", dataflow_view="none"),
    )
    assert result.generations == 3 and result.accepted_depth >= 1
    assert result.best.evaluation.benchmark.median_us == 5.0
    assert result.profile_calls >= 2  # the root and accepted candidates were profiled through ncu
    assert trace.events[0] == "run_started" and trace.events[-1] == "run_completed"
    assert "new_global_best" in trace.events


def _reference_search_setup(tmp_path):
    """The reference's evaluator over CudaSm100Backend with a fake runner whose
    candidates get faster one by one, plus a scripted generator."""
    sys.path.insert(0, str(REFERENCE_SRC))
    try:
        from kernel_mcts import domain as ref_domain
        from kernel_mcts.evaluation import BackendKernelEvaluator as RefEvaluator
        from kernel_mcts.evaluation import EvaluationContext as RefContext
        from kernel_mcts.generation import GenerationResult
    finally:
        sys.path.remove(str(REFERENCE_SRC))
    import json

    from kernel_mcts_b200.profiling import resolve_metric_set
    from test_backend import FakeRunner, LAUNCHER_SOURCE, ROOT_SOURCE, make_backend

    class Runner(FakeRunner):
        def __call__(self, command, *, timeout, env):
            out = super().__call__(command, timeout=timeout, env=env)
            command = list(command)
            if "-o" in command and command[0].endswith("nvcc"):
                # Compile: the object is the source; link: the executable is the object.
                inputs = [c for c in command if Path(c).name.startswith("candidate.") and c.endswith((".cu", ".o"))]
                if inputs:
                    Path(command[command.index("-o") + 1]).write_bytes(Path(inputs[0]).read_bytes())
            return out

    runner = Runner()
    metrics = resolve_metric_set("lightweight_v1", "sm_100a").metrics
    runner.ncu_stdout = "\n".join(['"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"'] +
                                   [f'"0","bf16_gemm_launch","{m}","u","{i + 1}"' for i, m in enumerate(metrics)])
    backend = make_backend(tmp_path, runner)
    times = iter([11.0] + [10.0 - 0.5 * i for i in range(40)])
    real_execute = backend._execute

    def execute(artifact, workload, mode, dimensions=None):
        if mode == "benchmark":
            t = next(times)
            runner.benchmark_stdout = json.dumps({"status": "ok", "timings_us": [t, t, t]})
        return real_execute(artifact, workload, mode, dimensions)

    backend._execute = execute
    workload = ref_domain.WorkloadContract(
        benchmark_id="bf16_gemm_4096_b200", operation="gemm", dtype="bfloat16",
        shapes=(ref_domain.ShapeCase({"M": 4096, "N": 4096, "K": 4096}, 1.0),), rtol=0.02, atol=0.02,
        metadata=dict(BF16_GEMM_4096_B200.metadata),
    )
    evaluator = RefEvaluator(backend=backend, root_benchmark=ref_domain.BenchmarkResult((11.0,), 11.0),
                             context=RefContext("w", "m", {}, {}))
    root = evaluator.evaluate(ref_domain.KernelProgram(ROOT_SOURCE), workload)

    class Generator:
        def __init__(self):
            self.calls = 0

        def generate(self, request):
            self.calls += 1
            source = LAUNCHER_SOURCE + f"\nstatic const int kCandidate = {self.calls};\n"
            return GenerationResult(f"g{self.calls}", source, ref_domain.KernelProgram(source), f"h{self.calls}")

    return ref_domain, evaluator, root, workload, Generator()


def test_reference_mcts_runs_on_the_b200_backend_with_pool_drift_probes(tmp_path):
    """The reference's MCTS (src/kernel_mcts/search/mcts.py) runs unchanged over
    its own evaluator on CudaSm100Backend, with PoolDriftMonitor (here over the
    same evaluator) as its measurement-drift probe."""
    if not REFERENCE_SRC.exists():
        pytest.skip("reference source tree not present")
    try:
        ref_domain, evaluator, root, workload, generator = _reference_search_setup(tmp_path)
        sys.path.insert(0, str(REFERENCE_SRC))
        from kernel_mcts.budget import GenerationBudget
        from kernel_mcts.search.mcts import MCTS, MCTSConfig
    except Exception as error:  # the reference needs packages this image may lack
        pytest.skip(f"reference MCTS not importable: {error}")
    finally:
        if str(REFERENCE_SRC) in sys.path:
            sys.path.remove(str(REFERENCE_SRC))
    from kernel_mcts_b200.autotune import PoolDriftMonitor

    class UniformPriors:
        name = "uniform"
        counts_toward_b_prior = False

        def get_priors(self, program, workload, strategies, profile):
            return {s.id: 1.0 / len(strategies) for s in strategies}

    strategies = [ref_domain.Strategy(f"s{i}", f"strategy {i}", {"cuda_cpp": f"try {i}"}) for i in range(3)]
    drift = PoolDriftMonitor(evaluator)
    search = MCTS(strategies=strategies, workload=workload, generator=generator, evaluator=evaluator,
                  prior_provider=UniformPriors(), budget=GenerationBudget(5), hardware={"gpu": "B200"},
                  config=MCTSConfig(measurement_drift_interval=1), seed=1, profiler=evaluator,
                  drift_monitor=drift)
    assert root.status.value == "VALID"
    result = search.run(root)
    assert result.best.reward > root.reward  # a faster candidate was found and kept
    assert generator.calls == 5 and drift.calls == result.drift_probe_calls >= 1
