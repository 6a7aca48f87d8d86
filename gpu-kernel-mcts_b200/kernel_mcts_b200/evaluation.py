"""Tier-0 evaluation: compile -> correctness -> benchmark -> reward -> state key.

The state machine, failure taxonomy and reward follow the reference
evaluator (src/kernel_mcts/evaluation.py:63-191 for the order and the
stop-on-failure rules, :25-38 for the exception classes, :222-237 for
benchmark validation, :240-259 for the root-normalised reward
log(T_root / T), :266-279 for the state key).  Any backend implementing the
KernelBackend protocol (src/kernel_mcts/backends.py:8-37) plugs in; the
sm_100a backend is :class:`kernel_mcts_b200.backend.CudaSm100Backend`.
"""

from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass
from typing import Any, Mapping, Protocol

from .domain import (
    BenchmarkResult,
    CompilationEvidence,
    CompileStatus,
    CorrectnessEvidence,
    CorrectnessStatus,
    EvaluationResult,
    InvalidReason,
    KernelProgram,
    ProposalStatus,
    WorkloadContract,
)
from .serialization import serialize_workload


class EvaluationInfrastructureError(RuntimeError):
    """A worker or tool failure unrelated to candidate validity."""


class CandidateBenchmarkError(RuntimeError):
    """A deterministic candidate launch or benchmark failure."""


class CandidateLaunchError(RuntimeError):
    """The compiled candidate could not launch successfully."""


class CandidateTimeoutError(RuntimeError):
    """A candidate exceeded a bounded compile or execution timeout."""


class KernelBackend(Protocol):
    name: str

    def normalize_program(self, program: KernelProgram) -> str: ...
    def compile(self, program: KernelProgram, workload: WorkloadContract) -> Any: ...
    def check_correctness(self, artifact: Any, workload: WorkloadContract) -> Any: ...
    def benchmark(self, artifact: Any, workload: WorkloadContract) -> BenchmarkResult: ...
    def lightweight_profile(self, artifact: Any, workload: WorkloadContract, metric_set: str = ...) -> Mapping[str, object]: ...
    def binary_fingerprint(self, artifact: Any, launch_config: Mapping[str, object]) -> str: ...


@dataclass(frozen=True, slots=True)
class EvaluationContext:
    worker_id: str
    environment_manifest_id: str
    launch_config: Mapping[str, object]
    hardware_toolchain: Mapping[str, object]


def _sha256_text(value: str) -> str:
    return hashlib.sha256(value.encode()).hexdigest()


def shape_key(dimensions: Mapping[str, int]) -> str:
    return ",".join(f"{name}={value}" for name, value in sorted(dimensions.items()))


def validate_benchmark(benchmark: BenchmarkResult, workload: WorkloadContract) -> None:
    timings = benchmark.timings_us
    if not timings or not all(math.isfinite(t) and t > 0 for t in timings):
        raise CandidateBenchmarkError("benchmark timings must be finite and positive")
    if not (math.isfinite(benchmark.median_us) and benchmark.median_us > 0):
        raise CandidateBenchmarkError("benchmark median must be finite and positive")
    if len(workload.shapes) > 1:
        for shape in workload.shapes:
            key = shape_key(shape.dimensions)
            value = benchmark.per_shape_median_us.get(key)
            if value is None or not math.isfinite(value) or value <= 0:
                raise CandidateBenchmarkError(f"missing valid timing for shape {key}")


def root_normalized_reward(root: BenchmarkResult, candidate: BenchmarkResult, workload: WorkloadContract) -> float:
    """log(T_root / T_candidate); weighted over shapes for multi-shape workloads."""
    if len(workload.shapes) == 1:
        if not (math.isfinite(root.median_us) and root.median_us > 0):
            raise ValueError("root benchmark median must be finite and positive")
        return math.log(root.median_us / candidate.median_us)
    total = 0.0
    for shape in workload.shapes:
        key = shape_key(shape.dimensions)
        root_time = root.per_shape_median_us.get(key)
        if root_time is None or not math.isfinite(root_time) or root_time <= 0:
            raise ValueError(f"missing valid root timing for shape {key}")
        total += shape.weight * math.log(root_time / candidate.per_shape_median_us[key])
    return total


def state_key(*, binary_hash: str, workload: WorkloadContract, context: EvaluationContext) -> str:
    identity = {
        "binary_hash": binary_hash,
        "workload": serialize_workload(workload),
        "launch_config": context.launch_config,
        "hardware_toolchain": context.hardware_toolchain,
    }
    return hashlib.sha256(json.dumps(identity, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


class BackendKernelEvaluator:
    """Runs compile, correctness and benchmark once for a candidate."""

    def __init__(self, *, backend: KernelBackend, root_benchmark: BenchmarkResult, context: EvaluationContext) -> None:
        self.backend = backend
        self.root_benchmark = root_benchmark
        self.context = context

    def evaluate(self, program: KernelProgram, workload: WorkloadContract) -> EvaluationResult:
        source_hash = _sha256_text(self.backend.normalize_program(program))
        stage: dict[str, Any] = {
            "compile_status": CompileStatus.NOT_ATTEMPTED,
            "correctness_status": CorrectnessStatus.NOT_TESTED,
            "compilation": None,
            "correctness": None,
            "artifact": None,
        }
        backend_metadata: dict[str, object] = {}

        def result(status: ProposalStatus, **values: Any) -> EvaluationResult:
            merged = {**stage, **values}
            artifact = merged.pop("artifact")
            return EvaluationResult(
                status=status,
                program=program,
                source_hash=source_hash,
                worker_id=self.context.worker_id,
                environment_manifest_id=self.context.environment_manifest_id,
                launch_config=self.context.launch_config,
                compiled_artifact=artifact,
                **merged,
            )

        try:
            compiled = self.backend.compile(program, workload)
            stage["compilation"] = CompilationEvidence(
                artifact_id=compiled.artifact.artifact_id if compiled.artifact else None,
                stdout=compiled.stdout,
                stderr=compiled.stderr,
                duration_seconds=getattr(compiled, "duration_seconds", None),
                artifact_paths=tuple(getattr(compiled, "artifact_paths", ())),
            )
            if not compiled.success or compiled.artifact is None:
                reason = InvalidReason.TIMEOUT if getattr(compiled, "timed_out", False) else InvalidReason.COMPILE_FAILURE
                return result(ProposalStatus.INVALID, invalid_reason=reason, compile_status=CompileStatus.FAIL)

            stage["artifact"] = compiled.artifact
            backend_metadata = self._backend_metadata(compiled.artifact)
            stage["compile_status"] = CompileStatus.SUCCESS
            checked = self.backend.check_correctness(compiled.artifact, workload)
            stage["correctness"] = CorrectnessEvidence(
                maximum_error=checked.maximum_error,
                mean_error=checked.mean_error,
                failed_test_id=getattr(checked, "failed_test_id", None),
                reference_metadata=getattr(checked, "reference_metadata", {}),
            )
            if not checked.success:
                return result(
                    ProposalStatus.INVALID,
                    invalid_reason=InvalidReason.CORRECTNESS_FAILURE,
                    correctness_status=CorrectnessStatus.FAIL,
                    metadata=backend_metadata,
                )

            stage["correctness_status"] = CorrectnessStatus.PASS
            benchmark = self.backend.benchmark(compiled.artifact, workload)
            validate_benchmark(benchmark, workload)
            reward = root_normalized_reward(self.root_benchmark, benchmark, workload)
            binary_hash = self.backend.binary_fingerprint(compiled.artifact, self.context.launch_config)
            metadata = dict(backend_metadata)
            compiler_context = getattr(compiled, "compiler_context", None)
            if compiler_context is not None:
                metadata["compiler_context"] = dict(compiler_context)
            return result(
                ProposalStatus.VALID,
                state_key=state_key(binary_hash=binary_hash, workload=workload, context=self.context),
                reward=reward,
                benchmark=benchmark,
                binary_hash=binary_hash,
                metadata=metadata,
            )
        except (CandidateBenchmarkError, CandidateLaunchError, CandidateTimeoutError) as error:
            if isinstance(error, CandidateLaunchError):
                reason = InvalidReason.LAUNCH_FAILURE
            elif isinstance(error, CandidateTimeoutError):
                reason = InvalidReason.TIMEOUT
            else:
                reason = InvalidReason.BENCHMARK_FAILURE
            return result(
                ProposalStatus.INVALID,
                invalid_reason=reason,
                metadata={**backend_metadata, "error_type": type(error).__name__},
            )
        except EvaluationInfrastructureError as error:
            return result(
                ProposalStatus.INFRASTRUCTURE_FAILURE,
                metadata={**backend_metadata, "error_type": type(error).__name__},
            )

    def prepare(self, workload: WorkloadContract) -> None:
        """Lets the backend build per-workload state (inputs, references) ahead
        of the evaluations that will be timed.  Optional for backends."""
        prepare = getattr(self.backend, "prepare", None)
        if callable(prepare):
            prepare(workload)

    def lightweight_profile(self, evaluation: EvaluationResult, workload: WorkloadContract,
                            metric_set: str = "lightweight_v1") -> Mapping[str, object]:
        if evaluation.status != ProposalStatus.VALID:
            raise ValueError("only valid evaluations can be profiled")
        if evaluation.compiled_artifact is None:
            raise EvaluationInfrastructureError("cached compiled artifact is unavailable for profiling")
        return self.backend.lightweight_profile(evaluation.compiled_artifact, workload, metric_set)

    def _backend_metadata(self, artifact: object) -> dict[str, object]:
        provider = getattr(self.backend, "evaluation_metadata", None)
        if not callable(provider):
            return {}
        value = provider(artifact)
        if not isinstance(value, Mapping):
            raise EvaluationInfrastructureError("backend evaluation metadata must be a mapping")
        return dict(value)
