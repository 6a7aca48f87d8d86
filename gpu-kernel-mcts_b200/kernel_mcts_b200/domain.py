"""Evaluation-contract data types.

This module restates the reference's domain types
(src/kernel_mcts/domain.py:8-135, serialised by serialization.py:24-79): the
same enums and frozen dataclasses, field for field, with the same validation.
They are the wire contract that the MCTS, sequential, autotune and profiling
callers read, so names, values and field order are kept as the reference has
them; only the layout of the source differs.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import StrEnum
from typing import Any, Mapping


class ProposalStatus(StrEnum):
    VALID = "VALID"
    INVALID = "INVALID"
    INFRASTRUCTURE_FAILURE = "INFRASTRUCTURE_FAILURE"


class InvalidReason(StrEnum):
    COMPILE_FAILURE = "COMPILE_FAILURE"
    LAUNCH_FAILURE = "LAUNCH_FAILURE"
    CORRECTNESS_FAILURE = "CORRECTNESS_FAILURE"
    TIMEOUT = "TIMEOUT"
    BENCHMARK_FAILURE = "BENCHMARK_FAILURE"
    OTHER = "OTHER"


class CompileStatus(StrEnum):
    NOT_ATTEMPTED = "NOT_ATTEMPTED"
    SUCCESS = "SUCCESS"
    FAIL = "FAIL"


class CorrectnessStatus(StrEnum):
    NOT_TESTED = "NOT_TESTED"
    PASS = "PASS"
    FAIL = "FAIL"


@dataclass(frozen=True, slots=True)
class ShapeCase:
    dimensions: Mapping[str, int]
    weight: float


@dataclass(frozen=True, slots=True)
class WorkloadContract:
    """One benchmark: operation, dtype, weighted shapes and tolerances."""

    benchmark_id: str
    operation: str
    dtype: str
    shapes: tuple[ShapeCase, ...]
    rtol: float
    atol: float
    metadata: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not self.shapes:
            raise ValueError("workload must contain at least one benchmark shape")
        if any(shape.weight <= 0 for shape in self.shapes):
            raise ValueError("shape weights must be positive")
        total = sum(shape.weight for shape in self.shapes)
        if abs(total - 1.0) > 1e-9:
            raise ValueError(f"shape weights must sum to 1, got {total}")


@dataclass(frozen=True, slots=True)
class Strategy:
    """A search strategy: an id, a description and one prompt per backend."""

    id: str
    description: str
    prompts: Mapping[str, str]

    def prompt_for(self, backend: str) -> str:
        try:
            return self.prompts[backend]
        except KeyError as error:
            raise ValueError(f"strategy {self.id!r} has no prompt for {backend!r}") from error


@dataclass(frozen=True, slots=True)
class KernelProgram:
    source: str
    backend: str = "cuda_cpp"


@dataclass(frozen=True, slots=True)
class BenchmarkResult:
    timings_us: tuple[float, ...]
    median_us: float
    per_shape_median_us: Mapping[str, float] = field(default_factory=dict)
    warmup_count: int | None = None
    mean_us: float | None = None
    stddev_us: float | None = None
    min_us: float | None = None
    max_us: float | None = None
    gpu_operating_state: Mapping[str, Any] = field(default_factory=dict)


@dataclass(frozen=True, slots=True)
class CompilationEvidence:
    artifact_id: str | None
    stdout: str
    stderr: str
    duration_seconds: float | None = None
    artifact_paths: tuple[str, ...] = ()


@dataclass(frozen=True, slots=True)
class CorrectnessEvidence:
    maximum_error: float | None
    mean_error: float | None
    failed_test_id: str | None = None
    reference_metadata: Mapping[str, Any] = field(default_factory=dict)


@dataclass(frozen=True, slots=True)
class EvaluationResult:
    """The result of evaluating one candidate program on one workload."""

    status: ProposalStatus
    program: KernelProgram | None = None
    state_key: str | None = None
    reward: float | None = None
    benchmark: BenchmarkResult | None = None
    invalid_reason: InvalidReason | None = None
    metadata: Mapping[str, Any] = field(default_factory=dict)
    compile_status: CompileStatus = CompileStatus.NOT_ATTEMPTED
    correctness_status: CorrectnessStatus = CorrectnessStatus.NOT_TESTED
    worker_id: str | None = None
    environment_manifest_id: str | None = None
    source_hash: str | None = None
    binary_hash: str | None = None
    launch_config: Mapping[str, Any] = field(default_factory=dict)
    compiled_artifact: Any | None = field(default=None, repr=False, compare=False)
    compilation: CompilationEvidence | None = None
    correctness: CorrectnessEvidence | None = None

    def __post_init__(self) -> None:
        if self.status == ProposalStatus.VALID:
            if self.program is None or self.state_key is None or self.reward is None:
                raise ValueError("valid evaluations require program, state_key, and reward")
        elif self.status == ProposalStatus.INVALID and self.invalid_reason is None:
            raise ValueError("invalid evaluations require an invalid_reason")
