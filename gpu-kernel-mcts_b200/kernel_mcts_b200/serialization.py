"""JSON codecs for the evaluation contract.

The key names are the reference's wire format
(src/kernel_mcts/serialization.py:24-79 for evaluations, :111-123 for
workloads); workers and controllers exchange exactly these objects.
"""

from __future__ import annotations

from enum import Enum
from pathlib import Path
from typing import Any, Mapping

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
    ShapeCase,
    WorkloadContract,
)


def json_value(value: object) -> Any:
    """Converts enums, paths, mappings and sequences into plain JSON values."""
    if isinstance(value, Enum):
        return value.value
    if value is None or isinstance(value, (str, int, float, bool)):
        return value
    if isinstance(value, Path):
        return str(value)
    if isinstance(value, Mapping):
        return {str(k): json_value(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [json_value(v) for v in value]
    raise TypeError(f"value of type {type(value).__name__} is not JSON serializable")


def serialize_benchmark(benchmark: BenchmarkResult | None) -> dict[str, Any] | None:
    if benchmark is None:
        return None
    return {
        "timings_us": list(benchmark.timings_us),
        "median_us": benchmark.median_us,
        "per_shape_median_us": json_value(benchmark.per_shape_median_us),
        "warmup_count": benchmark.warmup_count,
        "mean_us": benchmark.mean_us,
        "stddev_us": benchmark.stddev_us,
        "min_us": benchmark.min_us,
        "max_us": benchmark.max_us,
        "gpu_operating_state": json_value(benchmark.gpu_operating_state),
    }


def serialize_program(program: KernelProgram | None) -> dict[str, str] | None:
    return None if program is None else {"source": program.source, "backend": program.backend}


def serialize_workload(workload: WorkloadContract) -> dict[str, Any]:
    return {
        "benchmark_id": workload.benchmark_id,
        "operation": workload.operation,
        "dtype": workload.dtype,
        "shapes": [{"dimensions": json_value(s.dimensions), "weight": s.weight} for s in workload.shapes],
        "rtol": workload.rtol,
        "atol": workload.atol,
        "metadata": json_value(workload.metadata),
    }


def deserialize_workload(value: Mapping[str, Any]) -> WorkloadContract:
    return WorkloadContract(
        benchmark_id=str(value["benchmark_id"]),
        operation=str(value["operation"]),
        dtype=str(value["dtype"]),
        shapes=tuple(
            ShapeCase({str(k): int(v) for k, v in s["dimensions"].items()}, float(s["weight"]))
            for s in value["shapes"]
        ),
        rtol=float(value["rtol"]),
        atol=float(value["atol"]),
        metadata=value.get("metadata", {}),
    )


def serialize_evaluation(evaluation: EvaluationResult) -> dict[str, Any]:
    compilation = evaluation.compilation
    correctness = evaluation.correctness
    return {
        "status": evaluation.status.value,
        "program": serialize_program(evaluation.program),
        "state_key": evaluation.state_key,
        "reward": evaluation.reward,
        "benchmark": serialize_benchmark(evaluation.benchmark),
        "invalid_reason": evaluation.invalid_reason.value if evaluation.invalid_reason else None,
        "compile_status": evaluation.compile_status.value,
        "correctness_status": evaluation.correctness_status.value,
        "worker_id": evaluation.worker_id,
        "environment_manifest_id": evaluation.environment_manifest_id,
        "source_hash": evaluation.source_hash,
        "binary_hash": evaluation.binary_hash,
        "launch_config": json_value(evaluation.launch_config),
        "compilation": None
        if compilation is None
        else {
            "artifact_id": compilation.artifact_id,
            "stdout": compilation.stdout,
            "stderr": compilation.stderr,
            "duration_seconds": compilation.duration_seconds,
            "artifact_paths": list(compilation.artifact_paths),
        },
        "correctness": None
        if correctness is None
        else {
            "maximum_error": correctness.maximum_error,
            "mean_error": correctness.mean_error,
            "failed_test_id": correctness.failed_test_id,
            "reference_metadata": json_value(correctness.reference_metadata),
        },
        "metadata": json_value(evaluation.metadata),
    }


def deserialize_evaluation(value: Mapping[str, Any]) -> EvaluationResult:
    program = value.get("program")
    bench = value.get("benchmark")
    comp = value.get("compilation")
    corr = value.get("correctness")
    reason = value.get("invalid_reason")
    return EvaluationResult(
        status=ProposalStatus(value["status"]),
        program=KernelProgram(str(program["source"]), str(program["backend"])) if isinstance(program, Mapping) else None,
        state_key=value.get("state_key"),
        reward=value.get("reward"),
        benchmark=BenchmarkResult(
            tuple(float(v) for v in bench["timings_us"]),
            float(bench["median_us"]),
            bench.get("per_shape_median_us", {}),
            bench.get("warmup_count"),
            bench.get("mean_us"),
            bench.get("stddev_us"),
            bench.get("min_us"),
            bench.get("max_us"),
            bench.get("gpu_operating_state", {}),
        )
        if isinstance(bench, Mapping)
        else None,
        invalid_reason=InvalidReason(reason) if reason else None,
        metadata=value.get("metadata", {}),
        compile_status=CompileStatus(value.get("compile_status", "NOT_ATTEMPTED")),
        correctness_status=CorrectnessStatus(value.get("correctness_status", "NOT_TESTED")),
        worker_id=value.get("worker_id"),
        environment_manifest_id=value.get("environment_manifest_id"),
        source_hash=value.get("source_hash"),
        binary_hash=value.get("binary_hash"),
        launch_config=value.get("launch_config", {}),
        compilation=CompilationEvidence(
            comp.get("artifact_id"),
            str(comp.get("stdout", "")),
            str(comp.get("stderr", "")),
            comp.get("duration_seconds"),
            tuple(comp.get("artifact_paths", ())),
        )
        if isinstance(comp, Mapping)
        else None,
        correctness=CorrectnessEvidence(
            corr.get("maximum_error"),
            corr.get("mean_error"),
            corr.get("failed_test_id"),
            corr.get("reference_metadata", {}),
        )
        if isinstance(corr, Mapping)
        else None,
    )
