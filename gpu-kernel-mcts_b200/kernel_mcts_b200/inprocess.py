"""In-process evaluation of prebuilt schedules, and the hybrid backend.

A schedule program (``KernelProgram(<schedule JSON>, "kmcts_sm100")``) needs no
compiler and no new executable, so evaluating it in a fresh harness process
spends seconds on process start, CUDA and cuBLAS initialisation and host input
generation for ~0.1 ms of GPU work.  :class:`InProcessSm100Backend` keeps one
CUDA context per worker and caches, per (shape, layout, inputs, seed), the
inputs and the cuBLAS reference on the device.  Each evaluation then runs:
* the schedule once and checks it against the reference with the device-side
  comparison, applying the harness's acceptance test;
* the harness's timing protocol: warm-ups, one synchronise, then one CUDA event
  pair per measured launch.

The inputs come from the same library generator the harness uses, so both
paths see identical bits.

:class:`HybridSm100Backend` sends schedule programs here and candidate
sources (``cuda_cpp``) to the compile-and-run :class:`CudaSm100Backend`.
"""

from __future__ import annotations

import hashlib
import json
import statistics
import time
from dataclasses import dataclass, field
from typing import Any, Mapping

from . import _native
from . import build as native_build
from .backend import (
    SCHEDULE_BACKEND,
    SCHEDULE_FIELDS,
    CudaSm100Backend,
    Sm100CompilationResult,
    Sm100CorrectnessResult,
    merge_benchmarks,
    merge_correctness,
    schedule_from_source,
    schedule_program,
    shape_mnk,
)
from .domain import BenchmarkResult, KernelProgram, WorkloadContract
from .evaluation import CandidateLaunchError, EvaluationInfrastructureError


@dataclass(frozen=True, slots=True)
class ScheduleArtifact:
    artifact_id: str
    schedule: Mapping[str, int] = field(default_factory=dict)
    abi: str = "schedule"


class InProcessSm100Backend:
    name = "cuda_sm100_inprocess"

    def __init__(self, *, warmup_count: int = 10, measurement_count: int = 30, seed: int = 0,
                 flush_l2: bool = False, device_index: int = 0) -> None:
        import torch

        if not torch.cuda.is_available():
            raise EvaluationInfrastructureError("no CUDA device for in-process evaluation")
        self.torch = torch
        # The caller's current device (a pool worker sees only its own GPU; a
        # torchrun rank has selected its GPU with torch.cuda.set_device).
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.warmup_count = warmup_count
        self.measurement_count = measurement_count
        self.seed = seed
        self.flush_l2 = flush_l2
        self.device_index = device_index
        self._cache: dict[tuple, tuple] = {}
        self._flush = None
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._workspace = torch.empty(int(_native.load().kmcts_compare_workspace_bytes()), dtype=torch.uint8,
                                      device=self.device)
        self._library_digest = hashlib.sha256(native_build.LIBRARY.read_bytes()).hexdigest()

    # ------------------------------------------------------------------ inputs

    def _operands(self, workload: WorkloadContract, dimensions=None):
        torch = self.torch
        m, n, k = shape_mnk(dimensions if dimensions is not None else workload.shapes[0].dimensions)
        layout = workload.metadata.get("b_layout", "col")
        inputs = workload.metadata.get("inputs", "uniform")
        key = (m, n, k, layout, inputs, self.seed)
        if key not in self._cache:
            if len(self._cache) >= len(workload.shapes):
                self._cache.clear()  # one workload's shapes resident at a time
            a_bits, b_bits = _native.generate_inputs(inputs, self.seed, m * k, k * n)
            a = torch.from_numpy(a_bits.view("int16")).view(torch.bfloat16).reshape(m, k).to(self.device)
            # The stream fills B in its storage order: [N, K] for column-major B.
            b_shape = (n, k) if layout == "col" else (k, n)
            b = torch.from_numpy(b_bits.view("int16")).view(torch.bfloat16).reshape(b_shape).to(self.device)
            previous = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
            try:
                reference = torch.matmul(a, b.T if layout == "col" else b)  # cuBLAS, FP32 accumulate
            finally:
                torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = previous
            c = torch.empty((m, n), dtype=torch.bfloat16, device=self.device)
            torch.cuda.synchronize(self.device)
            self._cache[key] = (a, b, c, reference, layout)
        return self._cache[key]

    def prepare(self, workload: WorkloadContract) -> None:
        for shape in workload.shapes:
            self._operands(workload, shape.dimensions)

    # -------------------------------------------------------------- protocol

    def normalize_program(self, program: KernelProgram) -> str:
        return json.dumps(schedule_from_source(program.source), sort_keys=True)

    def compile(self, program: KernelProgram, workload: WorkloadContract) -> Sm100CompilationResult:
        started = time.monotonic()
        if program.backend != SCHEDULE_BACKEND:
            raise ValueError("the in-process backend evaluates schedule programs only")
        schedule = schedule_from_source(program.source)
        layout = _native.B_ROW if workload.metadata.get("b_layout", "col") == "row" else _native.B_COL
        cfg = _native.make_config(**schedule, kernel=_native.KERNEL_TCGEN05)
        for shape in workload.shapes:
            code, why = _native.config_legal(cfg, *shape_mnk(shape.dimensions), layout)
            if code != _native.KMCTS_OK:
                return Sm100CompilationResult(False, None, "", f"statically rejected: {why}",
                                              time.monotonic() - started)
        resolved = cfg.as_dict()
        digest = hashlib.sha256((self._library_digest + json.dumps(resolved, sort_keys=True)).encode()).hexdigest()
        artifact = ScheduleArtifact(digest, resolved)
        return Sm100CompilationResult(True, artifact, "", "", time.monotonic() - started,
                                      compiler_context={"schedule": resolved,
                                                        "smem_bytes": _native.config_smem_bytes(cfg, layout)})

    def _prepared(self, artifact: ScheduleArtifact, workload: WorkloadContract, dimensions=None):
        from . import gemm as kg

        a, b, c, _, layout = self._operands(workload, dimensions)
        key = (id(c), artifact.artifact_id)
        if getattr(self, "_prepared_key", None) != key:
            self._prepared_gemm = kg.PreparedGemm(a, b, c, b_layout=layout,
                                                  config=_native.make_config(**artifact.schedule),
                                                  stream=self.torch.cuda.current_stream(self.device),
                                                  status=self._status)
            self._prepared_key = key
        return self._prepared_gemm

    def _launch(self, artifact: ScheduleArtifact, workload: WorkloadContract, dimensions=None):
        try:
            self._prepared(artifact, workload, dimensions).launch()
        except _native.KmctsError as error:
            raise CandidateLaunchError(str(error)) from error

    def _check_status(self) -> None:
        value = int(self._status.item())
        if value != 0:
            self._status.zero_()
            raise CandidateLaunchError(f"device-side wait gave up (status {value:#x})")

    def check_correctness(self, artifact: ScheduleArtifact, workload: WorkloadContract) -> Sm100CorrectnessResult:
        return merge_correctness(workload, [self._check_shape(artifact, workload, shape.dimensions)
                                            for shape in workload.shapes])

    def _check_shape(self, artifact: ScheduleArtifact, workload: WorkloadContract, dimensions) -> Sm100CorrectnessResult:
        from . import gemm as kg

        _, _, c, reference, _ = self._operands(workload, dimensions)
        self._launch(artifact, workload, dimensions)
        self.torch.cuda.synchronize(self.device)
        self._check_status()
        cmp = kg.compare(c, reference, rtol=workload.rtol, atol=workload.atol, workspace=self._workspace)
        stats = {"max_ulp": cmp.max_ulp, "n_gt_1ulp": cmp.ulp_hist[2] + cmp.ulp_hist[3],
                 "ulp_hist": list(cmp.ulp_hist), "n_nonfinite": cmp.n_nonfinite, "kernel": "library:in-process"}
        return Sm100CorrectnessResult(
            success=cmp.success, maximum_error=cmp.maximum_error, mean_error=cmp.mean_error,
            failed_test_id=None if cmp.success else "fixed_shape",
            reference_metadata={"implementation": "cuBLAS", "compute_type": "CUBLAS_COMPUTE_32F",
                                "seed": self.seed, **stats},
            statistics=stats,
        )

    def benchmark(self, artifact: ScheduleArtifact, workload: WorkloadContract) -> BenchmarkResult:
        return merge_benchmarks(workload, [self._benchmark_shape(artifact, workload, shape.dimensions)
                                           for shape in workload.shapes], {"status": "in-process"})

    def _benchmark_shape(self, artifact: ScheduleArtifact, workload: WorkloadContract, dimensions) -> BenchmarkResult:
        torch = self.torch
        if self.flush_l2 and self._flush is None:
            self._flush = torch.empty(512 << 20, dtype=torch.uint8, device=self.device)
        prepared = self._prepared(artifact, workload, dimensions)
        # The harness protocol, looped in the library: no interpreter work
        # between a start event and its launch.
        try:
            timings = prepared.time(self.warmup_count, self.measurement_count, self._flush)
        except _native.KmctsError as error:
            if error.code == _native.KMCTS_ETIMEOUT:
                self._status.zero_()
                raise CandidateLaunchError(f"device-side wait gave up ({error})") from error
            raise CandidateLaunchError(str(error)) from error
        return BenchmarkResult(
            timings_us=tuple(timings), median_us=statistics.median(timings), warmup_count=self.warmup_count,
            mean_us=statistics.fmean(timings), stddev_us=statistics.pstdev(timings), min_us=min(timings),
            max_us=max(timings), gpu_operating_state={"status": "in-process"},
        )

    def binary_fingerprint(self, artifact: ScheduleArtifact, launch_config: Mapping[str, object]) -> str:
        return artifact.artifact_id

    def evaluation_metadata(self, artifact: ScheduleArtifact) -> Mapping[str, object]:
        return {"backend": self.name, "architecture": "sm_100a", "abi": "schedule", "schedule": dict(artifact.schedule)}

    def lightweight_profile(self, artifact, workload, metric_set="lightweight_v1"):
        raise EvaluationInfrastructureError("profile schedule programs through CudaSm100Backend (ncu on the harness)")


class HybridSm100Backend:
    """Schedules in process; candidate sources through nvcc and the harness."""

    name = "cuda_sm100"

    def __init__(self, subprocess_backend: CudaSm100Backend, inprocess_backend: Any | None) -> None:
        self.subprocess_backend = subprocess_backend
        self.inprocess_backend = inprocess_backend

    def _for_program(self, program: KernelProgram):
        if program.backend == SCHEDULE_BACKEND and self.inprocess_backend is not None:
            return self.inprocess_backend
        return self.subprocess_backend

    def _for_artifact(self, artifact: Any):
        if isinstance(artifact, ScheduleArtifact) and self.inprocess_backend is not None:
            return self.inprocess_backend
        return self.subprocess_backend

    def prepare(self, workload):
        if self.inprocess_backend is not None:
            self.inprocess_backend.prepare(workload)

    def normalize_program(self, program):
        return self._for_program(program).normalize_program(program)

    def compile(self, program, workload):
        return self._for_program(program).compile(program, workload)

    def check_correctness(self, artifact, workload):
        return self._for_artifact(artifact).check_correctness(artifact, workload)

    def benchmark(self, artifact, workload):
        return self._for_artifact(artifact).benchmark(artifact, workload)

    def binary_fingerprint(self, artifact, launch_config):
        return self._for_artifact(artifact).binary_fingerprint(artifact, launch_config)

    def evaluation_metadata(self, artifact):
        return self._for_artifact(artifact).evaluation_metadata(artifact)

    def lightweight_profile(self, artifact, workload, metric_set="lightweight_v1"):
        # A schedule evaluated in process is profiled as the same schedule run
        # by the harness executable under ncu (one kernel, one launch).
        if isinstance(artifact, ScheduleArtifact):
            schedule = {k: v for k, v in artifact.schedule.items() if k in SCHEDULE_FIELDS}
            compiled = self.subprocess_backend.compile(schedule_program(**schedule), workload)
            if not compiled.success or compiled.artifact is None:
                raise EvaluationInfrastructureError("the schedule could not be prepared for profiling: "
                                                    + compiled.stderr[-2000:])
            artifact = compiled.artifact
        return self.subprocess_backend.lightweight_profile(artifact, workload, metric_set)
