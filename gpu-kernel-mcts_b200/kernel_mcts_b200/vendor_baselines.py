"""Vendor baselines (cuBLAS and CUTLASS columns) under the evaluation protocol.

Same report shape as the reference suite (src/kernel_mcts/vendor_baselines.py:54-59,
96-148): ``{"cublas": {"correctness": {...}, "benchmark": BenchmarkResult},
"cutlass": {...}}``, measured by the same harness, flags, warm-ups and
CUDA-event loop as every candidate.  The cuBLAS column is the reference's
``cublasGemmEx`` call (COMPUTE_32F); the CUTLASS column is the reference's
fixed Sm80 128x128x32 template, built from the CUTLASS headers vendored in
this image.  Where a column cannot run (no CUTLASS headers, a row-major B for
the column-major template) it is reported as unavailable instead of failing
the whole suite, as the reference would.
"""

from __future__ import annotations

import hashlib
from typing import Mapping

from . import build as native_build
from .backend import CudaSm100Backend, Sm100Artifact
from .domain import WorkloadContract
from .evaluation import (
    CandidateBenchmarkError,
    CandidateLaunchError,
    CandidateTimeoutError,
    EvaluationInfrastructureError,
)

VENDOR_IMPLEMENTATIONS = (("cublas", "cublas"), ("cutlass", "cutlass_sm80"))


class VendorBaselineSuite:
    """Fixed cuBLAS and CUTLASS references outside the search state space."""

    def __init__(self, backend: CudaSm100Backend) -> None:
        self.backend = backend

    def artifact(self, kernel: str) -> Sm100Artifact:
        harness = native_build.build_harness()
        digest = hashlib.sha256(harness.read_bytes() + kernel.encode()).hexdigest()
        return Sm100Artifact(digest, harness, (f"--kernel={kernel}",), f"vendor:{kernel}")

    def run(self, workload: WorkloadContract) -> dict[str, Mapping[str, object]]:
        results: dict[str, Mapping[str, object]] = {}
        for name, kernel in VENDOR_IMPLEMENTATIONS:
            artifact = self.artifact(kernel)
            try:
                checked = self.backend.check_correctness(artifact, workload)
                bench = self.backend.benchmark(artifact, workload)
            except (EvaluationInfrastructureError, CandidateLaunchError, CandidateBenchmarkError,
                    CandidateTimeoutError) as error:
                results[name] = {"status": "unavailable", "reason": f"{type(error).__name__}: {error}"}
                continue
            results[name] = {
                "correctness": {
                    "success": bool(checked.success),
                    "maximum_error": checked.maximum_error,
                    "mean_error": checked.mean_error,
                },
                "benchmark": bench,
            }
        return results
