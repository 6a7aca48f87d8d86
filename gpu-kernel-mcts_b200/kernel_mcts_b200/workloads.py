"""Workload contracts for B200.

The schema is the reference's (src/kernel_mcts/benchmarks/bf16_gemm.py:8-45):
same operation, dtype, tolerances, tensor layouts and candidate ABI, so a
candidate written for the reference still evaluates.  New ids name the B200
target; ``launcher`` adds the host-launcher ABI that lets a candidate own its
grid, cluster and shared-memory launch (the reference notes the fixed 16x16
launch as a limitation, docs/local-autotuning.md:175-177).
"""

from __future__ import annotations

from .domain import KernelProgram, ShapeCase, WorkloadContract

_TENSORS_COL = {
    "A": {"shape": ["M", "K"], "layout": "row_major"},
    "B": {"shape": ["K", "N"], "layout": "column_major"},
    "C": {"shape": ["M", "N"], "layout": "row_major"},
}
_TENSORS_ROW = {
    "A": {"shape": ["M", "K"], "layout": "row_major"},
    "B": {"shape": ["K", "N"], "layout": "row_major"},
    "C": {"shape": ["M", "N"], "layout": "row_major"},
}
_ROOT_ABI = {
    "parameters": [
        "const __nv_bfloat16* A",
        "const __nv_bfloat16* B",
        "__nv_bfloat16* C",
        "int M",
        "int N",
        "int K",
    ],
    "launch": {
        "block": [16, 16, 1],
        "grid": ["ceil_div(N, 16)", "ceil_div(M, 16)", 1],
        "dynamic_shared_memory_bytes": 0,
    },
}
_LAUNCHER_ABI = {
    "symbol": "bf16_gemm_launch",
    "signature": 'extern "C" int bf16_gemm_launch(const void* A, const void* B, void* C, '
    "int M, int N, int K, cudaStream_t stream)",
    "returns": "0 on success",
}


def gemm_workload(
    benchmark_id: str,
    m: int,
    n: int,
    k: int,
    *,
    b_layout: str = "col",
    inputs: str = "uniform",
    rtol: float = 2.0e-2,
    atol: float = 2.0e-2,
) -> WorkloadContract:
    return multi_shape_gemm_workload(benchmark_id, [(m, n, k, 1.0)], b_layout=b_layout, inputs=inputs,
                                     rtol=rtol, atol=atol)


def multi_shape_gemm_workload(
    benchmark_id: str,
    shapes,
    *,
    b_layout: str = "col",
    inputs: str = "uniform",
    rtol: float = 2.0e-2,
    atol: float = 2.0e-2,
) -> WorkloadContract:
    """A GEMM workload over weighted shapes ``[(M, N, K, weight), ...]``
    (weights summing to 1): the reward weights log(T_root / T) per shape."""
    return WorkloadContract(
        benchmark_id=benchmark_id,
        operation="gemm",
        dtype="bfloat16",
        shapes=tuple(ShapeCase({"M": m, "N": n, "K": k}, float(w)) for m, n, k, w in shapes),
        rtol=rtol,
        atol=atol,
        metadata={
            "target": {"gpu_model": "B200", "form_factor": "SXM", "minimum_compute_capability": "10.0"},
            "entry_point": "bf16_gemm_root",
            "accumulation_dtype": "float32",
            "output_dtype": "bfloat16",
            "tensors": _TENSORS_COL if b_layout == "col" else _TENSORS_ROW,
            "abi": _ROOT_ABI,
            "launcher": _LAUNCHER_ABI,
            "inputs": inputs,
            "b_layout": b_layout,
        },
    )


#: The reference contract's shape on B200 (mt19937 U(-0.25, 0.25) inputs, column-major B).
BF16_GEMM_4096_B200 = gemm_workload("bf16_gemm_4096_b200", 4096, 4096, 4096)

#: BASELINE config 1: 256^3, N(0,1), A/B row-major.
BF16_GEMM_256_RANDN = gemm_workload("bf16_gemm_256_randn_b200", 256, 256, 256, b_layout="row", inputs="randn")
#: BASELINE config 2: 4096^3, N(0,1), A/B row-major.
BF16_GEMM_4096_RANDN = gemm_workload("bf16_gemm_4096_randn_b200", 4096, 4096, 4096, b_layout="row", inputs="randn")
#: BASELINE config 3: 4096^3 integers in {-2..2}: bit-exact expected.
BF16_GEMM_4096_INT = gemm_workload("bf16_gemm_4096_int_b200", 4096, 4096, 4096, b_layout="row", inputs="int")

#: A weighted mix of square and MLP-like shapes (N(0,1), A/B row-major).
BF16_GEMM_MIX_RANDN = multi_shape_gemm_workload(
    "bf16_gemm_mix_randn_b200",
    [(4096, 4096, 4096, 0.5), (8192, 3584, 8192, 0.25), (2048, 14336, 4096, 0.25)],
    b_layout="row", inputs="randn")

ALL_WORKLOADS = (BF16_GEMM_4096_B200, BF16_GEMM_256_RANDN, BF16_GEMM_4096_RANDN, BF16_GEMM_4096_INT,
                 BF16_GEMM_MIX_RANDN)


# The root program a worker calibrates against when no other is named: a
# host-launcher candidate running the library's CUDA-core kernel, which keeps
# the reference root's arithmetic (one FP32 accumulator per output, one FMA
# per k in order, src/kernel_mcts/benchmarks/kernels/bf16_gemm_root.cu:8-44).
SIMT_ROOT_LAUNCHER = r"""
#include <cuda_runtime.h>
#include "kmcts_gemm.h"
extern "C" int bf16_gemm_launch(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
    kmcts_gemm_config cfg;
    kmcts_default_config(&cfg);
    cfg.kernel = KMCTS_KERNEL_SIMT;
    return kmcts_bf16_gemm_ex(A, B, C, M, N, K, KMCTS_B_COL, &cfg, s, nullptr);
}
"""


def root_program(path: str | None = None) -> KernelProgram:
    """The worker's root program: the candidate source at ``path`` (for
    instance the reference's own bf16_gemm_root.cu), else the CUDA-core
    launcher above."""
    if path:
        with open(path, encoding="utf-8") as handle:
            return KernelProgram(handle.read(), "cuda_cpp")
    return KernelProgram(SIMT_ROOT_LAUNCHER, "cuda_cpp")
