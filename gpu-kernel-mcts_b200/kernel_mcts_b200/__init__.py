"""kernel_mcts_b200: the B200-native (sm_100a) BF16 GEMM hot path of kernel_mcts.

The GEMM, its correctness check and its timing protocol run in hand-written
CUDA (libkmcts_gemm_sm100.so, C ABI in include/kmcts_gemm.h); Python only
allocates device memory and wires the reference's evaluation contract on top.
"""

from ._native import (
    B_COL,
    B_ROW,
    GemmConfig,
    KmctsError,
    NativeLibraryError,
    config_legal,
    config_smem_bytes,
    default_config,
    launch_count,
    make_config,
    select_config,
    version,
)

__all__ = [
    "B_COL",
    "B_ROW",
    "GemmConfig",
    "KmctsError",
    "NativeLibraryError",
    "config_legal",
    "config_smem_bytes",
    "default_config",
    "launch_count",
    "make_config",
    "select_config",
    "version",
]
