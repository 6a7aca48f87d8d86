"""ctypes binding of libkmcts_gemm_sm100.so (C ABI in include/kmcts_gemm.h).

There is no fallback: if the library is missing or fails to load, every call
raises :class:`NativeLibraryError`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIBRARY

KMCTS_OK = 0
KMCTS_EHANDLE = 1
KMCTS_EGEMM = 2
KMCTS_ESYNC = 3
KMCTS_EINVAL = 4
KMCTS_ESMEM = 5
KMCTS_ETIMEOUT = 6
KMCTS_ENOTSUP = 7
KMCTS_ENOSCRATCH = 8

ERROR_NAMES = {
    KMCTS_OK: "ok",
    KMCTS_EHANDLE: "handle",
    KMCTS_EGEMM: "gemm_launch",
    KMCTS_ESYNC: "synchronize",
    KMCTS_EINVAL: "invalid_argument",
    KMCTS_ESMEM: "shared_memory",
    KMCTS_ETIMEOUT: "device_wait_timeout",
    KMCTS_ENOTSUP: "not_supported",
    KMCTS_ENOSCRATCH: "static_scratch_too_small",
}

B_COL = 0
B_ROW = 1

KERNEL_AUTO = 0
KERNEL_TCGEN05 = 1
KERNEL_SIMT = 2

FLAG_NO_TAIL_SPLIT = 1
FLAG_TAIL_SPLIT_N = 2
FLAG_TAIL_STREAM_K = 4
FLAG_TAIL_SPLIT_K = 32
FLAG_B_EVICT_FIRST = 8
FLAG_SWAP_AB = 16
FLAG_SPLIT_CLUSTER = 64
FLAG_A_EVICT_FIRST = 128
FLAG_SPLIT_SCATTER = 256

SPLIT_WORKSPACE, SPLIT_CLUSTER, SPLIT_SCATTER = 0, 1, 2

TAIL_NONE = 0
TAIL_SPLIT_N = 1
TAIL_STREAM_K = 2
TAIL_SPLIT_K = 3

INPUTS = {"uniform": 0, "randn": 1, "int": 2}

#: Every symbol include/kmcts_gemm.h declares.
EXPORTED_SYMBOLS = (
    "kmcts_default_config",
    "kmcts_select_config",
    "kmcts_bf16_gemm",
    "kmcts_bf16_gemm_ex",
    "kmcts_config_legal",
    "kmcts_config_smem_bytes",
    "kmcts_version",
    "kmcts_compare_workspace_bytes",
    "kmcts_bf16_compare",
    "kmcts_launch_count",
    "kmcts_time_gemm",
    "kmcts_bf16_gemm_host",
    "kmcts_gemm_plan_query",
    "kmcts_bf16_compare_noalloc",
    "kmcts_generate_inputs",
    "kmcts_ipc_export",
    "kmcts_ipc_import",
    "kmcts_ipc_close",
    "kmcts_copy_2d",
    "kmcts_bf16_gemm_allgather",
    "kmcts_selftest_bounded_wait",
)


class NativeLibraryError(RuntimeError):
    """The sm_100a library is not built or cannot be loaded."""


class KmctsError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, operation: str) -> None:
        self.code = code
        self.operation = operation
        super().__init__(f"{operation} failed: {ERROR_NAMES.get(code, code)} ({code})")


class GemmConfig(ctypes.Structure):
    """Mirror of ``kmcts_gemm_config``."""

    _fields_ = [
        ("tile_m", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("tile_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("cluster_m", ctypes.c_int32),
        ("cluster_n", ctypes.c_int32),
        ("persistent", ctypes.c_int32),
        ("raster_group", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("wait_limit_ns", ctypes.c_int64),
        ("k_splits", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]

    def as_dict(self) -> dict[str, int]:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class GemmPlan(ctypes.Structure):
    """Mirror of ``kmcts_gemm_plan``."""

    _fields_ = [
        ("kernel", ctypes.c_int32),
        ("ctas", ctypes.c_int32),
        ("cluster_size", ctypes.c_int32),
        ("workers", ctypes.c_int32),
        ("tiles", ctypes.c_int32),
        ("full_tiles", ctypes.c_int32),
        ("units", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("tail_split", ctypes.c_int32),
        ("tail_clusters", ctypes.c_int32),
        ("tail_segments", ctypes.c_int32),
        ("k_splits", ctypes.c_int32),
        ("split_reduce", ctypes.c_int32),
    ]

    def as_dict(self) -> dict[str, int]:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class CompareResult(ctypes.Structure):
    """Mirror of ``kmcts_compare_result``."""

    _fields_ = [
        ("maximum_error", ctypes.c_double),
        ("mean_error", ctypes.c_double),
        ("count", ctypes.c_int64),
        ("n_tolerance_fail", ctypes.c_int64),
        ("n_nonfinite", ctypes.c_int64),
        ("ulp_hist", ctypes.c_int64 * 4),
        ("max_ulp", ctypes.c_int32),
        ("success", ctypes.c_int32),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return LIBRARY


def load() -> ctypes.CDLL:
    """Loads (once) and returns the native library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIBRARY.exists():
            raise NativeLibraryError(
                f"{LIBRARY} is not built; run kernel_mcts_b200.build.build_all() (nvcc, sm_100a)"
            )
        try:
            lib = ctypes.CDLL(str(LIBRARY))
        except OSError as error:
            raise NativeLibraryError(f"cannot load {LIBRARY}: {error}") from error
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        lib.kmcts_default_config.argtypes = [ctypes.POINTER(GemmConfig)]
        lib.kmcts_default_config.restype = i32
        lib.kmcts_select_config.argtypes = [i32, i32, i32, i32, ctypes.POINTER(GemmConfig)]
        lib.kmcts_select_config.restype = i32
        lib.kmcts_bf16_gemm.argtypes = [vp, vp, vp, i32, i32, i32]
        lib.kmcts_bf16_gemm.restype = i32
        lib.kmcts_bf16_gemm_ex.argtypes = [
            vp, vp, vp, i32, i32, i32, i32, ctypes.POINTER(GemmConfig), vp, vp,
        ]
        lib.kmcts_bf16_gemm_ex.restype = i32
        lib.kmcts_config_legal.argtypes = [
            ctypes.POINTER(GemmConfig), i32, i32, i32, i32, ctypes.c_char_p, i32,
        ]
        lib.kmcts_config_legal.restype = i32
        lib.kmcts_config_smem_bytes.argtypes = [ctypes.POINTER(GemmConfig), i32]
        lib.kmcts_config_smem_bytes.restype = i64
        lib.kmcts_version.argtypes = []
        lib.kmcts_version.restype = ctypes.c_char_p
        lib.kmcts_compare_workspace_bytes.argtypes = []
        lib.kmcts_compare_workspace_bytes.restype = ctypes.c_size_t
        lib.kmcts_bf16_compare.argtypes = [
            vp, vp, i64, ctypes.c_double, ctypes.c_double, vp, vp, ctypes.POINTER(CompareResult),
        ]
        lib.kmcts_bf16_compare.restype = i32
        lib.kmcts_bf16_compare_noalloc.argtypes = [
            vp, vp, i64, ctypes.c_double, ctypes.c_double, vp, ctypes.POINTER(CompareResult),
        ]
        lib.kmcts_bf16_compare_noalloc.restype = i32
        lib.kmcts_gemm_plan_query.argtypes = [ctypes.POINTER(GemmConfig), i32, i32, i32, i32, ctypes.POINTER(GemmPlan)]
        lib.kmcts_gemm_plan_query.restype = i32
        lib.kmcts_generate_inputs.argtypes = [i32, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_size_t, vp, vp]
        lib.kmcts_generate_inputs.restype = i32
        lib.kmcts_ipc_export.argtypes = [vp, vp]
        lib.kmcts_ipc_export.restype = i32
        lib.kmcts_ipc_import.argtypes = [vp, ctypes.POINTER(ctypes.c_void_p)]
        lib.kmcts_ipc_import.restype = i32
        lib.kmcts_ipc_close.argtypes = [vp]
        lib.kmcts_ipc_close.restype = i32
        sz = ctypes.c_size_t
        lib.kmcts_copy_2d.argtypes = [vp, sz, vp, sz, sz, sz, vp]
        lib.kmcts_copy_2d.restype = i32
        lib.kmcts_bf16_gemm_allgather.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32,
                                                  ctypes.POINTER(GemmConfig), vp, vp]
        lib.kmcts_bf16_gemm_allgather.restype = i32
        lib.kmcts_selftest_bounded_wait.argtypes = [i64, i32, vp, vp, vp]
        lib.kmcts_selftest_bounded_wait.restype = i32
        lib.kmcts_launch_count.argtypes = []
        lib.kmcts_launch_count.restype = i64
        lib.kmcts_time_gemm.argtypes = [vp, vp, vp, i32, i32, i32, i32, ctypes.POINTER(GemmConfig), vp, vp, i32, i32,
                                        vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_float)]
        lib.kmcts_time_gemm.restype = i32
        lib.kmcts_bf16_gemm_host.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, ctypes.POINTER(GemmConfig),
                                             i32, vp, vp]
        lib.kmcts_bf16_gemm_host.restype = i32
        _lib = lib
        return lib


def default_config() -> GemmConfig:
    cfg = GemmConfig()
    check(load().kmcts_default_config(ctypes.byref(cfg)), "kmcts_default_config")
    return cfg


def select_config(m: int, n: int, k: int, b_layout: int = B_COL) -> GemmConfig:
    """The schedule a NULL config selects for this shape."""
    cfg = GemmConfig()
    check(load().kmcts_select_config(m, n, k, b_layout, ctypes.byref(cfg)), "kmcts_select_config")
    return cfg


def make_config(**overrides: int) -> GemmConfig:
    cfg = default_config()
    for name, value in overrides.items():
        if not hasattr(cfg, name):
            raise ValueError(f"unknown config field {name!r}")
        setattr(cfg, name, int(value))
    return cfg


def config_legal(cfg: GemmConfig, m: int, n: int, k: int, b_layout: int = B_COL) -> tuple[int, str]:
    why = ctypes.create_string_buffer(256)
    code = load().kmcts_config_legal(ctypes.byref(cfg), m, n, k, b_layout, why, len(why))
    return int(code), why.value.decode()


def config_smem_bytes(cfg: GemmConfig, b_layout: int = B_COL) -> int:
    return int(load().kmcts_config_smem_bytes(ctypes.byref(cfg), b_layout))


def plan(cfg: GemmConfig | None, m: int, n: int, k: int, b_layout: int = B_COL) -> dict[str, int]:
    """Launch shape of a schedule on the current CUDA device (no launch)."""
    out = GemmPlan()
    code = load().kmcts_gemm_plan_query(ctypes.byref(cfg) if cfg is not None else None, m, n, k, b_layout,
                                        ctypes.byref(out))
    check(code, "kmcts_gemm_plan_query")
    return out.as_dict()


def generate_inputs(kind: str, seed: int, a_count: int, b_count: int):
    """Evaluation inputs as two uint16 numpy arrays of BF16 bits (host)."""
    import numpy as np

    a = np.empty(a_count, dtype=np.uint16)
    b = np.empty(b_count, dtype=np.uint16)
    check(load().kmcts_generate_inputs(INPUTS[kind], seed, a_count, b_count, a.ctypes.data, b.ctypes.data),
          "kmcts_generate_inputs")
    return a, b


def version() -> str:
    return load().kmcts_version().decode()


def launch_count() -> int:
    return int(load().kmcts_launch_count())


def check(code: int, operation: str) -> None:
    if code != KMCTS_OK:
        raise KmctsError(int(code), operation)
