"""Torch-facing calls into the sm_100a GEMM library.

Layouts follow the reference workload contract
(src/kernel_mcts/benchmarks/bf16_gemm.py:24-28): A is ``[M, K]`` row-major; B is
``[K, N]`` column-major, which as a torch tensor is ``b_nk`` of shape
``[N, K]`` (row-major, K contiguous); C is ``[M, N]`` row-major.  The
``b_layout="row"`` variant takes B as a row-major ``[K, N]`` tensor instead.

Torch only allocates and carries device pointers and streams here; every
FLOP runs in libkmcts_gemm_sm100.so.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native
from ._native import B_COL, B_ROW, GemmConfig, KmctsError

_LAYOUTS = {"col": B_COL, "row": B_ROW}


def layout_code(b_layout: str | int) -> int:
    if isinstance(b_layout, int):
        if b_layout not in (B_COL, B_ROW):
            raise ValueError(f"unknown B layout {b_layout!r}")
        return b_layout
    try:
        return _LAYOUTS[b_layout]
    except KeyError as error:
        raise ValueError(f"unknown B layout {b_layout!r}; use 'col' or 'row'") from error


def _check_operand(name: str, tensor: torch.Tensor, shape: tuple[int, int]) -> None:
    if tensor.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {tensor.dtype}")
    if not tensor.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if tuple(tensor.shape) != shape:
        raise ValueError(f"{name} must have shape {shape}, got {tuple(tensor.shape)}")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def gemm_shapes(a: torch.Tensor, b: torch.Tensor, b_layout: int) -> tuple[int, int, int]:
    m, k = a.shape
    if b_layout == B_COL:
        n, kb = b.shape
    else:
        kb, n = b.shape
    if kb != k:
        raise ValueError(f"inner dimensions differ: A has K={k}, B has K={kb}")
    return int(m), int(n), int(k)


def bf16_gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    b_layout: str | int = "col",
    config: GemmConfig | None = None,
    stream: torch.cuda.Stream | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """C = A·B on the current CUDA device, asynchronously on ``stream``.

    ``status`` (optional) is a device ``int32`` tensor of one element that the
    kernel sets non-zero if a bounded device-side wait gives up.
    """
    code = layout_code(b_layout)
    m, n, k = gemm_shapes(a, b, code)
    _check_operand("A", a, (m, k))
    _check_operand("B", b, (n, k) if code == B_COL else (k, n))
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    else:
        _check_operand("C", out, (m, n))
    if stream is None:
        stream = torch.cuda.current_stream(a.device)
    status_ptr = None
    if status is not None:
        if status.dtype != torch.int32 or not status.is_cuda or status.numel() < 1:
            raise ValueError("status must be a CUDA int32 tensor with at least one element")
        status_ptr = status.data_ptr()
    lib = _native.load()
    rc = lib.kmcts_bf16_gemm_ex(
        a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, code,
        ctypes.byref(config) if config is not None else None,
        stream.cuda_stream, status_ptr,
    )
    _native.check(rc, "kmcts_bf16_gemm_ex")
    return out


class PreparedGemm:
    """A GEMM whose operands, schedule and stream are fixed: the ctypes
    arguments are built once, so each ``launch()`` costs one C call.  For
    timed loops, where host overhead between a start event and the launch
    would be counted as kernel time."""

    def __init__(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *, b_layout: str | int = "col",
                 config: GemmConfig | None = None, stream: torch.cuda.Stream | None = None,
                 status: torch.Tensor | None = None) -> None:
        code = layout_code(b_layout)
        m, n, k = gemm_shapes(a, b, code)
        _check_operand("A", a, (m, k))
        _check_operand("B", b, (n, k) if code == B_COL else (k, n))
        _check_operand("C", out, (m, n))
        if status is not None and (status.dtype != torch.int32 or not status.is_cuda):
            raise ValueError("status must be a CUDA int32 tensor")
        self._keep = (a, b, out, status)  # operands stay alive while prepared
        self.config = config if config is not None else _native.default_config()
        stream = stream if stream is not None else torch.cuda.current_stream(a.device)
        self._fn = _native.load().kmcts_bf16_gemm_ex
        self._args = (
            ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            m, n, k, code, ctypes.byref(self.config), ctypes.c_void_p(stream.cuda_stream),
            ctypes.c_void_p(status.data_ptr()) if status is not None else None,
        )

    def launch(self) -> None:
        rc = self._fn(*self._args)
        if rc != 0:
            _native.check(rc, "kmcts_bf16_gemm_ex")

    def time(self, warmups: int, measurements: int, flush: torch.Tensor | None = None) -> list[float]:
        """The reference harness's benchmark protocol, run by the library:
        warm-ups, one synchronise, then one event pair and synchronise per
        launch (``kmcts_time_gemm``).  Needs a status tensor.  Returns µs."""
        if self._args[-1] is None:
            raise ValueError("timing needs a status tensor")
        out = (ctypes.c_float * measurements)()
        flush_args = (ctypes.c_void_p(flush.data_ptr()), flush.numel() * flush.element_size()) if flush is not None \
            else (None, 0)
        rc = _native.load().kmcts_time_gemm(*self._args, warmups, measurements, *flush_args, out)
        _native.check(rc, "kmcts_time_gemm")
        return [float(v) for v in out]


def bf16_gemm_host(
    a_host: torch.Tensor,
    b_host: torch.Tensor,
    c_host: torch.Tensor,
    a_dev: torch.Tensor,
    b_dev: torch.Tensor,
    c_dev: torch.Tensor,
    *,
    b_layout: str | int = "col",
    config: GemmConfig | None = None,
    chunks: int = 0,
    stream: torch.cuda.Stream | None = None,
    status: torch.Tensor | None = None,
) -> None:
    """C = A·B with A, B, C in (pinned) host tensors, through the caller's
    device tensors of the same shapes; copies and GEMM blocks overlap
    (``kmcts_bf16_gemm_host``).  Asynchronous on ``stream``."""
    code = layout_code(b_layout)
    m, n, k = gemm_shapes(a_host, b_host, code)
    for name, t in (("A", a_host), ("B", b_host), ("C", c_host)):
        if t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} host tensor must be a contiguous bfloat16 CPU tensor")
    if tuple(c_host.shape) != (m, n):
        raise ValueError(f"C must have shape {(m, n)}")
    _check_operand("A", a_dev, (m, k))
    _check_operand("B", b_dev, (n, k) if code == B_COL else (k, n))
    _check_operand("C", c_dev, (m, n))
    if stream is None:
        stream = torch.cuda.current_stream(a_dev.device)
    rc = _native.load().kmcts_bf16_gemm_host(
        a_host.data_ptr(), b_host.data_ptr(), c_host.data_ptr(), a_dev.data_ptr(), b_dev.data_ptr(),
        c_dev.data_ptr(), m, n, k, code, ctypes.byref(config) if config is not None else None, chunks,
        stream.cuda_stream, status.data_ptr() if status is not None else None)
    _native.check(rc, "kmcts_bf16_gemm_host")


def bf16_gemm_sync(a: torch.Tensor, b_nk: torch.Tensor, out: torch.Tensor) -> int:
    """The drop-in entry point (column-major B, default stream, synchronising).

    Returns the C status code exactly as ``kernel_mcts_bf16_reference`` does.
    """
    m, n, k = gemm_shapes(a, b_nk, B_COL)
    return int(_native.load().kmcts_bf16_gemm(a.data_ptr(), b_nk.data_ptr(), out.data_ptr(), m, n, k))


@dataclass(frozen=True)
class Comparison:
    success: bool
    maximum_error: float
    mean_error: float
    count: int
    n_tolerance_fail: int
    n_nonfinite: int
    ulp_hist: tuple[int, int, int, int]
    max_ulp: int

    def as_dict(self) -> dict[str, object]:
        return {
            "success": self.success,
            "maximum_error": self.maximum_error,
            "mean_error": self.mean_error,
            "count": self.count,
            "n_tolerance_fail": self.n_tolerance_fail,
            "n_nonfinite": self.n_nonfinite,
            "ulp_hist": list(self.ulp_hist),
            "max_ulp": self.max_ulp,
            "n_gt_1ulp": self.ulp_hist[2] + self.ulp_hist[3],
        }


def compare(
    c: torch.Tensor,
    reference: torch.Tensor,
    *,
    rtol: float = 2.0e-2,
    atol: float = 2.0e-2,
    workspace: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> Comparison:
    """Device-side error statistics of ``c`` against ``reference`` (both BF16)."""
    if c.dtype != torch.bfloat16 or reference.dtype != torch.bfloat16:
        raise TypeError("compare takes two bfloat16 tensors")
    if c.shape != reference.shape or not c.is_cuda or not reference.is_cuda:
        raise ValueError("compare takes two CUDA tensors of one shape")
    if not c.is_contiguous() or not reference.is_contiguous():
        raise ValueError("compare takes contiguous tensors")
    lib = _native.load()
    nbytes = int(lib.kmcts_compare_workspace_bytes())
    if workspace is None:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=c.device)
    elif workspace.numel() * workspace.element_size() < nbytes or not workspace.is_cuda:
        raise ValueError(f"workspace must be a CUDA buffer of at least {nbytes} bytes")
    if stream is None:
        stream = torch.cuda.current_stream(c.device)
    result = _native.CompareResult()
    rc = lib.kmcts_bf16_compare(
        c.data_ptr(), reference.data_ptr(), c.numel(), float(rtol), float(atol),
        workspace.data_ptr(), stream.cuda_stream, ctypes.byref(result),
    )
    _native.check(rc, "kmcts_bf16_compare")
    return Comparison(
        success=bool(result.success),
        maximum_error=float(result.maximum_error),
        mean_error=float(result.mean_error),
        count=int(result.count),
        n_tolerance_fail=int(result.n_tolerance_fail),
        n_nonfinite=int(result.n_nonfinite),
        ulp_hist=tuple(int(v) for v in result.ulp_hist),
        max_ulp=int(result.max_ulp),
    )


__all__ = [
    "B_COL",
    "B_ROW",
    "Comparison",
    "GemmConfig",
    "KmctsError",
    "PreparedGemm",
    "bf16_gemm",
    "bf16_gemm_host",
    "bf16_gemm_sync",
    "compare",
    "gemm_shapes",
    "layout_code",
]
