"""CPU oracle for the BF16 GEMM hot path (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline / reference arm
of bench.py may import this module, and only as the checker or the timed CPU
baseline.  The product (kernel_mcts_b200) never imports it.

Pieces, each citing the reference behaviour it restates (paths relative to
the reference project):

* :func:`uniform_inputs` — the repository contract's input stream,
  ``bf16_gemm_harness.cu:92-95`` / ``bf16_input_generator.cu:23-37``
  (mt19937, U(-0.25, 0.25), RNE to BF16), from the C restatement in
  ``kmcts_oracle.c``.  Pinned against the reference's own compiled generator
  (tests/golden).
* :func:`root_gemm` — the root program's arithmetic, ``bf16_gemm_root.cu:8-44``
  (one FP32 accumulator per output, one FMA per k in order, RNE), in C.
  Pinned against the reference root kernel's outputs on a B200 (tests/golden).
* :func:`torch_reference` — the reference's CPU-runnable check,
  ``cute_independent_tma.py:1030-1032``:
  ``torch.matmul(a.float(), b.float().T).to(torch.bfloat16)``.
* :func:`harness_check` — the harness's acceptance test,
  ``bf16_gemm_harness.cu:154-164``.
* :func:`parity_report` — the ulp / error-bound criterion for N(0,1) inputs
  (FP32 sums in different orders may differ by more than one BF16 ulp near
  zero, so an element passes at <= 1 ulp OR within the forward-error bound
  ``0.5 ulp(ref64) + K * 2^-24 * (|A||B|)_ij`` of the FP64 product).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_LIB = ORACLE_DIR / "libkmcts_oracle.so"
REF_DIR = ORACLE_DIR / "_ref"
REF_GENERATOR = REF_DIR / "bf16_input_generator"
REF_ROOT_LIB = REF_DIR / "libref_root.so"
REF_CUBLAS_LIB = REF_DIR / "libkernel_mcts_bf16_reference.so"

_lib: ctypes.CDLL | None = None


def build(reference: bool = True) -> None:
    """Builds the oracle library (and the reference programs when their
    sources are present) with oracle/Makefile."""
    target = "all" if reference else "oracle"
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), target], check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            build(reference=False)
        lib = ctypes.CDLL(str(ORACLE_LIB))
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        lib.kmcts_oracle_uniform_inputs.argtypes = [ctypes.c_uint32, sz, sz, vp, vp]
        lib.kmcts_oracle_uniform_inputs.restype = None
        lib.kmcts_oracle_mt19937_words.argtypes = [ctypes.c_uint32, sz, vp]
        lib.kmcts_oracle_mt19937_words.restype = None
        lib.kmcts_oracle_gemm.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.kmcts_oracle_gemm.restype = ctypes.c_int
        lib.kmcts_oracle_check.argtypes = [vp, vp, sz, ctypes.c_double, ctypes.c_double, vp]
        lib.kmcts_oracle_check.restype = ctypes.c_int
        lib.kmcts_oracle_float_to_bf16.argtypes = [ctypes.c_float]
        lib.kmcts_oracle_float_to_bf16.restype = ctypes.c_uint16
        lib.kmcts_oracle_ulp_distance.argtypes = [ctypes.c_uint16, ctypes.c_uint16]
        lib.kmcts_oracle_ulp_distance.restype = ctypes.c_uint32
        _lib = lib
    return _lib


def _ptr(array: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(array.ctypes.data)


# ------------------------------------------------------------------ inputs


def uniform_inputs(m: int, n: int, k: int, seed: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """A then B from one mt19937(seed), U(-0.25, 0.25), as BF16 bits (uint16).

    A is ``[M, K]`` row-major; B is the contract's column-major ``[K, N]``,
    returned as its ``[N, K]`` row-major view (the flat order the reference
    writes it in).
    """
    a = np.empty(m * k, dtype=np.uint16)
    b = np.empty(k * n, dtype=np.uint16)
    load().kmcts_oracle_uniform_inputs(seed, a.size, b.size, _ptr(a), _ptr(b))
    return a.reshape(m, k), b.reshape(n, k)


def reference_generator_inputs(m: int, n: int, k: int, seed: int, workdir: Path) -> tuple[np.ndarray, np.ndarray]:
    """The same stream from the reference's own compiled generator
    (oracle/_ref/bf16_input_generator), for pinning."""
    a_path, b_path = workdir / "a.bf16", workdir / "b.bf16"
    subprocess.run([str(REF_GENERATOR), str(m), str(n), str(k), str(seed), str(a_path), str(b_path)], check=True)
    return (np.fromfile(a_path, dtype=np.uint16).reshape(m, k), np.fromfile(b_path, dtype=np.uint16).reshape(n, k))


def mt19937_words(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.uint32)
    load().kmcts_oracle_mt19937_words(seed, count, _ptr(out))
    return out


def randn_inputs(m: int, n: int, k: int, seed: int = 0, std: float = 1.0, b_layout: str = "col"):
    """N(0, std^2) inputs from a seeded CPU torch generator, cast to BF16
    (2 and 4).  Returns torch CPU tensors (A, B) with B as
    ``[N, K]`` for ``col`` or ``[K, N]`` for ``row``."""
    import torch

    g = torch.Generator().manual_seed(seed)
    a = torch.randn((m, k), generator=g, dtype=torch.float32)
    b = torch.randn((n, k) if b_layout == "col" else (k, n), generator=g, dtype=torch.float32)
    if std != 1.0:
        a, b = a * std, b * std
    return a.to(torch.bfloat16), b.to(torch.bfloat16)


def integer_inputs(m: int, n: int, k: int, seed: int = 0, low: int = -2, high: int = 2, b_layout: str = "col"):
    """Integers uniform in {low..high} as BF16: FP32
    accumulation of their products is exact while |sum| < 2^24."""
    import torch

    g = torch.Generator().manual_seed(seed)
    a = torch.randint(low, high + 1, (m, k), generator=g, dtype=torch.int32)
    b = torch.randint(low, high + 1, (n, k) if b_layout == "col" else (k, n), generator=g, dtype=torch.int32)
    return a.to(torch.bfloat16), b.to(torch.bfloat16)


# --------------------------------------------------------------- BF16 bits


def float_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Vectorised round-to-nearest-even float32 -> BF16 bits (canonical NaN)."""
    x = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    nan = ((x & 0x7F800000) == 0x7F800000) & ((x & 0x007FFFFF) != 0)
    rounded = ((x + (0x7FFF + ((x >> 16) & 1))) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FFF), rounded).astype(np.uint16)


def bf16_bits_to_float(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """BF16 ulps between bit patterns on the monotone line (+0 == -0);
    65535 where either is NaN."""
    a = np.asarray(a_bits, dtype=np.uint16).astype(np.int32)
    b = np.asarray(b_bits, dtype=np.uint16).astype(np.int32)

    def ordered(v):
        return np.where(v & 0x8000, -(v & 0x7FFF), v)

    d = np.abs(ordered(a) - ordered(b))
    nan = lambda v: ((v & 0x7F80) == 0x7F80) & ((v & 0x7F) != 0)  # noqa: E731
    return np.where(nan(a) | nan(b), 65535, d)


# -------------------------------------------------------------------- GEMM


def root_gemm(a_bits: np.ndarray, b_bits: np.ndarray, b_layout: str = "col") -> np.ndarray:
    """The root program's arithmetic on BF16 bit arrays.  ``b_bits`` is
    ``[N, K]`` for ``col`` or ``[K, N]`` for ``row``.  Returns C bits ``[M, N]``."""
    a = np.ascontiguousarray(a_bits, dtype=np.uint16)
    b = np.ascontiguousarray(b_bits, dtype=np.uint16)
    m, k = a.shape
    n = b.shape[0] if b_layout == "col" else b.shape[1]
    c = np.empty((m, n), dtype=np.uint16)
    rc = load().kmcts_oracle_gemm(_ptr(a), _ptr(b), _ptr(c), m, n, k, 0 if b_layout == "col" else 1)
    if rc != 0:
        raise RuntimeError(f"oracle GEMM failed ({rc})")
    return c


def torch_reference(a, b, b_layout: str = "col"):
    """``torch.matmul(a.float(), b.float().T).to(bfloat16)`` on the CPU
    (B as ``[N, K]``); for ``row`` B is ``[K, N]`` and is not transposed."""
    import torch

    a32 = a.float().cpu()
    b32 = b.float().cpu()
    prod = torch.matmul(a32, b32.T) if b_layout == "col" else torch.matmul(a32, b32)
    return prod.to(torch.bfloat16)


def fp64_reference(a, b, b_layout: str = "col"):
    """FP64 product (exact for BF16 inputs up to K ~ 2^37 terms' rounding) and
    the ``|A|·|B|`` magnitude, both as float64 numpy arrays."""
    import torch

    a64 = a.double().cpu()
    b64 = b.double().cpu()
    bt = b64.T if b_layout == "col" else b64
    return torch.matmul(a64, bt).numpy(), torch.matmul(a64.abs(), bt.abs()).numpy()


def torch_bits(t) -> np.ndarray:
    import torch

    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


# ------------------------------------------------------------------ checks


def harness_check(c_bits: np.ndarray, ref_bits: np.ndarray, rtol: float = 0.02, atol: float = 0.02) -> dict:
    """The reference harness's acceptance test, in C."""
    c = np.ascontiguousarray(c_bits, dtype=np.uint16).ravel()
    r = np.ascontiguousarray(ref_bits, dtype=np.uint16).ravel()
    out = np.zeros(2, dtype=np.float64)
    ok = load().kmcts_oracle_check(_ptr(c), _ptr(r), c.size, rtol, atol, _ptr(out))
    return {"success": bool(ok), "maximum_error": float(out[0]), "mean_error": float(out[1])}


def parity_report(c_bits: np.ndarray, ref32_bits: np.ndarray, ref64: np.ndarray, mag64: np.ndarray, k: int) -> dict:
    """Element passes if it is within 1 BF16 ulp of the FP32-accumulated
    oracle, or within ``0.5 ulp(ref64) + K*2^-24*|A||B|`` of the FP64 product.
    """
    c = np.asarray(c_bits, dtype=np.uint16)
    d = ulp_distance(c, ref32_bits)
    cf = bf16_bits_to_float(c).astype(np.float64)
    # ulp of BF16 at |ref64|: 2^(floor(log2|x|) - 7), floored at the subnormal step.
    mag = np.maximum(np.abs(ref64), np.finfo(np.float32).tiny)
    half_ulp = 0.5 * np.exp2(np.floor(np.log2(mag)) - 7)
    bound = half_ulp + k * 2.0 ** -24 * mag64
    within_bound = np.abs(cf - ref64) <= bound
    passed = (d <= 1) | within_bound
    big = np.abs(ref64) >= 2.0 ** -6
    return {
        "count": int(c.size),
        "max_ulp": int(d.max()) if d.size else 0,
        "max_ulp_where_ref_ge_2^-6": int(d[big].max()) if big.any() else 0,
        "max_ulp_where_ref_ge_0.5": int(d[np.abs(ref64) >= 0.5].max()) if (np.abs(ref64) >= 0.5).any() else 0,
        "n_gt_1ulp": int((d > 1).sum()),
        "n_fail_bound": int((~passed).sum()),
        "max_abs_error_vs_fp64": float(np.abs(cf - ref64).max()) if c.size else 0.0,
        "passed": bool(passed.all()),
    }
