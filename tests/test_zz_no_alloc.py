"""The allocation-free comparison entry point, kmcts_bf16_compare_noalloc.

It exists for callers that cannot allocate device memory when they check a
result: a worker whose device memory all belongs to another allocator that
must account for every byte, or a host application that embeds the library
and hands it only the tensors it passes in.  Its scratch is a static device
array inside the library instead of a workspace the caller passes.  This file
is named so pytest collects it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from kernel_mcts_b200 import _native
from kernel_mcts_b200 import gemm as kg
from oracle import oracle

pytestmark = pytest.mark.gpu


def _noalloc(c: torch.Tensor, ref: torch.Tensor, rtol: float, atol: float) -> _native.CompareResult:
    out = _native.CompareResult()
    rc = _native.load().kmcts_bf16_compare_noalloc(
        c.data_ptr(), ref.data_ptr(), c.numel(), rtol, atol,
        torch.cuda.current_stream().cuda_stream, ctypes.byref(out),
    )
    assert rc == _native.KMCTS_OK, rc
    return out


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def test_noalloc_compare_matches_workspace_compare_on_two_calls(cuda_device):
    # Two calls in a row on different data: the second must not see the first's
    # accumulators (the entry point zeroes what it reuses).
    cases = []
    a, b = oracle.uniform_inputs(192, 160, 96, 4)
    c = oracle.root_gemm(a, b)
    ref = c.copy()
    ref.ravel()[::53] ^= np.uint16(0x0005)
    cases.append((c, ref))
    a2, b2 = oracle.uniform_inputs(64, 300, 40, 9)
    c2 = oracle.root_gemm(a2, b2)
    ref2 = c2.copy()
    ref2.ravel()[7] = oracle.float_to_bf16_bits(np.array([2.0], np.float32))[0]
    cases.append((c2, ref2))
    for c_bits, ref_bits in cases:
        dc, dr = _bf16(c_bits), _bf16(ref_bits)
        expect = kg.compare(dc, dr, rtol=0.02, atol=0.02)  # the workspace entry point
        got = _noalloc(dc, dr, 0.02, 0.02)
        assert bool(got.success) == expect.success
        assert got.maximum_error == expect.maximum_error
        assert got.mean_error == pytest.approx(expect.mean_error, rel=1e-12, abs=0.0)
        assert got.count == expect.count
        assert got.n_tolerance_fail == expect.n_tolerance_fail
        assert got.n_nonfinite == expect.n_nonfinite
        assert tuple(got.ulp_hist) == expect.ulp_hist
        assert got.max_ulp == expect.max_ulp
        # And against the CPU restatement of the reference harness's check.
        host = oracle.harness_check(c_bits, ref_bits, rtol=0.02, atol=0.02)
        assert bool(got.success) == host["success"]
        assert got.maximum_error == pytest.approx(host["maximum_error"], rel=1e-12, abs=0.0)
        assert got.mean_error == pytest.approx(host["mean_error"], rel=1e-9, abs=0.0)


def test_noalloc_compare_rejects_bad_arguments(cuda_device):
    t = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    out = _native.CompareResult()
    rc = _native.load().kmcts_bf16_compare_noalloc(t.data_ptr(), t.data_ptr(), -1, 0.02, 0.02, None,
                                                   ctypes.byref(out))
    assert rc == _native.KMCTS_EINVAL
