"""Failure detection on the GPU without a GPU fault: the bounded wait that
guards every GEMM barrier gives up on a flag nothing sets and reports
KMCTS_ETIMEOUT, and the context stays usable afterwards."""

from __future__ import annotations

import ctypes

import pytest
import torch

from kernel_mcts_b200 import _native
from kernel_mcts_b200 import gemm as kg
from oracle import oracle

pytestmark = pytest.mark.gpu


def probe(limit_ns: int, arrive: int) -> tuple[int, int]:
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    rc = _native.load().kmcts_selftest_bounded_wait(limit_ns, arrive, torch.cuda.current_stream().cuda_stream,
                                                    status.data_ptr(), waited.data_ptr())
    assert rc == _native.KMCTS_OK
    torch.cuda.synchronize()
    return int(status.item()), int(waited.item())


def test_wait_on_an_unset_flag_times_out_and_reports(cuda_device):
    status, waited = probe(limit_ns=50_000_000, arrive=0)  # 50 ms
    assert status & 0xFF == _native.KMCTS_ETIMEOUT and status >> 8 == 2
    assert 50_000_000 <= waited < 5_000_000_000


def test_completed_phase_returns_at_once(cuda_device):
    status, waited = probe(limit_ns=1_000_000_000, arrive=1)
    assert status == 0 and waited < 10_000_000


def test_context_stays_usable_after_a_timeout(cuda_device):
    probe(limit_ns=10_000_000, arrive=0)
    a_t, b_t = oracle.integer_inputs(256, 256, 256, seed=3)
    c = kg.bf16_gemm(a_t.cuda(), b_t.cuda())
    torch.cuda.synchronize()
    expect = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(b_t))
    assert (oracle.torch_bits(c) == expect).all()


def test_limits_are_validated(cuda_device):
    lib = _native.load()
    dummy = torch.zeros(2, dtype=torch.int64, device="cuda")
    assert lib.kmcts_selftest_bounded_wait(0, 0, None, dummy.data_ptr(), dummy.data_ptr()) == _native.KMCTS_EINVAL
    assert lib.kmcts_selftest_bounded_wait(20_000_000_000, 0, None, dummy.data_ptr(), dummy.data_ptr()) == \
        _native.KMCTS_EINVAL
