"""Known-answer tests of the sm_100a kernels (through the C ABI).

Each case has an answer that needs no reference implementation: identity and
permutation matrices, rank-1 integer outer products, an all-zero B, exact
round-to-nearest-even ties, short and ragged K, and non-finite inputs (which
the device compare must flag, as the reference harness does at
src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:163).  Every case runs
on the default CTA-pair schedule and on the 1-CTA schedule, in both B layouts.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kernel_mcts_b200 import _native
from kernel_mcts_b200 import gemm as kg
from oracle import oracle

pytestmark = pytest.mark.gpu

SCHEDULES = {
    "pair": dict(kernel=_native.KERNEL_TCGEN05),
    "one_cta": dict(kernel=_native.KERNEL_TCGEN05, tile_m=128, cluster_m=1, tile_n=256, tile_k=64, stages=4),
    "pair_whole": dict(kernel=_native.KERNEL_TCGEN05, flags=_native.FLAG_NO_TAIL_SPLIT),
}


def gemm(a: torch.Tensor, b_kn: torch.Tensor, layout: str, schedule: str) -> torch.Tensor:
    """C = A @ B for A [M,K] and B given as [K,N]; passed in `layout`."""
    b = b_kn.T.contiguous() if layout == "col" else b_kn.contiguous()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = kg.bf16_gemm(a.cuda().contiguous(), b.cuda(), b_layout=layout,
                     config=_native.make_config(**SCHEDULES[schedule]), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return c.cpu()


def bits(t: torch.Tensor) -> np.ndarray:
    return oracle.torch_bits(t)


CASES = [(layout, schedule) for layout in ("col", "row") for schedule in SCHEDULES]


@pytest.mark.parametrize("layout,schedule", CASES)
def test_identity_returns_b_exactly(cuda_device, layout, schedule):
    n = 384
    g = torch.Generator().manual_seed(1)
    b = torch.randn((n, 520), generator=g).to(torch.bfloat16)
    c = gemm(torch.eye(n).to(torch.bfloat16), b, layout, schedule)
    np.testing.assert_array_equal(bits(c), bits(b))


@pytest.mark.parametrize("layout,schedule", CASES)
def test_permutation_permutes_rows_exactly(cuda_device, layout, schedule):
    n = 512
    g = torch.Generator().manual_seed(2)
    perm = torch.randperm(n, generator=g)
    p = torch.zeros((n, n))
    p[torch.arange(n), perm] = 1.0
    b = torch.randn((n, 264), generator=g).to(torch.bfloat16)
    c = gemm(p.to(torch.bfloat16), b, layout, schedule)
    np.testing.assert_array_equal(bits(c), bits(b[perm]))


@pytest.mark.parametrize("layout,schedule", CASES)
def test_rank_one_integer_outer_product(cuda_device, layout, schedule):
    m, n, k = 300, 272, 16
    g = torch.Generator().manual_seed(3)
    u = torch.randint(-64, 65, (m,), generator=g).float()
    v = torch.randint(-64, 65, (n,), generator=g).float()
    a = torch.zeros((m, k))
    b = torch.zeros((k, n))
    a[:, 5] = u  # one non-zero K column: C = u v^T, exact in FP32, rounded once to BF16
    b[5, :] = v
    c = gemm(a.to(torch.bfloat16), b.to(torch.bfloat16), layout, schedule)
    expect = torch.outer(u, v).to(torch.bfloat16)  # exact FP32 product, one RNE rounding
    # Compared as values: a zero output is the sum of zero products, whose sign
    # (+0 from -0 + +0) the single outer product does not model.
    np.testing.assert_array_equal(c.float().numpy(), expect.float().numpy())
    assert (bits(c)[c.float().numpy() != 0] == bits(expect)[c.float().numpy() != 0]).all()


@pytest.mark.parametrize("layout,schedule", CASES)
def test_all_zero_b_gives_zero(cuda_device, layout, schedule):
    g = torch.Generator().manual_seed(4)
    a = torch.randn((256, 512), generator=g).to(torch.bfloat16)
    c = gemm(a, torch.zeros((512, 256), dtype=torch.bfloat16), layout, schedule)
    assert torch.all(c.float() == 0.0)


@pytest.mark.parametrize("layout,schedule", CASES)
def test_round_to_nearest_even_ties(cuda_device, layout, schedule):
    """Each output is 1 + j * 2^-8 for j = 0..255, summed exactly in FP32 from
    two products.  Odd j sit exactly halfway between BF16 neighbours (spacing
    2^-7 in [1, 2)) and must round to the even mantissa."""
    m, n, k = 256, 256, 16
    a = torch.zeros((m, k))
    b = torch.zeros((k, n))
    a[:, 0] = 1.0
    b[0, :] = 1.0
    j = torch.arange(m, dtype=torch.float32)
    a[:, 1] = j * 2.0 ** -8  # exact in BF16 for j < 256 (at most 8 significant bits)
    b[1, :] = 1.0
    c = gemm(a.to(torch.bfloat16), b.to(torch.bfloat16), layout, schedule)
    exact = (1.0 + j.double() * 2.0 ** -8).numpy()
    want = oracle.float_to_bf16_bits(exact.astype(np.float32))  # RNE of the exact FP32 value
    got = bits(c)
    for col in (0, 17, 255):
        np.testing.assert_array_equal(got[:, col], want)
    # and the ties really went to even: 1 + 2^-8 -> 1.0, 1 + 3*2^-8 -> 1 + 2^-6
    assert float(c[1, 0]) == 1.0 and float(c[3, 0]) == 1.0 + 2.0 ** -6


@pytest.mark.parametrize("layout,schedule", CASES)
@pytest.mark.parametrize("k", [8, 16, 24, 64, 72, 136, 200])
def test_short_and_ragged_k_integer_exact(cuda_device, layout, schedule, k):
    m, n = 136, 264  # ragged against every tile
    a, b_nk = oracle.integer_inputs(m, n, k, seed=k)
    expect = oracle.root_gemm(bits(a), bits(b_nk))
    c = gemm(a, b_nk.T, layout, schedule)
    np.testing.assert_array_equal(bits(c), expect)


@pytest.mark.parametrize("layout,schedule", CASES)
def test_non_finite_inputs_propagate_and_fail_the_check(cuda_device, layout, schedule):
    g = torch.Generator().manual_seed(5)
    a = torch.randn((256, 256), generator=g)
    b = torch.randn((256, 256), generator=g)
    a[3, 7] = float("nan")
    a[10, 0] = float("inf")
    c = gemm(a.to(torch.bfloat16), b.to(torch.bfloat16), layout, schedule)
    assert torch.isnan(c[3]).all()  # NaN times anything finite is NaN
    assert not torch.isfinite(c[10]).any()  # inf times non-zero finite is +-inf (or NaN)
    assert torch.isfinite(c[[0, 1, 2, 4, 100]]).all()
    ref = torch.matmul(a.nan_to_num(0.0, 0.0, 0.0), b).to(torch.bfloat16)
    cmp = kg.compare(c.cuda(), ref.cuda())
    assert not cmp.success and cmp.n_nonfinite >= 2 * 256


def test_reference_stream_256_agrees_with_cublas_and_the_oracle(cuda_device):
    """BASELINE config 1 on the reference's own generator (mt19937 seed 0,
    U(-0.25, 0.25)): the kernel, the CPU oracle and cuBLAS agree within the
    parity criterion, and the kernel matches the oracle's harness check."""
    a_bits, b_bits = oracle.uniform_inputs(256, 256, 256, 0)
    a = torch.from_numpy(a_bits.view(np.int16)).view(torch.bfloat16)
    b_nk = torch.from_numpy(b_bits.view(np.int16)).view(torch.bfloat16)
    root = oracle.root_gemm(a_bits, b_bits)
    ref64, mag = oracle.fp64_reference(a, b_nk)
    cublas = bits(torch.matmul(a.cuda(), b_nk.cuda().T))
    assert oracle.parity_report(cublas, root, ref64, mag, 256)["passed"]
    for layout, schedule in CASES:
        got = bits(gemm(a, b_nk.T, layout, schedule))
        assert oracle.harness_check(got, root)["success"]
        assert oracle.parity_report(got, root, ref64, mag, 256)["passed"]
        assert oracle.parity_report(got, cublas, ref64, mag, 256)["passed"]
