"""Parity of the sm_100a GEMM (through the C ABI) with the CPU oracle.

Bars (written into the asserts below):
* integer-valued inputs: bit-exact against the oracle (FP32 sums are exact);
* the SIMT kernel: bit-exact against the root-order oracle for any input;
* N(0,1) / U(-0.25,0.25) inputs on the tcgen05 kernel: every element within
  1 BF16 ulp of the FP32-accumulated oracle, or within
  0.5 ulp(ref64) + K*2^-24*(|A||B|)_ij of the FP64 product.
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


def to_cuda(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def bits_of(t: torch.Tensor) -> np.ndarray:
    return oracle.torch_bits(t)


def run(a, b, layout="col", **cfg):
    config = _native.make_config(**cfg) if cfg else None
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    c = kg.bf16_gemm(a, b, b_layout=layout, config=config, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item()):#x}"
    return c


def b_for(layout: str, b_nk: torch.Tensor) -> torch.Tensor:
    return b_nk if layout == "col" else b_nk.T.contiguous()


# ---------------------------------------------------------------- oracle pin


def test_reference_root_kernel_matches_cpu_oracle(cuda_device):
    """The reference's own root kernel (built from its source for sm_100a)
    and the C oracle agree bit for bit: the oracle restates it exactly."""
    if not oracle.REF_ROOT_LIB.exists():
        pytest.skip("oracle/_ref/libref_root.so not built")
    lib = ctypes.CDLL(str(oracle.REF_ROOT_LIB))
    lib.kmcts_ref_root_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    for m, n, k, seed in [(37, 29, 53, 7), (128, 96, 256, 0), (256, 256, 256, 0)]:
        a, b = oracle.uniform_inputs(m, n, k, seed)
        da, db = to_cuda(a), to_cuda(b)
        dc = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        assert lib.kmcts_ref_root_gemm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k) == 0
        np.testing.assert_array_equal(bits_of(dc), oracle.root_gemm(a, b))


# ---------------------------------------------------------------- SIMT path


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape", [(37, 29, 53), (64, 64, 64), (130, 70, 301)])
def test_simt_kernel_bit_exact_with_root_order(cuda_device, layout, shape):
    m, n, k = shape
    a, b = oracle.uniform_inputs(m, n, k, 1)
    c = run(to_cuda(a), b_for(layout, to_cuda(b)), layout, kernel=_native.KERNEL_SIMT)
    np.testing.assert_array_equal(bits_of(c), oracle.root_gemm(a, b))


# ------------------------------------------------------------- tcgen05 path


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize(
    "shape", [(128, 256, 64), (256, 256, 256), (300, 264, 200), (1024, 768, 512), (64, 8, 8)]
)
def test_tcgen05_integer_inputs_bit_exact(cuda_device, layout, shape):
    m, n, k = shape
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=0)
    expect = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, kernel=_native.KERNEL_TCGEN05)  # default: pair
    np.testing.assert_array_equal(bits_of(c), expect)
    c1 = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, kernel=_native.KERNEL_TCGEN05, tile_m=128,
             cluster_m=1, tile_n=256, tile_k=64, stages=4)
    np.testing.assert_array_equal(bits_of(c1), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
def test_tcgen05_uniform_inputs_within_criterion(cuda_device, layout):
    m, n, k = 512, 384, 1024
    a, b = oracle.uniform_inputs(m, n, k, 0)
    c = run(to_cuda(a), b_for(layout, to_cuda(b)), layout, kernel=_native.KERNEL_TCGEN05)
    a_t = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    b_t = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)
    ref64, mag = oracle.fp64_reference(a_t, b_t)
    report = oracle.parity_report(bits_of(c), oracle.root_gemm(a, b), ref64, mag, k)
    assert report["passed"], report
    assert oracle.harness_check(bits_of(c), oracle.root_gemm(a, b))["success"]


VARIANTS = [
    (256, 64, 3), (256, 64, 4), (128, 64, 3), (128, 64, 4), (128, 64, 5), (128, 64, 6),
    (128, 128, 3), (256, 128, 2), (192, 64, 4), (64, 64, 6),
]


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_n,tile_k,stages", VARIANTS)
@pytest.mark.parametrize("persistent", [1, 0])
def test_every_one_cta_schedule_bit_exact(cuda_device, layout, tile_n, tile_k, stages, persistent):
    """tile_m 128 = one CTA per tile (tcgen05.mma.cta_group::1)."""
    m, n, k = 392, 520, 328  # ragged against every tile size
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=7)
    expect = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, kernel=_native.KERNEL_TCGEN05, tile_m=128,
            cluster_m=1, tile_n=tile_n, tile_k=tile_k, stages=stages, persistent=persistent, raster_group=3)
    np.testing.assert_array_equal(bits_of(c), expect)


PAIR_VARIANTS = [
    (256, 64, 3), (256, 64, 4), (256, 64, 5), (256, 64, 6), (256, 128, 3),
    (128, 64, 3), (128, 64, 4), (128, 64, 5), (128, 64, 6), (128, 128, 3), (128, 128, 4),
]


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_n,tile_k,stages", PAIR_VARIANTS)
@pytest.mark.parametrize("persistent", [1, 0])
def test_every_cta_pair_schedule_bit_exact(cuda_device, layout, tile_n, tile_k, stages, persistent):
    """tile_m 256 = one CTA pair (cluster 2x1, tcgen05.mma.cta_group::2)."""
    m, n, k = 392, 520, 328  # ragged: the last pair tile has an empty second CTA
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=11)
    expect = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, kernel=_native.KERNEL_TCGEN05, tile_m=256,
            cluster_m=2, tile_n=tile_n, tile_k=tile_k, stages=stages, persistent=persistent, raster_group=2)
    np.testing.assert_array_equal(bits_of(c), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
def test_cta_pair_uniform_inputs_within_criterion(cuda_device, layout):
    m, n, k = 1024, 768, 2048
    a, b = oracle.uniform_inputs(m, n, k, 3)
    c = run(to_cuda(a), b_for(layout, to_cuda(b)), layout, kernel=_native.KERNEL_TCGEN05, tile_m=256,
            cluster_m=2, tile_n=256, tile_k=64, stages=6)
    a_t = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    b_t = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)
    ref64, mag = oracle.fp64_reference(a_t, b_t)
    report = oracle.parity_report(bits_of(c), oracle.root_gemm(a, b), ref64, mag, k)
    assert report["passed"], report


def plan_of(m, n, k, layout="col", **cfg):
    return _native.plan(_native.make_config(**cfg), m, n, k, kg.layout_code(layout))


PAIR_256 = dict(kernel=_native.KERNEL_TCGEN05, tile_m=256, cluster_m=2, tile_n=256, tile_k=64, stages=6)


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,flags,mode", [
    # 32 tiles < 74 pairs: the N split by default.
    ((1024, 2048, 512), 0, _native.TAIL_SPLIT_N),
    ((1024, 2048, 512), _native.FLAG_TAIL_SPLIT_N, _native.TAIL_SPLIT_N),
    ((1024, 2048, 512), _native.FLAG_NO_TAIL_SPLIT, _native.TAIL_NONE),
    # 128 tiles = 74 + 54: too many for the N split; stream-K on request.
    ((2048, 4096, 512), 0, _native.TAIL_NONE),
    ((2048, 4096, 512), _native.FLAG_TAIL_STREAM_K, _native.TAIL_STREAM_K),
    # 256 tiles = 3 x 74 + 34: the N split by default, stream-K on request.
    ((4096, 4096, 256), 0, _native.TAIL_SPLIT_N),
    ((4096, 4096, 256), _native.FLAG_TAIL_STREAM_K, _native.TAIL_STREAM_K),
])
def test_cta_pair_split_tail_bit_exact(cuda_device, layout, shape, flags, mode):
    """Every way the last wave can run keeps integer inputs bit-exact."""
    m, n, k = shape
    plan = plan_of(m, n, k, layout, flags=flags, **PAIR_256)
    assert plan["tail_split"] == mode, plan
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=5)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))  # exact for these integers
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, flags=flags, **PAIR_256)
    np.testing.assert_array_equal(bits_of(c), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (1024, 2048, 512), (3072, 5120, 1024)])
def test_cta_pair_n_split_tail_changes_no_bit(cuda_device, layout, shape):
    """Splitting the last wave into half-width units keeps every output one
    full-K UMMA chain: N(0,1) results are bit-identical with and without it."""
    m, n, k = shape
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=2, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    split = run(a, b, layout, flags=_native.FLAG_TAIL_SPLIT_N, **PAIR_256)
    whole = run(a, b, layout, flags=_native.FLAG_NO_TAIL_SPLIT, **PAIR_256)
    assert torch.equal(split.view(torch.int16), whole.view(torch.int16))


# The default pair schedule, the one the slot schedule (cluster_n 2) is compiled for.
PAIR_128K = dict(kernel=_native.KERNEL_TCGEN05, tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3)


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape", [(256, 256, 256), (300, 264, 136), (1234, 2312, 1000), (512, 768, 512),
                                   (4096, 4096, 4096), (2048, 1280, 2048), (4096, 4160, 512), (3072, 5120, 1024)])
def test_slot_schedule_bit_identical_to_pairs(cuda_device, layout, shape):
    """cluster_n 2: two CTA pairs of a 4-CTA cluster share their rows of A
    (each CTA loads one K half and copies it to the other pair over
    distributed shared memory).  Every output is the same full-K UMMA chain
    as on the pair schedule, so N(0,1) results are bit-identical; the shapes
    cover ragged edges, a super tile holding one tile, and the split tail."""
    m, n, k = shape
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=3, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    slots = run(a, b, layout, cluster_n=2, **PAIR_128K)
    pair = run(a, b, layout, **PAIR_128K)
    assert torch.equal(slots.view(torch.int16), pair.view(torch.int16))


def test_slot_schedule_integer_exact_and_plan(cuda_device):
    """The slot schedule on integer inputs matches the oracle bit for bit; its
    plan is groups of four CTAs (4-CTA clusters where they fit, pairs on the
    SMs left over) walking 256 x 512 super tiles."""
    m, n, k = 1000, 1288, 520
    a, b_nk = oracle.integer_inputs(m, n, k, seed=11)
    expect = oracle.root_gemm(bits_of(a), bits_of(b_nk))
    c = run(a.cuda(), b_nk.cuda(), "col", cluster_n=2, **PAIR_128K)
    np.testing.assert_array_equal(bits_of(c), expect)
    plan = plan_of(4096, 4096, 4096, cluster_n=2, **PAIR_128K)
    pair = plan_of(4096, 4096, 4096, **PAIR_128K)
    assert plan["cluster_size"] == 4 and plan["workers"] == pair["workers"] // 2
    assert plan["tiles"] == 16 * 8 and plan["ctas"] % 4 == 0
    rem = plan["tiles"] % plan["workers"]
    if rem and 2 * rem <= plan["workers"]:
        assert plan["tail_split"] == _native.TAIL_SPLIT_N and plan["units"] == plan["tiles"] - rem + 2 * rem


SK = _native.FLAG_TAIL_STREAM_K


def test_tail_plans(cuda_device):
    """4096^3: 256 tiles = 3 W + rem on W pairs.  By default the last rem
    tiles run as 2 rem half-width units; with the stream-K flag the first 2 W
    tiles run whole and the last W + rem are shared by all W pairs."""
    plan = plan_of(4096, 4096, 4096)
    w = plan["workers"]
    assert w > 0
    q, rem = divmod(plan["tiles"], w)
    if rem and 2 * rem <= w:
        assert plan["tail_split"] == _native.TAIL_SPLIT_N
        assert plan["full_tiles"] == plan["tiles"] - rem and plan["units"] == plan["full_tiles"] + 2 * rem
    sk = plan_of(4096, 4096, 4096, flags=SK)
    if rem and q >= 1:
        assert sk["tail_split"] == _native.TAIL_STREAM_K
        assert sk["full_tiles"] == (q - 1) * w
        assert sk["tail_clusters"] == w and sk["tail_segments"] == 2
        assert sk["ctas"] == 2 * w
        assert sk["units"] > sk["tiles"]
    # Fewer tiles than pairs: the N split, or whole tiles for tile_n 128.
    assert plan_of(1024, 2048, 128, tile_k=128)["tail_split"] == _native.TAIL_SPLIT_N
    assert plan_of(1024, 2048, 128, tile_k=128, flags=SK)["tail_split"] == _native.TAIL_SPLIT_N
    narrow = dict(tile_n=128, tile_k=64, stages=4)
    assert plan_of(1024, 1024, 512, **narrow)["tail_split"] == _native.TAIL_NONE
    assert plan_of(2048, 4096, 512, flags=SK, **narrow)["tail_split"] == _native.TAIL_STREAM_K
    # A whole number of waves runs whole.
    assert plan_of(256 * 74, 256, 512, flags=SK)["tail_split"] == _native.TAIL_NONE


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,cfg", [
    ((4096, 4096, 4096), {}),
    ((3072, 5120, 1024), {}),
    ((2048, 4096, 2048), dict(tile_k=64, stages=6)),
    ((2048, 2048, 8192), dict(tile_n=128, tile_k=128, stages=4)),
])
def test_stream_k_tail_within_criterion(cuda_device, layout, shape, cfg):
    """A tile cut at a stream-K range boundary sums two FP32 chains (one
    rounding more than a whole tile); N(0,1) outputs still meet the parity
    criterion against the FP64 product, and sit within 1 ulp of the unsplit
    kernel wherever |C| >= 0.5 (near-zero outputs of heavy cancellation
    differ by more ulps, by less than the FP32 accumulation error).  Two
    launches agree bit for bit."""
    m, n, k = shape
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=4, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    base = dict(kernel=_native.KERNEL_TCGEN05, tile_m=256, cluster_m=2, **cfg)
    assert plan_of(m, n, k, layout, flags=SK, **base)["tail_split"] == _native.TAIL_STREAM_K
    c = run(a, b, layout, flags=SK, **base)
    again = run(a, b, layout, flags=SK, **base)
    assert torch.equal(c.view(torch.int16), again.view(torch.int16))
    whole = run(a, b, layout, flags=_native.FLAG_NO_TAIL_SPLIT, **base)
    assert kg.compare(c, whole).success
    # FP64 check on the last 512-row band, which holds stream-K tiles (they
    # are the end of the raster order); the band keeps the CPU time short.
    sub = slice(m - min(m, 512), m)
    ref64, mag = oracle.fp64_reference(a_t[sub], b_t, layout)
    report = oracle.parity_report(bits_of(c)[sub], bits_of(whole)[sub], ref64, mag, k)
    assert report["passed"] and report["max_ulp_where_ref_ge_0.5"] <= 1, report


def test_stream_k_repeat_and_concurrent_streams(cuda_device):
    """Launch epochs keep repeated launches on one stream and overlapping
    launches on two streams (each with its own workspace) exact."""
    m, n, k = 2048, 4096, 1024
    x_a, x_b = oracle.integer_inputs(m, n, k, seed=8)
    y_a, y_b = oracle.integer_inputs(m, n, k, seed=9)
    ex = oracle.torch_bits(oracle.torch_reference(x_a, x_b))  # exact for these integers
    ey = oracle.torch_bits(oracle.torch_reference(y_a, y_b))
    xa, xb, ya, yb = x_a.cuda(), x_b.cuda(), y_a.cuda(), y_b.cuda()
    assert plan_of(m, n, k, flags=SK)["tail_split"] == _native.TAIL_STREAM_K
    cfg = _native.make_config(flags=SK)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(8):
        cx = kg.bf16_gemm(xa, xb, config=cfg, stream=s1, status=status[0:1])
        cy = kg.bf16_gemm(ya, yb, config=cfg, stream=s2, status=status[1:2])
        outs.append((cx, cy))
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    for cx, cy in outs:
        np.testing.assert_array_equal(bits_of(cx), ex)
        np.testing.assert_array_equal(bits_of(cy), ey)


def test_tcgen05_4096_integer_bit_exact_and_matches_cublas(cuda_device):
    """4096^3, integers in {-2..2}; exact, so the torch CPU
    FP32 reference, cuBLAS and this kernel must agree bit for bit."""
    n = 4096
    a_t, b_t = oracle.integer_inputs(n, n, n, seed=0)
    ref = oracle.torch_reference(a_t, b_t).cuda()
    a, b = a_t.cuda(), b_t.cuda()
    c = run(a, b, "col")
    cmp = kg.compare(c, ref)
    assert cmp.ulp_hist[0] == n * n, cmp
    cublas = torch.matmul(a, b.T)
    assert kg.compare(cublas, ref).ulp_hist[0] == n * n
    c_row = run(a, b.T.contiguous(), "row")
    assert kg.compare(c_row, ref).ulp_hist[0] == n * n


@pytest.mark.parametrize("layout", ["row", "col"])
def test_config1_256_randn_seed0_against_the_reference_cpu_path(cuda_device, layout):
    """BASELINE config 1 exactly: M = N = K = 256, A and B N(0,1) from seed 0
    (CPU generator, B generated row-major [K, N] as the config states) cast to
    BF16, against the reference's CPU-runnable check
    torch.matmul(a.float(), b.float().T).to(bfloat16)
    (src/kernel_mcts/cute_independent_tma.py:1030-1032) and the FP64 bound.
    Both B layouts carry the same matrix; every tcgen05 schedule (the NULL-config
    selection, the CTA-pair default, a one-CTA schedule) gives the same bits."""
    n = 256
    a_t, b_kn = oracle.randn_inputs(n, n, n, seed=0, b_layout="row")
    ref32 = oracle.torch_bits(oracle.torch_reference(a_t, b_kn, "row"))
    ref64, mag = oracle.fp64_reference(a_t, b_kn, "row")
    b_dev = b_kn.cuda() if layout == "row" else b_kn.T.contiguous().cuda()
    schedules = {
        "select": None,
        "pair": dict(kernel=_native.KERNEL_TCGEN05),
        "one_cta": dict(kernel=_native.KERNEL_TCGEN05, tile_m=128, cluster_m=1, tile_n=256, tile_k=64, stages=4),
    }
    outputs = {}
    for name, cfg in schedules.items():
        c = run(a_t.cuda(), b_dev, layout) if cfg is None else run(a_t.cuda(), b_dev, layout, **cfg)
        bits = bits_of(c)
        report = oracle.parity_report(bits, ref32, ref64, mag, n)
        assert report["passed"] and report["max_ulp_where_ref_ge_0.5"] <= 1, (name, report)
        assert oracle.harness_check(bits, ref32)["success"], name
        outputs[name] = bits
    np.testing.assert_array_equal(outputs["pair"], outputs["select"])
    np.testing.assert_array_equal(outputs["one_cta"], outputs["select"])


@pytest.mark.parametrize("layout", ["row", "col"])
def test_tcgen05_4096_randn_within_one_ulp_or_bound(cuda_device, layout):
    """4096^3 N(0,1) BF16 inputs, seed 0, in the bench's
    layout (row-major B, generated as [K, N]) and the reference contract's
    (column-major B, generated as [N, K])."""
    n = 4096
    a_t, b_t = oracle.randn_inputs(n, n, n, seed=0, b_layout=layout)
    c = run(a_t.cuda(), b_t.cuda(), layout)
    ref32 = oracle.torch_bits(oracle.torch_reference(a_t, b_t, layout))
    ref64, mag = oracle.fp64_reference(a_t, b_t, layout)
    report = oracle.parity_report(bits_of(c), ref32, ref64, mag, n)
    assert report["passed"], report
    # Where |ref| >= 0.5 the FP32 reordering error (~K^0.5 * 2^-24 * |partial
    # sums|) is far below half a BF16 ulp, so those elements sit within 1 ulp.
    d = oracle.ulp_distance(bits_of(c), ref32)
    assert int(d[np.abs(ref64) >= 0.5].max()) <= 1
    assert oracle.harness_check(bits_of(c), ref32)["success"]
    # Same-run cuBLAS (tensor cores, FP32 accumulate, the same K order per
    # output) gives the same bits.
    b_torch = b_t.cuda().T if layout == "col" else b_t.cuda()
    cublas = oracle.torch_bits(torch.matmul(a_t.cuda(), b_torch))
    np.testing.assert_array_equal(bits_of(c), cublas)
    # The stream-K tail sums two FP32 chains in its cut tiles: within 1 ulp of
    # cuBLAS wherever |ref| >= 0.5, and within the criterion everywhere.
    sk = bits_of(run(a_t.cuda(), b_t.cuda(), layout, flags=SK))
    assert int(oracle.ulp_distance(sk, cublas)[np.abs(ref64) >= 0.5].max()) <= 1
    assert oracle.parity_report(sk, cublas, ref64, mag, n)["passed"]


def test_config4_full_size_integer_exact_and_randn_matches_cublas(cuda_device):
    """BASELINE config 4 at its full size on one GPU, 8192 x 28672 x 8192, with
    size-independent checks on the device: integer inputs in {-2..2} (sums
    exact in FP32) give cuBLAS's bits everywhere in both B layouts; N(0, 0.02)
    inputs pass the reference harness's tolerance against same-run cuBLAS and
    sit within 1 BF16 ulp of it everywhere; both layouts give the same bits."""
    m, n, k = 8192, 28672, 8192
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randint(-2, 3, (m, k), generator=g, device="cuda").to(torch.bfloat16)
    b_nk = torch.randint(-2, 3, (n, k), generator=g, device="cuda").to(torch.bfloat16)
    ref = torch.matmul(a, b_nk.T)
    for layout in ("col", "row"):
        c = run(a, b_nk if layout == "col" else b_nk.T.contiguous(), layout)
        cmp = kg.compare(c, ref)
        assert cmp.ulp_hist[0] == m * n, (layout, cmp)
        del c
    a = (torch.randn((m, k), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b_nk = (torch.randn((n, k), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    ref = torch.matmul(a, b_nk.T)
    c_col = run(a, b_nk, "col")
    cmp = kg.compare(c_col, ref)
    assert cmp.success and cmp.n_nonfinite == 0 and sum(cmp.ulp_hist[2:]) == 0, cmp  # none beyond 1 ulp
    c_row = run(a, b_nk.T.contiguous(), "row")
    assert torch.equal(c_row.view(torch.int16), c_col.view(torch.int16))
    # A row sample against the CPU oracle: the first and last 32 rows (the
    # first and last row tiles), all 28,672 columns, checked against the
    # reference's CPU path torch.matmul(a.float(), b.float().T).bfloat16()
    # and the FP64 bound.
    rows = torch.cat([torch.arange(0, 32), torch.arange(m - 32, m)])
    a_rows = a[rows.cuda()].cpu()
    b_cpu = b_nk.cpu()
    ref32 = oracle.torch_bits(oracle.torch_reference(a_rows, b_cpu))
    ref64, mag = oracle.fp64_reference(a_rows, b_cpu)
    sample = bits_of(c_col[rows.cuda()])
    report = oracle.parity_report(sample, ref32, ref64, mag, k)
    assert report["passed"] and report["max_ulp_where_ref_ge_2^-6"] <= 1, report
    assert oracle.harness_check(sample, ref32)["success"]


# ------------------------------------------------------------- ABI details


def test_dropin_entry_point_matches_oracle(cuda_device):
    m, n, k = 256, 256, 256
    a, b = oracle.uniform_inputs(m, n, k, 0)
    da, db = to_cuda(a), to_cuda(b)
    dc = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    assert kg.bf16_gemm_sync(da, db, dc) == 0
    report = oracle.harness_check(bits_of(dc), oracle.root_gemm(a, b))
    assert report["success"], report


def test_degenerate_shapes(cuda_device):
    a = torch.ones((64, 0), dtype=torch.bfloat16, device="cuda")
    b = torch.ones((32, 0), dtype=torch.bfloat16, device="cuda")
    c = torch.full((64, 32), 7.0, dtype=torch.bfloat16, device="cuda")
    kg.bf16_gemm(a, b, out=c)
    torch.cuda.synchronize()
    assert torch.count_nonzero(c).item() == 0  # K == 0 gives zeros
    e = kg.bf16_gemm(torch.ones((0, 16), dtype=torch.bfloat16, device="cuda"),
                     torch.ones((8, 16), dtype=torch.bfloat16, device="cuda"))
    assert e.shape == (0, 8)


def test_auto_falls_back_to_simt_for_unaligned_k(cuda_device):
    m, n, k = 96, 64, 45  # K % 8 != 0: TMA cannot take it
    a, b = oracle.uniform_inputs(m, n, k, 4)
    c = run(to_cuda(a), to_cuda(b), "col")
    np.testing.assert_array_equal(bits_of(c), oracle.root_gemm(a, b))
    with pytest.raises(kg.KmctsError):
        run(to_cuda(a), to_cuda(b), "col", kernel=_native.KERNEL_TCGEN05)


def test_compare_kernel_matches_harness_check(cuda_device):
    a, b = oracle.uniform_inputs(200, 136, 64, 2)
    c_bits = oracle.root_gemm(a, b)
    ref_bits = c_bits.copy()
    ref_bits.ravel()[::97] ^= np.uint16(0x0003)  # perturb some mantissas
    ref_bits.ravel()[5] = oracle.float_to_bf16_bits(np.array([0.5], np.float32))[0]
    expect = oracle.harness_check(c_bits, ref_bits)
    got = kg.compare(to_cuda(c_bits), to_cuda(ref_bits))
    assert got.success == expect["success"]
    assert got.maximum_error == pytest.approx(expect["maximum_error"], rel=0, abs=0)
    assert got.mean_error == pytest.approx(expect["mean_error"], rel=1e-12)
    d = oracle.ulp_distance(c_bits, ref_bits).ravel()
    assert got.max_ulp == int(d.max())
    assert got.ulp_hist == (int((d == 0).sum()), int((d == 1).sum()), int((d == 2).sum()), int((d > 2).sum()))
    nan_bits = c_bits.copy()
    nan_bits.ravel()[0] = 0x7FC0
    bad = kg.compare(to_cuda(nan_bits), to_cuda(c_bits))
    assert not bad.success and bad.n_nonfinite == 1


def test_launch_counter_counts_library_launches(cuda_device):
    a_t, b_t = oracle.integer_inputs(256, 256, 256, seed=1)
    a, b = a_t.cuda(), b_t.cuda()
    before = _native.launch_count()
    for _ in range(3):
        kg.bf16_gemm(a, b)
    torch.cuda.synchronize()
    assert _native.launch_count() - before == 3


# ------------------------------------------------------------------ split K

SPLIT = dict(kernel=_native.KERNEL_TCGEN05, tile_m=128, cluster_m=1, tile_n=128, tile_k=128, stages=3)


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,splits", [
    ((16, 1024, 2048), 2), ((16, 1024, 2048), 5), ((100, 520, 1032), 3), ((300, 136, 640), 4),
    ((8, 264, 256), 16),  # more splits than K blocks: capped at 2
    ((8192, 16, 1024), 4),
])
def test_split_k_integer_inputs_bit_exact(cuda_device, layout, shape, splits):
    """Each tile's K ranges add up exactly on integer inputs, whatever the
    split count, the raggedness and the layout."""
    m, n, k = shape
    plan = plan_of(m, n, k, layout, k_splits=splits, **SPLIT)
    assert plan["k_splits"] == min(splits, -(-k // 128)) and plan["units"] == plan["tiles"] * plan["k_splits"]
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=splits)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, k_splits=splits, **SPLIT)
    np.testing.assert_array_equal(bits_of(c), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
def test_split_k_randn_within_criterion_and_deterministic(cuda_device, layout):
    m, n, k = 64, 2048, 8192
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=6, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    c = run(a, b, layout, k_splits=7, **SPLIT)
    again = run(a, b, layout, k_splits=7, **SPLIT)
    assert torch.equal(c.view(torch.int16), again.view(torch.int16))  # fixed split order
    whole = run(a, b, layout, **SPLIT)
    ref64, mag = oracle.fp64_reference(a_t, b_t, layout)
    report = oracle.parity_report(bits_of(c), bits_of(whole), ref64, mag, k)
    assert report["passed"] and report["max_ulp_where_ref_ge_0.5"] <= 1, report


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_k,stages", [(128, 3), (64, 6)])
@pytest.mark.parametrize("shape,splits", [((512, 520, 2048), 3), ((300, 264, 1032), 4), ((256, 256, 4096), 16),
                                          ((1024, 1024, 1024), 2)])
def test_cta_pair_split_k_integer_inputs_bit_exact(cuda_device, layout, tile_k, stages, shape, splits):
    """Split K on the CTA pair: each unit's FP32 rows of both CTAs go to the
    workspace and the tile's last unit adds them in split order; integer
    inputs stay exact (ragged tiles, empty second CTAs included)."""
    m, n, k = shape
    cfg = dict(kernel=_native.KERNEL_TCGEN05, tile_m=256, cluster_m=2, tile_n=256, tile_k=tile_k, stages=stages)
    plan = plan_of(m, n, k, layout, k_splits=splits, **cfg)
    want = min(splits, -(-k // tile_k))
    assert plan["k_splits"] == want and plan["units"] == plan["tiles"] * want and plan["tail_split"] == _native.TAIL_NONE
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=splits)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, k_splits=splits, **cfg)
    np.testing.assert_array_equal(bits_of(c), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
def test_cta_pair_split_k_persistent_round_robin_bit_exact(cuda_device, layout):
    """More split units than co-resident pairs: each persistent pair runs
    several split units in turn, alternating TMEM accumulators and staging
    buffers between them, with the last arriver of each tile reducing.
    Integer inputs are exact, and a second launch repeats every bit."""
    m, n, k, splits = 2048, 2048, 8192, 4
    cfg = dict(PAIR_128K, persistent=1)
    plan = plan_of(m, n, k, layout, k_splits=splits, **cfg)
    assert plan["units"] == plan["tiles"] * splits and plan["units"] > plan["ctas"] // 2, plan
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=11)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    a, b = a_t.cuda(), b_for(layout, b_t.cuda())
    first = run(a, b, layout, k_splits=splits, **cfg)
    second = run(a, b, layout, k_splits=splits, **cfg)
    np.testing.assert_array_equal(bits_of(first), expect)
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("splits", [2, 3, 4])
def test_cta_pair_split_k_randn_within_criterion_and_deterministic(cuda_device, layout, splits):
    """Two or three splits: the last unit brings the partials on chip by bulk
    loads (its stages are free); four: it reads them from L2.  Either way the
    same split order, deterministic, within the criterion."""
    m, n, k = 512, 1024, 8192
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=8, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    c = run(a, b, layout, k_splits=splits, **PAIR_128K)
    again = run(a, b, layout, k_splits=splits, **PAIR_128K)
    assert torch.equal(c.view(torch.int16), again.view(torch.int16))  # fixed split order
    whole = run(a, b, layout, **PAIR_128K)
    ref64, mag = oracle.fp64_reference(a_t, b_t, layout)
    report = oracle.parity_report(bits_of(c), bits_of(whole), ref64, mag, k)
    assert report["passed"] and report["max_ulp_where_ref_ge_0.5"] <= 1, report


def test_split_k_concurrent_streams_and_selection(cuda_device):
    """Skinny shapes select split K; two streams use separate workspaces."""
    m, n, k = 16, 4096, 8192
    sel = _native.select_config(m, n, k, _native.B_COL)
    assert sel.tile_m == 32 and sel.k_splits > 1
    x_a, x_b = oracle.integer_inputs(m, n, k, seed=1)
    y_a, y_b = oracle.integer_inputs(m, n, k, seed=2)
    ex = oracle.torch_bits(oracle.torch_reference(x_a, x_b))
    ey = oracle.torch_bits(oracle.torch_reference(y_a, y_b))
    xa, xb, ya, yb = x_a.cuda(), x_b.cuda(), y_a.cuda(), y_b.cuda()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(6):
        outs.append((kg.bf16_gemm(xa, xb, stream=s1, status=status[0:1]),   # NULL config: the selection
                     kg.bf16_gemm(ya, yb, stream=s2, status=status[1:2])))
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    for cx, cy in outs:
        np.testing.assert_array_equal(bits_of(cx), ex)
        np.testing.assert_array_equal(bits_of(cy), ey)


SKINNY = [(256, 64, 5), (128, 64, 9), (128, 128, 4)]


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_n,tile_k,stages", SKINNY)
@pytest.mark.parametrize("shape,splits", [((1, 520, 1032), 1), ((16, 1024, 2048), 3), ((32, 264, 4096), 8),
                                          ((7, 2048, 512), 1)])
def test_skinny_a_rows_integer_exact(cuda_device, layout, tile_n, tile_k, stages, shape, splits):
    """tile_m 32 stages 32 rows of A; the MMA's other 96 rows are discarded.
    The evict-first cache policy on B's loads changes no bit."""
    m, n, k = shape
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=m + splits)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    for flags in (0, _native.FLAG_B_EVICT_FIRST):
        c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, kernel=_native.KERNEL_TCGEN05, tile_m=32,
                cluster_m=1, tile_n=tile_n, tile_k=tile_k, stages=stages, k_splits=splits, flags=flags)
        np.testing.assert_array_equal(bits_of(c), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,cfg", [
    ((256, 2048, 4096), {}),                                   # default pair, last wave N-split
    ((200, 1024, 8192), dict(tile_k=64, stages=6, k_splits=2)),  # pair split K, ragged M
    ((256, 4096, 1024), dict(tile_n=128, tile_k=128, stages=4)),  # half-width pair tiles
])
def test_cta_pair_b_evict_first_same_bits(cuda_device, layout, shape, cfg):
    """B's loads at L2 evict-first priority on the CTA pair (selected for one
    row of pair tiles) change the cache policy only: exact on integer
    inputs, and the same bits as without the hint on N(0,1) inputs."""
    m, n, k = shape
    base = dict(kernel=_native.KERNEL_TCGEN05, **cfg)
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=9)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, flags=_native.FLAG_B_EVICT_FIRST, **base)
    np.testing.assert_array_equal(bits_of(c), expect)
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=5, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    hinted = run(a, b, layout, flags=_native.FLAG_B_EVICT_FIRST, **base)
    plain = run(a, b, layout, **base)
    assert torch.equal(hinted.view(torch.int16), plain.view(torch.int16))
    sel = _native.select_config(m, n, k, kg.layout_code(layout))
    if sel.tile_m == 256:
        assert sel.flags & _native.FLAG_B_EVICT_FIRST  # one row of pair tiles
        np.testing.assert_array_equal(bits_of(run(a, b, layout)), bits_of(run(a, b, layout, **{
            nm: getattr(sel, nm) for nm, _ in sel._fields_})))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,cfg", [
    ((2048, 256, 4096), dict(tile_m=128, cluster_m=1, tile_n=128, tile_k=128, stages=3)),
    ((2048, 256, 8192), dict(tile_m=128, cluster_m=1, tile_n=128, tile_k=128, stages=3, k_splits=4)),
    ((3000, 512, 2048), {}),  # CTA pair, ragged M
])
def test_a_evict_first_same_bits(cuda_device, layout, shape, cfg):
    """A's loads at L2 evict-first priority (selected when N fits one or two
    tile columns) change the cache policy only: exact on integer inputs, the
    same bits as without the hint on N(0,1) inputs."""
    m, n, k = shape
    base = dict(kernel=_native.KERNEL_TCGEN05, **cfg)
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=12)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, flags=_native.FLAG_A_EVICT_FIRST, **base)
    np.testing.assert_array_equal(bits_of(c), expect)
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=6, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    hinted = run(a, b, layout, flags=_native.FLAG_A_EVICT_FIRST | _native.FLAG_B_EVICT_FIRST, **base)
    plain = run(a, b, layout, **base)
    assert torch.equal(hinted.view(torch.int16), plain.view(torch.int16))
    sel = _native.select_config(m, n, k, kg.layout_code(layout))
    columns = -(-n // sel.tile_n)
    assert bool(sel.flags & _native.FLAG_A_EVICT_FIRST) == (columns <= 2), (sel.tile_n, columns)


HALF = [(128, 128, 4), (128, 128, 3), (64, 128, 6)]


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_n,tile_k,stages", HALF)
@pytest.mark.parametrize("shape,splits", [((64, 520, 1032), 1), ((33, 1024, 2048), 3), ((50, 264, 4096), 4),
                                          ((1, 2048, 512), 1)])
def test_64_row_staging_integer_exact(cuda_device, layout, tile_n, tile_k, stages, shape, splits):
    """tile_m 64 stages 64 rows of A; the MMA's other 64 rows are discarded.
    Exact on integer inputs with and without split K, evict-first or not."""
    m, n, k = shape
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=m + splits)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    for flags in (0, _native.FLAG_B_EVICT_FIRST):
        c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, kernel=_native.KERNEL_TCGEN05, tile_m=64,
                cluster_m=1, tile_n=tile_n, tile_k=tile_k, stages=stages, k_splits=splits, flags=flags)
        np.testing.assert_array_equal(bits_of(c), expect)


@pytest.mark.parametrize("layout", ["col", "row"])
def test_64_row_staging_same_bits_as_128(cuda_device, layout):
    """Staging 64 rows of A instead of 128 changes which rows the MMA reads
    past M, not the K order of any stored row: the same bits on N(0,1)."""
    m, n, k = 64, 1024, 4096
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=4, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    common = dict(kernel=_native.KERNEL_TCGEN05, cluster_m=1, tile_n=128, tile_k=128, stages=3)
    c64 = run(a, b, layout, tile_m=64, **common)
    c128 = run(a, b, layout, tile_m=128, **common)
    assert torch.equal(c64.view(torch.int16), c128.view(torch.int16))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_m,tile_n,tile_k,stages,shape,splits,cluster", [
    (64, 64, 128, 6, (64, 2048, 8192), 4, 4),    # 64 rows: received in the stages
    (64, 128, 128, 3, (50, 1000, 4096), 3, 3),   # 64 rows, ragged: in a receive buffer
    (32, 128, 128, 4, (16, 1024, 2048), 2, 2),
    (32, 128, 128, 4, (32, 264, 4096), 4, 4),    # ragged N
    (32, 128, 64, 9, (7, 2048, 1032), 3, 3),     # ragged K: 17 K blocks over 3 splits
    (32, 256, 64, 5, (16, 1024, 2048), 2, 2),
    (128, 128, 64, 4, (100, 520, 1032), 2, 2),   # four lane quarters, ragged M
    (32, 128, 128, 4, (16, 520, 8192), 8, 8),    # buffer over 227 KB: received in the stages
    (32, 128, 128, 4, (16, 1024, 256), 4, 2),    # two K blocks: two splits
    (128, 128, 128, 3, (512, 512, 8192), 4, 4),  # received in the stages
    (128, 128, 128, 3, (100, 520, 1032), 3, 3),  # ragged M, N and K, in the stages
    (128, 256, 64, 4, (300, 520, 2048), 2, 2),   # 256-column tiles, in the stages
    (128, 128, 128, 3, (256, 256, 16384), 12, 1),  # more than 8 splits: workspace path
])
def test_cluster_split_k_same_bits_as_workspace_split_k(cuda_device, layout, tile_m, tile_n, tile_k, stages, shape,
                                                        splits, cluster):
    """KMCTS_FLAG_SPLIT_CLUSTER runs a tile's K splits as one cluster that
    adds them in split 0's shared memory (a buffer of its own, or its
    pipeline stages once its MMAs are done): exact on integer inputs, and on
    N(0,1) inputs the same bits as the workspace reduction (same sum order),
    launch after launch."""
    m, n, k = shape
    base = dict(kernel=_native.KERNEL_TCGEN05, tile_m=tile_m, cluster_m=1, tile_n=tile_n, tile_k=tile_k,
                stages=stages, k_splits=splits)
    flagged = dict(base, flags=_native.FLAG_SPLIT_CLUSTER)
    plan = plan_of(m, n, k, layout, **flagged)
    assert plan["cluster_size"] == cluster and plan["units"] == plan["tiles"] * plan["k_splits"], plan
    assert plan_of(m, n, k, layout, **base)["cluster_size"] == 1
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=splits + m)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, **flagged)
    np.testing.assert_array_equal(bits_of(c), expect)
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=3, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    workspace = run(a, b, layout, **base)
    first = run(a, b, layout, **flagged)
    second = run(a, b, layout, **flagged)
    assert torch.equal(first.view(torch.int16), workspace.view(torch.int16))
    assert torch.equal(second.view(torch.int16), workspace.view(torch.int16))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_n,tile_k,stages,shape,splits,reduce", [
    (128, 128, 3, (512, 512, 8192), 6, _native.SPLIT_SCATTER),   # 8 pieces over 6 ranks, in the stages
    (128, 128, 3, (512, 512, 8192), 8, _native.SPLIT_SCATTER),   # more clusters than fit at once
    (128, 64, 4, (384, 384, 8192), 8, _native.SPLIT_SCATTER),    # one piece per rank, in a buffer
    (128, 64, 4, (300, 1000, 2048), 4, _native.SPLIT_SCATTER),   # ragged M and N
    (128, 128, 3, (70, 520, 1032), 3, _native.SPLIT_SCATTER),    # a quarter past M, ragged K
    (128, 128, 3, (128, 128, 4096), 7, _native.SPLIT_SCATTER),   # rank 0 owns two pieces
    (64, 64, 6, (512, 512, 4096), 4, _native.SPLIT_SCATTER),     # 64-column tiles: 4 pieces
    (256, 128, 2, (384, 768, 4096), 2, _native.SPLIT_SCATTER),   # 16 pieces, eight per rank
    (128, 64, 5, (200, 520, 1000), 5, _native.SPLIT_SCATTER),    # 8 pieces over 5 ranks, ragged
    (64, 64, 6, (256, 256, 2048), 5, _native.SPLIT_SCATTER),     # more ranks than pieces: rank 4 only sends
    (256, 64, 3, (384, 768, 4096), 8, _native.SPLIT_WORKSPACE),  # pieces and copies exceed the stages
])
def test_scatter_split_k_same_bits_as_workspace_split_k(cuda_device, layout, tile_n, tile_k, stages, shape, splits,
                                                        reduce):
    """KMCTS_FLAG_SPLIT_SCATTER spreads a cluster split K's additions over
    the cluster (piece p of 32 rows x 64 columns to rank p % splits): exact
    on integer inputs, and on N(0,1) inputs the same bits as the workspace
    reduction (each piece adds its splits in split order), launch after
    launch.  Splits past the pieces only send; where the pieces and the
    copies received do not fit the stages, the workspace path runs."""
    m, n, k = shape
    base = dict(kernel=_native.KERNEL_TCGEN05, tile_m=128, cluster_m=1, tile_n=tile_n, tile_k=tile_k,
                stages=stages, k_splits=splits)
    flagged = dict(base, flags=_native.FLAG_SPLIT_CLUSTER | _native.FLAG_SPLIT_SCATTER)
    plan = plan_of(m, n, k, layout, **flagged)
    clustered = reduce != _native.SPLIT_WORKSPACE
    assert plan["cluster_size"] == (splits if clustered else 1) and plan["split_reduce"] == reduce, plan
    assert plan_of(m, n, k, layout, **base)["split_reduce"] == _native.SPLIT_WORKSPACE
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=splits + m)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, **flagged)
    np.testing.assert_array_equal(bits_of(c), expect)
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=6, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    workspace = run(a, b, layout, **base)
    first = run(a, b, layout, **flagged)
    second = run(a, b, layout, **flagged)
    assert torch.equal(first.view(torch.int16), workspace.view(torch.int16))
    assert torch.equal(second.view(torch.int16), workspace.view(torch.int16))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_m,tile_n,tile_k,stages,shape,splits", [
    (32, 128, 128, 4, (16, 8192, 8192), 2),    # 2 pieces, one per rank
    (32, 64, 128, 8, (16, 1024, 16384), 6),    # 1 piece: ranks 1-5 only send
    (32, 128, 128, 4, (7, 2048, 1032), 3),     # ragged M and K
    (32, 256, 64, 5, (16, 1024, 2048), 2),     # 4 pieces
    (64, 128, 128, 3, (64, 8192, 8192), 2),    # two lane quarters: 4 pieces
    (64, 64, 128, 6, (50, 1000, 4096), 4),     # ragged, 2 pieces over 4 ranks
])
def test_scatter_split_k_skinny_same_bits_as_workspace_split_k(cuda_device, layout, tile_m, tile_n, tile_k, stages,
                                                               shape, splits):
    """The scatter form on tiles staging 32 or 64 rows of A (only their lane
    quarters hold pieces): exact on integer inputs and the workspace path's
    bits on N(0,1) inputs."""
    m, n, k = shape
    base = dict(kernel=_native.KERNEL_TCGEN05, tile_m=tile_m, cluster_m=1, tile_n=tile_n, tile_k=tile_k,
                stages=stages, k_splits=splits)
    flagged = dict(base, flags=_native.FLAG_SPLIT_CLUSTER | _native.FLAG_SPLIT_SCATTER)
    plan = plan_of(m, n, k, layout, **flagged)
    assert plan["cluster_size"] == splits and plan["split_reduce"] == _native.SPLIT_SCATTER, plan
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=splits + m + 1)
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout, **flagged)
    np.testing.assert_array_equal(bits_of(c), oracle.torch_bits(oracle.torch_reference(a_t, b_t)))
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=7, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    workspace = run(a, b, layout, **base)
    assert torch.equal(run(a, b, layout, **flagged).view(torch.int16), workspace.view(torch.int16))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape", [(512, 512, 8192), (384, 384, 8192), (300, 1000, 2048), (2048, 256, 8192),
                                   (1024, 1024, 8192), (512, 4096, 8192), (16, 2048, 16384), (48, 4096, 8192)])
def test_scatter_selection_within_bound_and_exact_on_integers(cuda_device, layout, shape):
    """The NULL-config selection for few 128 x 128 tiles over a long K runs
    the scatter split: within the parity bound of the CPU oracle on N(0,1)
    inputs, exact on integer inputs."""
    m, n, k = shape
    bl = _native.B_ROW if layout == "row" else _native.B_COL
    sel = _native.select_config(m, n, k, bl)
    assert sel.flags & _native.FLAG_SPLIT_SCATTER and sel.k_splits >= 2
    assert _native.plan(sel, m, n, k, bl)["split_reduce"] == _native.SPLIT_SCATTER
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=9)
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout)  # NULL config
    np.testing.assert_array_equal(bits_of(c), oracle.torch_bits(oracle.torch_reference(a_t, b_t)))
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=10, b_layout=layout)
    c = run(a_t.cuda(), b_t.cuda(), layout)
    ref32 = oracle.torch_bits(oracle.torch_reference(a_t, b_t, layout))
    ref64, mag = oracle.fp64_reference(a_t, b_t, layout)
    report = oracle.parity_report(bits_of(c), ref32, ref64, mag, k)
    assert report["passed"], report


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape", [(768, 2048, 8192), (640, 2000, 8200)])
def test_pair_three_split_selection_within_bound_and_exact_on_integers(cuda_device, layout, shape):
    """19-24 pair tiles over a long K select three K splits of the CTA-pair
    tiles (workspace reduction): within the parity bound of the CPU oracle,
    exact on integer inputs, deterministic."""
    m, n, k = shape
    bl = _native.B_ROW if layout == "row" else _native.B_COL
    sel = _native.select_config(m, n, k, bl)
    assert (sel.tile_m, sel.k_splits) == (256, 3)
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=11)
    c = run(a_t.cuda(), b_for(layout, b_t.cuda()), layout)
    np.testing.assert_array_equal(bits_of(c), oracle.torch_bits(oracle.torch_reference(a_t, b_t)))
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=12, b_layout=layout)
    first = run(a_t.cuda(), b_t.cuda(), layout)
    second = run(a_t.cuda(), b_t.cuda(), layout)
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))
    ref32 = oracle.torch_bits(oracle.torch_reference(a_t, b_t, layout))
    ref64, mag = oracle.fp64_reference(a_t, b_t, layout)
    report = oracle.parity_report(bits_of(first), ref32, ref64, mag, k)
    assert report["passed"], report


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape", [(16, 8192, 8192), (128, 16384, 4096), (100, 1000, 2048), (48, 4096, 8192),
                                   (64, 2048, 8192)])
def test_skinny_selection_streams_b_evict_first_same_bits(cuda_device, layout, shape):
    """The NULL-config selection for one-tile-row shapes sets the evict-first
    policy; its results equal the same schedule without it, bit for bit, and
    are exact on integer inputs."""
    m, n, k = shape
    sel = _native.select_config(m, n, k, _native.B_ROW if layout == "row" else _native.B_COL)
    assert sel.flags & _native.FLAG_B_EVICT_FIRST and sel.tile_m in (32, 64, 128)
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=5)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    a, b = a_t.cuda(), b_for(layout, b_t.cuda())
    c = run(a, b, layout)  # NULL config
    np.testing.assert_array_equal(bits_of(c), expect)
    plain = {name: getattr(sel, name) for name, _ in sel._fields_}
    plain["flags"] &= ~_native.FLAG_B_EVICT_FIRST
    c_plain = run(a, b, layout, **plain)
    assert torch.equal(c.view(torch.int16), c_plain.view(torch.int16))


def test_library_timing_loop_matches_the_protocol(cuda_device):
    """kmcts_time_gemm: warm-ups, then one event pair per launch; the times are
    positive and the GEMM's result is the same as a plain launch's."""
    m = n = k = 1024
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=3)
    a, b = a_t.cuda(), b_t.cuda()
    c = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    launches = _native.launch_count()
    prepared = kg.PreparedGemm(a, b, c, config=_native.make_config(), status=status)
    times = prepared.time(3, 7)
    assert len(times) == 7 and all(t > 0 for t in times)
    assert _native.launch_count() - launches == 10
    flush = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    assert len(prepared.time(0, 2, flush)) == 2
    np.testing.assert_array_equal(bits_of(c), oracle.torch_bits(oracle.torch_reference(a_t, b_t)))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,chunks", [((1000, 520, 264), 3), ((4096, 1024, 512), 0), ((64, 256, 128), 8)])
def test_host_buffer_gemm_overlapped_copies(cuda_device, layout, shape, chunks):
    """kmcts_bf16_gemm_host: pinned host operands, device scratch buffers, A
    row blocks and B column blocks whose copies and block GEMMs overlap; the
    host C is exact on integer inputs."""
    m, n, k = shape
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=m % 7)
    b_host = (b_t if layout == "col" else b_t.T.contiguous()).pin_memory()
    a_host = a_t.pin_memory()
    c_host = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    a_dev = torch.empty_like(a_host, device="cuda")
    b_dev = torch.empty_like(b_host, device="cuda")
    c_dev = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()
    kg.bf16_gemm_host(a_host, b_host, c_host, a_dev, b_dev, c_dev, b_layout=layout, chunks=chunks,
                      stream=stream, status=status)
    stream.synchronize()
    assert int(status.item()) == 0
    np.testing.assert_array_equal(oracle.torch_bits(c_host), oracle.torch_bits(oracle.torch_reference(a_t, b_t)))


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,chunks", [((2048, 2304, 1024), 0), ((1152, 1000, 2048), 3), ((4096, 4096, 512), 4)])
def test_host_buffer_gemm_bit_identical_to_device_call(cuda_device, layout, shape, chunks):
    """The 2-D block pipeline runs every C block with the schedule chosen for
    the whole problem, so N(0,1) results match the one-call device GEMM bit
    for bit (ragged row and column blocks included)."""
    m, n, k = shape
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=5, b_layout=layout)
    a_host, b_host = a_t.pin_memory(), b_t.pin_memory()
    c_host = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    a_dev, b_dev = a_t.cuda(), b_t.cuda()
    device = run(a_dev, b_dev, layout)
    c_dev = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kg.bf16_gemm_host(a_host, b_host, c_host, torch.empty_like(a_dev), torch.empty_like(b_dev), c_dev, b_layout=layout,
                      chunks=chunks, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(c_host.view(torch.int16), device.cpu().view(torch.int16))


# ------------------------------------------------------- swapped skinny path

SWAP = dict(kernel=_native.KERNEL_TCGEN05, tile_m=32, cluster_m=1, tile_n=128, flags=_native.FLAG_SWAP_AB)


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("tile_k,stages", [(64, 10), (128, 5)])
@pytest.mark.parametrize("shape", [(1, 520, 1032), (7, 2048, 512), (16, 1024, 2048), (17, 264, 4096),
                                   (32, 8192, 1024), (16, 128, 8192), (3, 136, 8)])
def test_swapped_skinny_schedule_integer_exact(cuda_device, layout, tile_k, stages, shape):
    """C^T = B^T A^T with every SM streaming a contiguous range of (tile, K
    block) pairs; cut tiles are summed from FP32 partials.  Integer inputs are
    exact whatever the cuts (ragged N and K, one tile over many ranges, M from
    1 to 32), and a second launch repeats every bit (the counters reset)."""
    m, n, k = shape
    cfg = dict(SWAP, tile_k=tile_k, stages=stages)
    plan = plan_of(m, n, k, layout, **cfg)
    assert plan["kernel"] == 3 and plan["tiles"] == -(-n // 128) and plan["units"] >= plan["tiles"]
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=m + k)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    a, b = a_t.cuda(), b_for(layout, b_t.cuda())
    first = run(a, b, layout, **cfg)
    np.testing.assert_array_equal(bits_of(first), expect)
    second = run(a, b, layout, **cfg)
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))


@pytest.mark.parametrize("layout", ["row", "col"])
def test_swapped_skinny_randn_within_criterion_deterministic_and_concurrent(cuda_device, layout):
    """16 x 8192 x 8192 N(0,1): within the parity criterion against the
    reference's CPU path and the FP64 bound; bit-identical across launches
    and across two streams running at once (separate workspaces)."""
    m, n, k = 16, 8192, 8192
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=3, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    cfg = _native.make_config(**SWAP, tile_k=64, stages=10)
    c = run(a, b, layout, **cfg.as_dict())
    ref32 = oracle.torch_bits(oracle.torch_reference(a_t, b_t, layout))
    ref64, mag = oracle.fp64_reference(a_t, b_t, layout)
    report = oracle.parity_report(bits_of(c), ref32, ref64, mag, k)
    assert report["passed"] and report["max_ulp_where_ref_ge_0.5"] <= 1, report
    assert oracle.harness_check(bits_of(c), ref32)["success"]
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = [(kg.bf16_gemm(a, b, b_layout=layout, config=cfg, stream=s1, status=status[0:1]),
             kg.bf16_gemm(a, b, b_layout=layout, config=cfg, stream=s2, status=status[1:2])) for _ in range(3)]
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    for x, y in outs:
        assert torch.equal(x.view(torch.int16), c.view(torch.int16))
        assert torch.equal(y.view(torch.int16), c.view(torch.int16))


# --------------------------------------------------- K-half exchange tail

KX = _native.FLAG_TAIL_SPLIT_K


@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("shape,cfg", [
    ((4096, 4096, 4096), {}),                          # 3 W + 34 tiles
    ((3072, 5120, 1024), {}),                          # 3 W + 18
    ((1024, 2048, 512), {}),                           # 32 tiles < W: every tile split
    ((1000, 1800, 1000), {}),                          # ragged M, N, K (32 tiles)
    ((4096, 4096, 2048), dict(tile_k=64, stages=6)),
])
def test_k_half_exchange_tail_integer_exact_and_repeatable(cuda_device, layout, shape, cfg):
    """The last wave's tiles as two K halves on two pairs, each writing the
    FP32 sum for its 128 columns after swapping partials: integer inputs
    stay exact, and repeated launches (same stream workspace, new epochs)
    repeat every bit."""
    m, n, k = shape
    base = dict(PAIR_128K, **cfg)
    plan = plan_of(m, n, k, layout, flags=KX, **base)
    w = plan["workers"]
    rem = plan["tiles"] % w
    assert plan["tail_split"] == _native.TAIL_SPLIT_K and 2 * rem <= w, plan
    assert plan["units"] == plan["tiles"] - rem + 2 * rem and plan["tail_segments"] == 2
    a_t, b_t = oracle.integer_inputs(m, n, k, seed=13)
    expect = oracle.torch_bits(oracle.torch_reference(a_t, b_t))
    a, b = a_t.cuda(), b_for(layout, b_t.cuda())
    first = run(a, b, layout, flags=KX, **base)
    np.testing.assert_array_equal(bits_of(first), expect)
    for _ in range(2):
        again = run(a, b, layout, flags=KX, **base)
        assert torch.equal(first.view(torch.int16), again.view(torch.int16))


@pytest.mark.parametrize("layout", ["row", "col"])
def test_k_half_exchange_tail_randn_within_criterion(cuda_device, layout):
    """4096^3 N(0,1) with the K-half exchange tail: within the parity
    criterion against the FP64 product on the last row band (where the
    exchanged tiles lie), within 1 ulp of the unsplit kernel wherever
    |C| >= 0.5, deterministic across launches and concurrent streams."""
    m = n = k = 4096
    a_t, b_t = oracle.randn_inputs(m, n, k, seed=0, b_layout=layout)
    a, b = a_t.cuda(), b_t.cuda()
    cfg = _native.make_config(flags=KX)
    c = run(a, b, layout, flags=KX)
    whole = run(a, b, layout, flags=_native.FLAG_NO_TAIL_SPLIT)
    assert kg.compare(c, whole).success
    sub = slice(m - 512, m)
    ref64, mag = oracle.fp64_reference(a_t[sub], b_t, layout)
    report = oracle.parity_report(bits_of(c)[sub], bits_of(whole)[sub], ref64, mag, k)
    assert report["passed"] and report["max_ulp_where_ref_ge_0.5"] <= 1, report
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = [(kg.bf16_gemm(a, b, b_layout=layout, config=cfg, stream=s1, status=status[0:1]),
             kg.bf16_gemm(a, b, b_layout=layout, config=cfg, stream=s2, status=status[1:2])) for _ in range(3)]
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    for x, y in outs:
        assert torch.equal(x.view(torch.int16), c.view(torch.int16))
        assert torch.equal(y.view(torch.int16), c.view(torch.int16))
