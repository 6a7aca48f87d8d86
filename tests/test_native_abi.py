"""The C-ABI library loads, exports what include/kmcts_gemm.h declares, and
its host-only entry points (no GPU work) behave."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

import kernel_mcts_b200 as km
from kernel_mcts_b200 import _native

ROOT = Path(__file__).resolve().parent.parent


def _declared_functions() -> set[str]:
    names: set[str] = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", " ", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(kmcts_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = _native.load()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    missing = [name for name in sorted(declared) if not hasattr(lib, name)]
    assert not missing, missing
    assert set(_native.EXPORTED_SYMBOLS) == declared


def test_struct_sizes_match_header():
    assert ctypes.sizeof(_native.GemmConfig) == 56
    assert ctypes.sizeof(_native.CompareResult) == 8 * 2 + 8 * 3 + 8 * 4 + 4 * 2


def test_version_and_default_config():
    assert "sm_100a" in km.version()
    cfg = km.default_config()
    assert (cfg.tile_m, cfg.tile_n, cfg.tile_k, cfg.stages, cfg.cluster_m) == (256, 256, 128, 3, 2)
    assert km.config_legal(cfg, 4096, 4096, 4096) == (0, "ok")


def test_skinny_a_rows_take_at_most_32_rows():
    cfg = km.make_config(tile_m=32, cluster_m=1, tile_n=256, tile_k=64, stages=5)
    assert km.config_legal(cfg, 32, 4096, 4096, km.B_ROW)[0] == 0
    code, why = km.config_legal(cfg, 33, 4096, 4096, km.B_ROW)
    assert code == _native.KMCTS_ENOTSUP and "M <= 32" in why
    assert km.config_legal(km.make_config(tile_m=32, cluster_m=2), 16, 4096, 4096)[0] == _native.KMCTS_ENOTSUP


def test_64_row_staging_takes_at_most_64_rows():
    cfg = km.make_config(tile_m=64, cluster_m=1, tile_n=128, tile_k=128, stages=4)
    assert km.config_legal(cfg, 64, 4096, 4096, km.B_ROW) == (0, "ok")
    code, why = km.config_legal(cfg, 65, 4096, 4096, km.B_ROW)
    assert code == _native.KMCTS_ENOTSUP and "M <= 64" in why
    # 4 x (64 + 128) x 128 x 2 of stages, two warps' staging buffers, reserve
    assert km.config_smem_bytes(cfg) == 4 * 192 * 128 * 2 + 2 * 2 * 4096 + 2048
    assert km.config_legal(km.make_config(tile_m=64, cluster_m=1, tile_n=256, tile_k=64, stages=4),
                           64, 4096, 4096)[0] == _native.KMCTS_ENOTSUP  # not compiled


def test_select_config_splits_k_for_skinny_shapes():
    cfg = km.select_config(16, 8192, 8192, km.B_ROW)
    assert (cfg.tile_m, cfg.tile_n, cfg.k_splits) == (32, 128, 2)  # 64 tiles -> 128 units
    assert cfg.flags & _native.FLAG_SPLIT_CLUSTER  # the two splits add up in shared memory
    wide = km.select_config(8, 28672, 8192, km.B_ROW)
    assert (wide.tile_m, wide.tile_n, wide.k_splits) == (32, 256, 0)  # 112 tiles: no split
    assert not wide.flags & _native.FLAG_SPLIT_CLUSTER
    # Fewer tiles: as many splits as keep every cluster resident (at most 8;
    # the B200 capacities without a GPU: 16 clusters of 6, not of 7 or 8),
    # added up across the cluster (scatter).
    scatter = _native.FLAG_SPLIT_CLUSTER | _native.FLAG_SPLIT_SCATTER
    narrow = km.select_config(16, 2048, 16384, km.B_ROW)
    assert (narrow.tile_m, narrow.tile_n, narrow.tile_k, narrow.stages, narrow.k_splits) == (32, 128, 128, 4, 6)
    assert narrow.flags & scatter == scatter
    assert not cfg.flags & _native.FLAG_SPLIT_SCATTER  # two splits of 32-row tiles: split 0 adds
    assert km.select_config(16, 4096, 8192, km.B_ROW).k_splits == 4  # 32 tiles of 128 columns
    long_k = km.select_config(16, 1024, 32768, km.B_ROW)
    assert (long_k.tile_n, long_k.k_splits) == (128, 8) and long_k.flags & scatter == scatter
    assert km.select_config(65, 8192, 8192, km.B_ROW).tile_m == 128
    mid = km.select_config(64, 2048, 8192, km.B_ROW)  # 16 tiles of 64 x 128, six splits
    assert (mid.tile_m, mid.tile_n, mid.stages, mid.k_splits) == (64, 128, 3, 6) and mid.flags & scatter == scatter
    wide64 = km.select_config(64, 16384, 4096, km.B_ROW)  # 128 tiles of 128 columns: unsplit, four stages
    assert (wide64.tile_m, wide64.tile_n, wide64.stages, wide64.k_splits) == (64, 128, 4, 0)
    split64 = km.select_config(64, 8192, 8192, km.B_ROW)  # 64 tiles: two splits, three stages
    assert (split64.tile_m, split64.tile_n, split64.stages, split64.k_splits) == (64, 128, 3, 2)
    assert split64.flags & scatter == scatter
    assert km.select_config(33, 1024, 16384, km.B_ROW).k_splits == 8
    for shape in ((16, 2048, 16384), (64, 2048, 8192), (33, 1024, 16384)):
        plan = _native.plan(km.select_config(*shape, km.B_ROW), *shape, km.B_ROW)
        assert plan["split_reduce"] == _native.SPLIT_SCATTER and plan["tiles"] <= plan["workers"], shape
    # Few 128 x 128 tiles over a long K: the same, on 128-row tiles.
    m128 = km.select_config(128, 4096, 8192, km.B_ROW)
    assert (m128.tile_n, m128.tile_k, m128.stages, m128.k_splits) == (128, 128, 3, 4)
    assert m128.flags & scatter == scatter and m128.flags & _native.FLAG_B_EVICT_FIRST
    sq = km.select_config(512, 512, 8192, km.B_ROW)
    # 16 tiles: six splits would fit, five run faster on 128-row tiles.
    assert (sq.tile_n, sq.tile_k, sq.stages, sq.k_splits) == (128, 128, 3, 5) and sq.flags & scatter == scatter
    # Ranges of at most 1024: 64-deep stages, receiving past them; longer: 128-deep.
    eight = km.select_config(384, 384, 8192, km.B_ROW)
    assert (eight.tile_k, eight.stages, eight.k_splits) == (64, 4, 8) and eight.flags & scatter == scatter
    deep = km.select_config(256, 512, 16384, km.B_ROW)
    assert (deep.tile_k, deep.stages, deep.k_splits) == (128, 3, 8) and deep.flags & scatter == scatter
    short = km.select_config(300, 1000, 2048, km.B_ROW)
    assert (short.tile_k, short.stages, short.k_splits) == (64, 4, 4) and short.flags & scatter == scatter
    assert km.select_config(1024, 1024, 8192, km.B_ROW).k_splits == 2
    assert km.select_config(1024, 1024, 2048, km.B_ROW).k_splits == 0  # two splits only from K = 4096
    assert km.select_config(768, 768, 2048, km.B_ROW).k_splits == 3
    for shape in ((512, 512, 8192), (384, 384, 8192), (300, 1000, 2048), (128, 4096, 8192)):
        plan = _native.plan(km.select_config(*shape, km.B_ROW), *shape, km.B_ROW)
        assert plan["split_reduce"] == _native.SPLIT_SCATTER, shape
        assert plan["tiles"] <= plan["workers"], shape  # every cluster resident at once
    assert km.select_config(1024, 1024, 1024, km.B_ROW).k_splits == 0  # short K: no split
    assert km.select_config(4096, 4096, 4096, km.B_ROW).k_splits == 0
    assert km.select_config(256, 256, 256, km.B_ROW).k_splits == 0  # K too short to split
    # 32 pair tiles over a long K: the pair schedule in two K splits.
    pair_split = km.select_config(4096, 512, 16384, km.B_ROW)
    assert (pair_split.tile_m, pair_split.tile_k, pair_split.stages, pair_split.k_splits) == (256, 64, 6, 2)
    # 19-24 pair tiles over a long K: three K splits of the pair tiles.
    three = km.select_config(768, 2048, 8192, km.B_ROW)
    assert (three.tile_m, three.tile_k, three.stages, three.k_splits) == (256, 64, 6, 3)
    assert km.select_config(768, 2048, 4096, km.B_ROW).k_splits == 0  # K = 4096: unsplit
    # ... with more than two tile columns, one CTA per 128 x 256 tile in two K
    # splits added up across a 2-CTA cluster instead.
    wide_split = km.select_config(256, 8192, 8192, km.B_ROW)
    assert (wide_split.tile_m, wide_split.tile_n, wide_split.tile_k, wide_split.stages, wide_split.k_splits) == \
        (128, 256, 64, 4, 2)
    assert wide_split.flags & scatter == scatter and wide_split.flags & _native.FLAG_B_EVICT_FIRST
    assert _native.plan(wide_split, 256, 8192, 8192, km.B_ROW)["split_reduce"] == _native.SPLIT_SCATTER
    # One or two rows of pair tiles: B streams at evict-first priority; more: not.
    for shape in ((256, 16384, 4096), (200, 28672, 8192), (512, 16384, 4096)):
        sel = km.select_config(*shape, km.B_ROW)
        assert sel.tile_m == 256 and sel.flags & _native.FLAG_B_EVICT_FIRST, shape
    assert not km.select_config(1024, 16384, 4096, km.B_ROW).flags & _native.FLAG_B_EVICT_FIRST
    # One or two tile columns: A streams at evict-first priority; N <= 128
    # leaves the pair (half of its 256-column tile would be empty).
    tall = km.select_config(16384, 128, 4096, km.B_ROW)
    assert (tall.tile_m, tall.tile_n) == (128, 128) and tall.flags & _native.FLAG_A_EVICT_FIRST
    narrow_pair = km.select_config(28672, 256, 4096, km.B_ROW)
    assert narrow_pair.tile_m == 256 and narrow_pair.flags & _native.FLAG_A_EVICT_FIRST
    assert not km.select_config(4096, 4096, 4096, km.B_ROW).flags & _native.FLAG_A_EVICT_FIRST
    assert not km.select_config(4096, 4096, 4096, km.B_ROW).flags & _native.FLAG_B_EVICT_FIRST
    # ... not at K = 4096: one CTA per 128 x 256 tile.
    assert km.select_config(2048, 1024, 4096, km.B_ROW).tile_m == 128
    assert km.select_config(2048, 256, 8192, km.B_ROW).k_splits == 4  # 32 tiles -> 128 units, one wave
    # One tile over a very long K: sixteen workspace splits, more than a cluster holds.
    one_tile = km.select_config(128, 128, 65536, km.B_ROW)
    assert one_tile.k_splits == 16 and not one_tile.flags & _native.FLAG_SPLIT_CLUSTER


@pytest.mark.parametrize(
    "shape,expect",
    [
        # 256 pair tiles >= 74 co-resident pairs (148 SMs assumed without a GPU): the default.
        ((4096, 4096, 4096), (256, 256, 128, 3, 2)),
        ((2048, 4096, 2048), (256, 256, 128, 3, 2)),
        # K <= 768: 64-deep stages, six of them (five for K <= 256).
        ((8192, 8192, 512), (256, 256, 64, 6, 2)),
        ((16384, 4096, 384), (256, 256, 64, 6, 2)),
        ((8192, 8192, 768), (256, 256, 64, 6, 2)),
        ((8192, 8192, 256), (256, 256, 64, 5, 2)),
        ((8192, 8192, 1024), (256, 256, 128, 3, 2)),
        # 64 pair tiles, 128 one-CTA 128x256 tiles: one CTA per 128x256 tile.
        ((2048, 2048, 2048), (128, 256, 64, 4, 1)),
        # ... unless K is long: the pair's mainloop wins back its idle SMs.
        ((2048, 2048, 8192), (256, 256, 128, 3, 2)),
        # few tiles: one CTA per 128x128 tile.
        ((1024, 1024, 1024), (128, 128, 128, 3, 1)),
        ((256, 256, 256), (128, 128, 128, 3, 1)),
        # N not a multiple of 8: no tensor-core schedule is legal; the default
        # stays and AUTO launches go to the SIMT kernel.
        ((256, 250, 256), (256, 256, 128, 3, 2)),
        ((16, 250, 256), (256, 256, 128, 3, 2)),
    ],
)
def test_select_config_by_shape(shape, expect):
    cfg = km.select_config(*shape, km.B_ROW)
    assert (cfg.tile_m, cfg.tile_n, cfg.tile_k, cfg.stages, cfg.cluster_m) == expect
    if shape[1] % 8 == 0:
        assert km.config_legal(cfg, *shape, km.B_ROW) == (0, "ok")


@pytest.mark.parametrize(
    "overrides,shape,code",
    [
        ({"tile_m": 128, "cluster_m": 1, "tile_n": 256, "tile_k": 64, "stages": 5}, (4096, 4096, 4096), _native.KMCTS_ESMEM),
        ({"tile_m": 256, "cluster_m": 1}, (4096, 4096, 4096), _native.KMCTS_ENOTSUP),
        ({"tile_m": 128, "cluster_m": 2}, (4096, 4096, 4096), _native.KMCTS_ENOTSUP),
        ({"cluster_n": 2}, (4096, 4096, 4096), _native.KMCTS_OK),  # two pairs per 4-CTA cluster sharing A
        ({"cluster_n": 2, "tile_k": 64, "stages": 6}, (4096, 4096, 4096), _native.KMCTS_ENOTSUP),
        ({"cluster_n": 2, "tile_m": 128, "cluster_m": 1}, (4096, 4096, 4096), _native.KMCTS_ENOTSUP),
        ({"cluster_n": 4}, (4096, 4096, 4096), _native.KMCTS_ENOTSUP),
        ({"tile_k": 128, "stages": 4}, (4096, 4096, 4096), _native.KMCTS_ESMEM),
        ({"tile_n": 192}, (4096, 4096, 4096), _native.KMCTS_ENOTSUP),
        ({}, (4096, 4096, 4100), _native.KMCTS_ENOTSUP),  # K not a multiple of 8
        ({}, (4096, 4100, 4096), _native.KMCTS_ENOTSUP),  # N not a multiple of 8
        ({"raster_group": 0}, (256, 256, 256), _native.KMCTS_EINVAL),
        ({"tile_m": 128, "cluster_m": 1, "tile_n": 128, "tile_k": 64, "stages": 6}, (256, 256, 256), _native.KMCTS_OK),
        ({"tile_m": 128, "cluster_m": 1, "tile_n": 128, "tile_k": 128, "stages": 3}, (256, 256, 256), _native.KMCTS_OK),
        ({"tile_n": 128, "tile_k": 64, "stages": 6}, (256, 256, 256), _native.KMCTS_OK),
    ],
)
def test_config_legality(overrides, shape, code):
    cfg = km.make_config(**overrides)
    got, why = km.config_legal(cfg, *shape)
    assert got == code, why
    assert why


def test_smem_accounting():
    cfg = km.make_config(tile_m=128, cluster_m=1, tile_n=256, tile_k=64, stages=4)
    assert km.config_smem_bytes(cfg) == 4 * (128 + 256) * 64 * 2 + 4 * 2 * 4096 + 2048
    assert km.config_smem_bytes(cfg) <= 232448
    pair = km.default_config()  # each CTA of a pair stages 128 rows of A and BN/2 of B
    assert km.config_smem_bytes(pair) == 3 * (128 + 128) * 128 * 2 + 4 * 2 * 4096 + 2048


def test_bad_arguments_rejected_without_gpu_work():
    lib = _native.load()
    assert lib.kmcts_bf16_gemm_ex(None, None, None, -1, 4, 4, 0, None, None, None) == _native.KMCTS_EINVAL
    assert lib.kmcts_bf16_gemm_ex(None, None, None, 4, 4, 4, 7, None, None, None) == _native.KMCTS_EINVAL
    assert lib.kmcts_bf16_gemm_ex(None, None, None, 4, 4, 4, 0, None, None, None) == _native.KMCTS_EINVAL
    assert lib.kmcts_default_config(None) == _native.KMCTS_EINVAL


@pytest.mark.parametrize("tile_m,tile_n,tile_k,stages,splits,reduce,extra", [
    # 128 x 64-deep x 4 stages (162 KB own): received copies fit past it.
    (128, 128, 64, 4, 8, _native.SPLIT_SCATTER, 7 * 8192),       # one piece per rank, 7 copies
    (128, 128, 64, 4, 5, _native.SPLIT_SCATTER, 2 * 4 * 8192),   # two pieces for rank 0
    (128, 128, 64, 4, 6, _native.SPLIT_WORKSPACE, 0),            # neither a buffer nor the stages hold them
    # 128 x 128-deep x 3 stages (226 KB own): received in the stages.
    (128, 128, 128, 3, 6, _native.SPLIT_SCATTER, 0),
    # 32-row tiles: 2 pieces, splits past them only send.
    (32, 128, 128, 4, 6, _native.SPLIT_SCATTER, 1 * 5 * 8192),
])
def test_scatter_receive_placement(tile_m, tile_n, tile_k, stages, splits, reduce, extra):
    """Where a scatter split's copies land: a buffer past the schedule's own
    shared memory when that fits 227 KB (the plan adds its size), else the
    stages past the outgoing pieces, else no cluster split at all."""
    m = 32 if tile_m == 32 else 512
    cfg = km.make_config(tile_m=tile_m, cluster_m=1, tile_n=tile_n, tile_k=tile_k, stages=stages, k_splits=splits,
                         flags=_native.FLAG_SPLIT_CLUSTER | _native.FLAG_SPLIT_SCATTER)
    plan = _native.plan(cfg, m, 512, 8192, km.B_ROW)
    assert plan["split_reduce"] == reduce, plan
    assert plan["smem_bytes"] == km.config_smem_bytes(cfg) + extra, plan



def test_selection_properties_over_a_shape_grid():
    """Over a grid of shapes (148 SMs and the B200 cluster capacities assumed
    without a GPU): every selected schedule is legal, a cluster split keeps
    every cluster resident with one unit per SM and at most 8 splits, and a
    workspace split never asks for more than 16."""
    dims_m = (1, 16, 33, 64, 100, 128, 200, 256, 384, 512, 768, 1024, 2048, 4096)
    dims_n = (128, 256, 512, 1000, 1024, 2048, 4096, 8192, 16384)
    dims_k = (256, 1024, 2048, 4096, 8192, 16384, 32768)
    checked = 0
    for m in dims_m:
        for n in dims_n:
            for k in dims_k:
                cfg = km.select_config(m, n, k, km.B_ROW)
                code, why = _native.config_legal(cfg, m, n, k, km.B_ROW)
                assert code == _native.KMCTS_OK, (m, n, k, why)
                checked += 1
                if cfg.tile_m == 256:
                    continue  # a pair's plan asks the occupancy calculator: it needs a device
                plan = _native.plan(cfg, m, n, k, km.B_ROW)
                if plan["cluster_size"] > 1 and cfg.tile_m != 256:
                    assert cfg.flags & _native.FLAG_SPLIT_CLUSTER, (m, n, k)
                    assert 2 <= plan["k_splits"] <= 8 and plan["cluster_size"] == plan["k_splits"], (m, n, k, plan)
                    assert plan["ctas"] <= 148 and plan["tiles"] <= plan["workers"], (m, n, k, plan)
                    assert plan["split_reduce"] in (_native.SPLIT_CLUSTER, _native.SPLIT_SCATTER), (m, n, k, plan)
                else:
                    assert plan["k_splits"] <= 16, (m, n, k, plan)
    assert checked == len(dims_m) * len(dims_n) * len(dims_k)
