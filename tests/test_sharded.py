"""Host logic of the N-sharded GEMM on CPU: shard arithmetic, and the IPC
handle exchange over a real 2-rank gloo group (fake IPC, no GPU)."""

from __future__ import annotations

import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kernel_mcts_b200.sharded import exchange_handles, peer_pointers, shard_columns


def test_shard_columns_cover_n_in_whole_tiles():
    spans = [shard_columns(28672, 8, r) for r in range(8)]
    assert spans[0] == (0, 3584) and spans[-1] == (28672 - 3584, 28672)
    assert all(b == c for (_, b), (c, _) in zip(spans, spans[1:]))
    for world in (1, 2, 4, 8):
        assert shard_columns(28672, world, world - 1)[1] == 28672
    with pytest.raises(ValueError):
        shard_columns(1000, 3, 0)
    with pytest.raises(ValueError):
        shard_columns(28672 * 2 + 256, 2, 0)  # 14464 columns per rank: not whole tiles


def _exchange_worker(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = bytes([rank]) * 72
        handles = exchange_handles(local)
        opened = []
        ptrs = peer_pointers(1000 + rank, handles, rank, lambda h: opened.append(h[0]) or 5000 + h[0])
        results.put((rank, [h[0] for h in handles], ptrs, opened))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_orders_by_rank_and_opens_only_peers():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict()
    for _ in range(2):
        rank, order, ptrs, opened = results.get(timeout=120)
        got[rank] = (order, ptrs, opened)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == ([0, 1], [1000, 5001], [1])
    assert got[1] == ([0, 1], [5000, 1001], [0])


def test_copy_engine_row_blocks_fill_waves_and_cover_m():
    from kernel_mcts_b200.sharded import copy_engine_row_blocks

    # 8 GPUs on config 4: 14 tile columns per rank; 5 tile rows = 70 tiles on 74 pairs.
    blocks = copy_engine_row_blocks(8192, 3584, 74)
    assert blocks[0] == (0, 1280) and blocks[-1][1] == 8192 and len(blocks) == 7
    assert all(b == c for (_, b), (c, _) in zip(blocks, blocks[1:]))
    # 4 GPUs: 28 tile columns; 5 tile rows = 140 tiles, 0.95 of two waves.
    assert copy_engine_row_blocks(8192, 7168, 74)[0] == (0, 1280)
    # At least four blocks whenever there are four tile rows; ragged M covered.
    small = copy_engine_row_blocks(2048, 2048, 74)
    assert len(small) >= 4 and small[-1][1] == 2048
    ragged = copy_engine_row_blocks(1000, 512, 74)
    assert ragged[0][0] == 0 and ragged[-1][1] == 1000 and all(r1 > r0 for r0, r1 in ragged)
