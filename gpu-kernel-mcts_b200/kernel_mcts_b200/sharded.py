"""N-sharded BF16 GEMM over the GPUs of one box.

C[M, N] = A[M, K] · B[K, N] with A replicated and B's columns split over G
ranks (one process per GPU).  Rank r owns columns [r·N/G, (r+1)·N/G).

* ``ShardedGemm.run`` is the fused path.  One kernel computes rank r's
  columns and writes every finished tile into all G ranks' full C: its own by
  TMA store, its peers' by plain stores through CUDA-IPC-mapped pointers over
  NVLink.  The all-gather of C overlaps the GEMM tile by tile, with no
  collective library call, no multicast objects and no NVLS.
* ``ShardedGemm.run_copy_engines`` moves the all-gather off the SMs: the
  shard's GEMM runs as row blocks into a local buffer (each block a whole
  number of near-full waves of CTA pairs), and as each block finishes, one
  stream per destination copies its rows into that rank's C with
  ``kmcts_copy_2d`` (cudaMemcpy2DAsync into IPC-mapped peer memory: the copy
  engines drive NVLink while the SMs compute the next block).
* ``ShardedGemm.run_nccl`` is the baseline: the same GEMM into a local shard,
  ``all_gather_into_tensor`` over NCCL, then the column-block-to-row-major
  copy.

All three leave C bit-identical to the single-GPU kernel on the full problem
under the N tail split (the default here): shard widths are whole
256-column tiles, so every output element has the same K-ordered
accumulation.

The reference has no multi-GPU code (device 0 only); this is a B200
addition, with its host logic tested on CPU (gloo) and the kernel on 2 GPUs.

Self-check / benchmark (one process per GPU)::

    torchrun --nproc-per-node 2 -m kernel_mcts_b200.sharded --M 8192 --N 28672 --K 8192
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
from typing import Any, Callable, Sequence

import torch
import torch.distributed as dist

from . import _native
from .gemm import B_COL, B_ROW, layout_code

HANDLE_BYTES = 72


def shard_columns(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's columns; shards must be whole 256-column tiles."""
    if n_total % world:
        raise ValueError(f"N={n_total} does not split over {world} ranks")
    width = n_total // world
    if width % 256:
        raise ValueError(f"shard width {width} is not a multiple of 256")
    return rank * width, (rank + 1) * width


def exchange_handles(local: bytes, group: Any = None) -> list[bytes]:
    """All ranks' IPC handles, ordered by rank (one all_gather_object)."""
    out: list[Any] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(local), group=group)
    return [bytes(h) for h in out]


class _Ipc:
    """The library's CUDA IPC entry points (a seam the CPU tests replace)."""

    def export(self, ptr: int) -> bytes:
        buf = (ctypes.c_uint8 * HANDLE_BYTES)()
        _native.check(_native.load().kmcts_ipc_export(ctypes.c_void_p(ptr), buf), "kmcts_ipc_export")
        return bytes(buf)

    def open(self, handle: bytes) -> int:
        out = ctypes.c_void_p()
        buf = (ctypes.c_uint8 * HANDLE_BYTES).from_buffer_copy(handle)
        _native.check(_native.load().kmcts_ipc_import(buf, ctypes.byref(out)), "kmcts_ipc_import")
        return int(out.value)

    def close(self, ptr: int) -> None:
        _native.load().kmcts_ipc_close(ctypes.c_void_p(ptr))


def peer_pointers(own_ptr: int, handles: Sequence[bytes], rank: int, opener: Callable[[bytes], int]) -> list[int]:
    """C pointer per rank: this rank's own buffer, imported peers elsewhere."""
    return [own_ptr if r == rank else opener(h) for r, h in enumerate(handles)]


def copy_engine_row_blocks(m: int, shard_width: int, workers: int, min_blocks: int = 4) -> list[tuple[int, int]]:
    """Row ranges for the copy-engine path: whole 256-row tile rows per range,
    chosen so each range's 256 x 256 pair tiles fill the ``workers``
    co-resident pairs' waves as fully as possible (the last range may be
    shorter), with at least ``min_blocks`` ranges so the first copies start
    early."""
    workers = max(1, workers)
    num_m = -(-m // 256)
    tiles_n = -(-shard_width // 256)
    best, best_eff = 1, -1.0
    for per in range(1, num_m + 1):
        if -(-num_m // per) < min(min_blocks, num_m):
            break
        tiles = per * tiles_n
        eff = tiles / (-(-tiles // workers) * workers)
        if eff > best_eff + 1e-9:
            best, best_eff = per, eff
    rows = best * 256
    return [(r0, min(m, r0 + rows)) for r0 in range(0, m, rows)]


class ShardedGemm:
    """One rank's view of an N-sharded GEMM of shape (M, N, K)."""

    def __init__(self, m: int, n: int, k: int, *, b_layout: str = "row", group: Any = None,
                 config: _native.GemmConfig | None = None, ipc: _Ipc | None = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one box)")
        self.m, self.n, self.k = m, n, k
        self.col0, self.col1 = shard_columns(n, self.world, self.rank)
        self.layout = layout_code(b_layout)
        if config is None:
            # The N tail split on both paths: every output stays one full-K
            # chain, so C matches the single-GPU kernel bit for bit whatever
            # the sharding (a K-split tail would depend on the tile count).
            config = _native.default_config()
            config.flags |= _native.FLAG_TAIL_SPLIT_N
        self.config = config
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.c = torch.empty((m, n), dtype=torch.bfloat16, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ipc = ipc or _Ipc()
        handles = exchange_handles(self._ipc.export(self.c.data_ptr()), group)
        self.c_ptrs = peer_pointers(self.c.data_ptr(), handles, self.rank, self._ipc.open)
        self._c_array = (ctypes.c_void_p * self.world)(*self.c_ptrs)
        self._shard = None  # local shard of C (copy-engine and NCCL paths), made on first use
        self._gathered = None  # NCCL baseline's gathered shards, made on first use
        self._ce = None  # copy-engine path: streams and events, made on first use

    @property
    def shard_width(self) -> int:
        return self.col1 - self.col0

    def b_shard_shape(self) -> tuple[int, int]:
        return (self.shard_width, self.k) if self.layout == B_COL else (self.k, self.shard_width)

    def run(self, a: torch.Tensor, b_shard: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Fused GEMM + all-gather.  Asynchronous: call ``finish()`` before reading C."""
        stream = stream or torch.cuda.current_stream(self.device)
        rc = _native.load().kmcts_bf16_gemm_allgather(
            ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b_shard.data_ptr()), self._c_array, self.world,
            self.rank, self.m, self.n, self.k, self.layout, ctypes.byref(self.config),
            ctypes.c_void_p(stream.cuda_stream), ctypes.c_void_p(self.status.data_ptr()))
        _native.check(rc, "kmcts_bf16_gemm_allgather")

    def row_blocks(self) -> list[tuple[int, int]]:
        """Row ranges of the copy-engine path (see copy_engine_row_blocks)."""
        workers = int(_native.plan(self.config, self.m, self.shard_width, self.k, self.layout)["workers"])
        return copy_engine_row_blocks(self.m, self.shard_width, workers)

    def run_copy_engines(self, a: torch.Tensor, b_shard: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """GEMM of the shard in row blocks; each finished block copied into
        every rank's C (own and peers') by the copy engines, one stream per
        destination.  Asynchronous: call ``finish()`` before reading C."""
        from . import gemm as kg

        stream = stream or torch.cuda.current_stream(self.device)
        if self._shard is None:
            self._shard = torch.empty((self.m, self.shard_width), dtype=torch.bfloat16, device=self.device)
        if self._ce is None:
            blocks = self.row_blocks()
            self._ce = {
                "blocks": blocks,
                "streams": [torch.cuda.Stream(self.device) for _ in range(self.world)],
                "events": [torch.cuda.Event() for _ in blocks],
                "done": [torch.cuda.Event() for _ in range(self.world)],
            }
        lib = _native.load()
        ce = self._ce
        w = self.shard_width
        pitch = self.n * 2
        for (r0, r1), event in zip(ce["blocks"], ce["events"]):
            kg.bf16_gemm(a[r0:r1], b_shard, out=self._shard[r0:r1], b_layout=self.layout, config=self.config,
                         stream=stream, status=self.status)
            event.record(stream)
            for dest, copy_stream in enumerate(ce["streams"]):
                copy_stream.wait_event(event)
                dst = self.c_ptrs[dest] + (r0 * self.n + self.col0) * 2
                rc = lib.kmcts_copy_2d(ctypes.c_void_p(dst), pitch,
                                       ctypes.c_void_p(self._shard.data_ptr() + r0 * w * 2), w * 2, w * 2, r1 - r0,
                                       ctypes.c_void_p(copy_stream.cuda_stream))
                _native.check(rc, "kmcts_copy_2d")
        for done, copy_stream in zip(ce["done"], ce["streams"]):
            done.record(copy_stream)
            stream.wait_event(done)

    def run_nccl(self, a: torch.Tensor, b_shard: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Baseline: local GEMM, NCCL all-gather, column-block -> row-major copy."""
        from . import gemm as kg

        stream = stream or torch.cuda.current_stream(self.device)
        if self._shard is None:
            self._shard = torch.empty((self.m, self.shard_width), dtype=torch.bfloat16, device=self.device)
        if self._gathered is None:
            self._gathered = torch.empty((self.world, self.m, self.shard_width), dtype=torch.bfloat16,
                                         device=self.device)
        with torch.cuda.stream(stream):
            kg.bf16_gemm(a, b_shard, out=self._shard, b_layout=self.layout, config=self.config, stream=stream,
                         status=self.status)
            dist.all_gather_into_tensor(self._gathered, self._shard, group=self.group)
            self.c.view(self.m, self.world, self.shard_width).copy_(self._gathered.permute(1, 0, 2))

    def finish(self) -> None:
        """Every rank's stores have landed in every C (stream sync + barrier)."""
        torch.cuda.synchronize(self.device)
        if int(self.status.item()) != 0:
            raise RuntimeError(f"device status {int(self.status.item()):#x}")
        if self.world > 1:
            if dist.get_backend(self.group) == "nccl":
                dist.barrier(group=self.group, device_ids=[self.device.index])
            else:
                dist.barrier(group=self.group)

    def close(self) -> None:
        for r, ptr in enumerate(self.c_ptrs):
            if r != self.rank:
                self._ipc.close(ptr)
        self.c_ptrs = []


def _main(argv: Sequence[str] | None = None) -> None:
    from datetime import timedelta

    from . import gemm as kg

    p = argparse.ArgumentParser(description="N-sharded GEMM self-check and timing (run under torchrun)")
    p.add_argument("--M", type=int, default=8192)
    p.add_argument("--N", type=int, default=28672)
    p.add_argument("--K", type=int, default=8192)
    p.add_argument("--b-layout", choices=("col", "row"), default="row")
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--check", action="store_true", help="compare with the single-GPU kernel on the full problem")
    args = p.parse_args(argv)

    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    g = torch.Generator(device=device).manual_seed(0)  # same A and B on every rank
    a = (torch.randn((args.M, args.K), generator=g, device=device) * 0.02).to(torch.bfloat16)
    b_full = (torch.randn((args.K, args.N) if args.b_layout == "row" else (args.N, args.K), generator=g,
                          device=device) * 0.02).to(torch.bfloat16)
    sg = ShardedGemm(args.M, args.N, args.K, b_layout=args.b_layout)
    b_shard = (b_full[:, sg.col0:sg.col1] if args.b_layout == "row" else b_full[sg.col0:sg.col1]).contiguous()
    out: dict[str, Any] = {"world": world, "shape": [args.M, args.N, args.K], "b_layout": args.b_layout}
    try:
        if args.check:
            full = kg.bf16_gemm(a, b_full, b_layout=args.b_layout, config=sg.config)
            for name, fn in (("fused", sg.run), ("copy_engines", sg.run_copy_engines), ("nccl", sg.run_nccl)):
                sg.c.zero_()
                dist.barrier(device_ids=[local_rank])
                fn(a, b_shard)
                sg.finish()
                out[f"{name}_bit_identical"] = bool(torch.equal(sg.c.view(torch.int16), full.view(torch.int16)))
        stream = torch.cuda.current_stream(device)
        for name, fn in (("fused", sg.run), ("copy_engines", sg.run_copy_engines), ("nccl", sg.run_nccl)):
            for _ in range(args.warmup):
                fn(a, b_shard)
                sg.finish()
            times = []
            for _ in range(args.steps):
                dist.barrier(device_ids=[local_rank])
                torch.cuda.synchronize(device)
                start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                fn(a, b_shard)
                stop.record(stream)
                sg.finish()
                times.append(start.elapsed_time(stop) * 1e3)
            med = torch.tensor([statistics.median(times)], dtype=torch.float64, device=device)
            dist.all_reduce(med, op=dist.ReduceOp.MAX)
            out[f"{name}_median_us"] = float(med.item())
            out[f"{name}_tflops"] = 2.0 * args.M * args.N * args.K / (float(med.item()) * 1e-6) / 1e12
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        sg.close()
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == "__main__":
    _main()
