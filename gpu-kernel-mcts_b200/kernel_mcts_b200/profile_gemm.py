"""Runs a few launches of one GEMM schedule, for ncu captures and quick timing.

    python -m kernel_mcts_b200.profile_gemm --M 4096 --N 4096 --K 4096 \
        --b-layout row --launches 3
    python -m kernel_mcts_b200.profile_gemm --M 16 --N 8192 --K 8192 --select

Prints one JSON line with the CUDA-event time of each launch.  Inputs are
N(0,1) BF16 from a seeded generator on the device; nothing else runs on the
GPU, so an ncu capture of ``gemm_bf16_tcgen05`` sees exactly these launches.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch

from . import _native
from . import gemm as kg


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--M", type=int, default=4096)
    p.add_argument("--N", type=int, default=4096)
    p.add_argument("--K", type=int, default=4096)
    p.add_argument("--b-layout", choices=("col", "row"), default="row")
    p.add_argument("--launches", type=int, default=3)
    p.add_argument("--kernel", choices=("auto", "tcgen05", "simt"), default="tcgen05")
    fields = ("tile_m", "tile_n", "tile_k", "stages", "cluster_m", "persistent", "raster_group", "k_splits", "flags")
    for name in fields:
        p.add_argument(f"--{name.replace('_', '-')}", type=int, default=None)
    p.add_argument("--select", action="store_true", help="start from the library's schedule for the shape")
    p.add_argument("--cublas", action="store_true",
                   help="after this library's launches, the same number of torch.matmul (cuBLAS) launches")
    args = p.parse_args()

    overrides = {name: getattr(args, name) for name in fields if getattr(args, name) is not None}
    overrides["kernel"] = {"auto": _native.KERNEL_AUTO, "tcgen05": _native.KERNEL_TCGEN05,
                           "simt": _native.KERNEL_SIMT}[args.kernel]
    layout = _native.B_ROW if args.b_layout == "row" else _native.B_COL
    cfg = _native.select_config(args.M, args.N, args.K, layout) if args.select else _native.default_config()
    for name, value in overrides.items():
        setattr(cfg, name, int(value))
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(0)
    a = torch.randn((args.M, args.K), generator=g, device=device).to(torch.bfloat16)
    b_shape = (args.N, args.K) if args.b_layout == "col" else (args.K, args.N)
    b = torch.randn(b_shape, generator=g, device=device).to(torch.bfloat16)
    c = torch.empty((args.M, args.N), dtype=torch.bfloat16, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    times = []
    for _ in range(args.launches):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        kg.bf16_gemm(a, b, out=c, b_layout=args.b_layout, config=cfg, stream=stream, status=status)
        stop.record(stream)
        stop.synchronize()
        times.append(start.elapsed_time(stop) * 1e3)
    if int(status.item()) != 0:
        raise SystemExit(f"device status {int(status.item()):#x}")
    cublas_times = []
    if args.cublas:
        b_op = b if args.b_layout == "row" else b.T
        ref = torch.empty_like(c)
        for _ in range(args.launches):
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            torch.matmul(a, b_op, out=ref)
            stop.record(stream)
            stop.synchronize()
            cublas_times.append(start.elapsed_time(stop) * 1e3)
    flops = 2.0 * args.M * args.N * args.K
    layout_code = _native.B_ROW if args.b_layout == "row" else _native.B_COL
    plan = _native.plan(cfg, args.M, args.N, args.K, layout_code)
    print(json.dumps({"config": cfg.as_dict(), "plan": plan, "shape": [args.M, args.N, args.K], "b_layout": args.b_layout,
                      "times_us": times, "median_us": statistics.median(times),
                      "tflops": flops / (statistics.median(times) * 1e-6) / 1e12,
                      "cublas_times_us": cublas_times}))


if __name__ == "__main__":
    main()
