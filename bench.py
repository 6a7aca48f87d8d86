"""Headline benchmark: 4096^3 BF16 GEMM on B200.

Metric: "4096³ BF16 GEMM median µs & TFLOP/s (% BF16 peak) vs
same-run cuBLAS; evals/sec @1–8 GPU".  ``value`` is TFLOP/s of the whole job:
N GPUs each run the same GEMM (one candidate evaluation per GPU, no
collective on the data path: weak scaling); value = N * 2MNK / max-over-ranks
median launch time.

Timing protocol: W warm-up launches, then K steps; each step flushes L2
(writes a 512 MiB buffer; the 64 MiB of inputs would otherwise stay
L2-resident) and times one launch with a CUDA event pair on the launching
stream.  Same protocol, same run, for cuBLAS (torch.matmul).

``--impl reference`` times the reference's CPU path for this workload
(torch CPU BF16 matmul, all host threads) on rank 0 and prints the same line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gpu-kernel-mcts_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "4096³ BF16 GEMM median µs & TFLOP/s (% BF16 peak) vs same-run cuBLAS; evals/sec @1–8 GPU"
UNIT = "TFLOP/s"
M = N = K = 4096
FLOPS = 2.0 * M * N * K
L2_FLUSH_BYTES = 512 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--b-layout", choices=("row", "col"), default="row",
                   help="row: BASELINE config (A/B row-major); col: the reference contract")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-evals", action="store_true", help="skip the evaluation-throughput pass")
    p.add_argument("--eval-repeat", type=int, default=3)
    p.add_argument("--no-sharded", action="store_true", help="skip the sharded 8192x28672x8192 GEMM")
    p.add_argument("--no-skinny", action="store_true", help="skip the HBM-bound skinny shapes")
    p.add_argument("--no-shapes", action="store_true", help="skip the one-shape-per-class comparison")
    return p.parse_args()


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profiled_traffic() -> float | None:
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "gemm_tcgen05_pair_4096.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons through NVML every
    ~2 ms while the timed region runs (nvidia-smi is too slow to catch a
    region of a few tens of ms)."""

    # NVML clocks-event reason bits (nvml.h: nvmlClocksEventReason*).
    REASONS = {
        0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x4: "sw_power_cap",
        0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int) -> None:
        self.device_index = device_index
        self.samples: list[tuple[float, int, float]] = []
        self.max_mhz: float | None = None
        self.error: str | None = None
        self._handle = None
        self._nvml = None
        self._stop = threading.Event()
        self._first = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _sample(self) -> None:
        nvml, handle = self._nvml, self._handle
        sm = float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM))
        reasons = int(nvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
        power = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
        self.samples.append((sm, reasons, power))

    def _run(self) -> None:
        try:
            while True:  # at least one sample, then every ~2 ms until stopped
                self._sample()
                self._first.set()
                if self._stop.wait(0.002):
                    break
            self._sample()  # and one as the region ends
        except Exception as error:  # NVML refused mid-run: report it, do not fail the bench
            self.error = f"{type(error).__name__}: {error}"
        finally:
            self._first.set()

    def __enter__(self):
        # NVML is opened here, before the timed region: its first call can take
        # longer than a short region lasts.
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.device_index]) if visible else self.device_index
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nvml = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM))
        except Exception as error:  # NVML missing or refused: report it, do not fail the bench
            self.error = f"{type(error).__name__}: {error}"
            return self
        self._thread.start()
        self._first.wait(timeout=5.0)
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread.is_alive():
            self._thread.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"],
                    "samples": 0, "error": self.error}
        reasons = sorted({name for _, bits, _ in self.samples for bit, name in self.REASONS.items() if bits & bit})
        return {
            "sm_mhz": statistics.median(s for s, _, _ in self.samples),
            "sm_min_mhz": min(s for s, _, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(self.samples),
            "power_w_max": max(p for _, _, p in self.samples),
            "source": "NVML, ~2 ms polling during the timed region",
        }


# ---------------------------------------------------------------- reference arm


def cpu_matmul_tflops(seconds: float, threads: int | None = None) -> dict:
    """The reference's CPU path, torch CPU BF16 matmul,
    on a bounded row-sample of the 4096^3 workload, repeated for ~`seconds`."""
    import torch

    from oracle import oracle

    if threads:
        torch.set_num_threads(threads)
    rows = 256
    a, b = oracle.randn_inputs(M, N, K, seed=0, b_layout="row")
    sample_a = a[:rows].contiguous()
    torch.matmul(sample_a, b)  # warm-up
    # Grow the sample until one call takes >= 0.2 s (or covers all of M).
    while True:
        t0 = time.perf_counter()
        torch.matmul(sample_a, b)
        dt = time.perf_counter() - t0
        if dt >= 0.2 or rows >= M:
            break
        rows = min(M, rows * 2)
        sample_a = a[:rows].contiguous()
    times = []
    start = time.perf_counter()
    while time.perf_counter() - start < seconds and len(times) < 1000:
        t0 = time.perf_counter()
        torch.matmul(sample_a, b)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {
        "value": 2.0 * rows * N * K / med / 1e12,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "rows": rows,
        "median_s": med,
        "calls": len(times),
    }


def run_reference(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from oracle import oracle

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    a, b = oracle.randn_inputs(M, N, K, seed=0, b_layout="row")
    # Step = one row-sample of the workload sized to ~0.25 s of CPU work.
    rows = 128
    sample = a[:rows].contiguous()
    torch.matmul(sample, b)
    while rows < M:
        t0 = time.perf_counter()
        torch.matmul(sample, b)
        if time.perf_counter() - t0 >= 0.25:
            break
        rows = min(M, rows * 2)
        sample = a[:rows].contiguous()
    for _ in range(args.warmup):
        torch.matmul(sample, b)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        torch.matmul(sample, b)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    value = 2.0 * rows * N * K / med / 1e12
    sample_desc = (f"torch CPU BF16 matmul of rows [0,{rows}) of the 4096^3 N(0,1) workload "
                   f"(A[{rows},4096] @ B[4096,4096] row-major), median of {args.steps}")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": med * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: torch.randn seed 0 cast to bf16",
        "config": {"workload": "bf16_gemm_4096", "M": M, "N": N, "K": K, "b_layout": "row",
                   "sample_rows": rows, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "reference", "sample": sample_desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------- our arm


def time_launches(fn, steps: int, stream, flush) -> list[float]:
    """Per-launch event timing (µs) with an L2 flush before each launch."""
    return time_interleaved([fn], steps, stream, flush)[0]


def time_interleaved(fns, steps: int, stream, flush) -> list[list[float]]:
    """Per-launch event timing (µs) of several callables, interleaved step by
    step (flush, fn0, flush, fn1, ...) so clock and power drift hit all of
    them alike.  Events are recorded on the launching stream."""
    import torch

    starts = [[torch.cuda.Event(enable_timing=True) for _ in range(steps)] for _ in fns]
    stops = [[torch.cuda.Event(enable_timing=True) for _ in range(steps)] for _ in fns]
    with torch.cuda.stream(stream):
        for i in range(steps):
            for j, fn in enumerate(fns):
                flush.fill_((i + j) & 0xFF)
                starts[j][i].record(stream)
                fn()
                stops[j][i].record(stream)
    stream.synchronize()
    return [[s.elapsed_time(e) * 1e3 for s, e in zip(starts[j], stops[j])] for j in range(len(fns))]


SKINNY_SHAPES = ((16, 8192, 8192), (128, 16384, 4096))

# One shape per class of the library's schedule selection, beside same-run
# cuBLAS: where each class stands (the mid-size class is the one behind).
SHAPE_CLASSES = (
    ("M <= 32, long K: K splits added in shared memory", (16, 1024, 16384)),
    ("33 <= M <= 64: 64 rows of A per tile", (64, 8192, 8192)),
    ("one row of pair tiles: B at L2 evict-first", (256, 16384, 4096)),
    ("two rows of pair tiles: B at L2 evict-first", (512, 8192, 8192)),
    ("N <= 128: one CTA per 128 x 128 tile, A at L2 evict-first", (16384, 128, 4096)),
    ("two columns of pair tiles: A at L2 evict-first", (28672, 256, 4096)),
    ("rectangular, CTA pair", (8192, 4096, 4096)),
    ("mid-size, few tiles over a long K: K splits added across a cluster", (512, 512, 8192)),
)

FLAG_NAMES = (("B_EVICT_FIRST", 8), ("A_EVICT_FIRST", 128), ("SPLIT_CLUSTER", 64), ("SPLIT_SCATTER", 256),
              ("SWAP_AB", 16))


def shape_classes(device, stream, flush, steps: int = 40) -> list[dict]:
    """The NULL-config call (the library's selection) on one shape per class
    against same-run cuBLAS, L2 flushed, interleaved; B row-major, N(0,1)
    seed 0.  `speedup` = cuBLAS mean / our mean (above 1: ahead)."""
    import torch

    from kernel_mcts_b200 import _native
    from kernel_mcts_b200 import gemm as kg

    rows = []
    for name, (m, n, k) in SHAPE_CLASSES:
        g = torch.Generator(device=device).manual_seed(0)
        a = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
        b = torch.randn((k, n), generator=g, device=device).to(torch.bfloat16)
        c = torch.empty((m, n), dtype=torch.bfloat16, device=device)
        c_ref = torch.empty_like(c)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        cfg = _native.select_config(m, n, k, _native.B_ROW)
        ours = kg.PreparedGemm(a, b, c, b_layout="row", config=cfg, stream=stream, status=status)

        def cublas():
            torch.matmul(a, b, out=c_ref)

        with torch.cuda.stream(stream):
            for _ in range(3):
                ours.launch()
                cublas()
        ours_us, cublas_us = time_interleaved([ours.launch, cublas], steps, stream, flush)
        if int(status.item()) != 0:
            raise RuntimeError(f"device status {int(status.item()):#x}")
        parity = kg.compare(c, c_ref, stream=stream)
        mean, mean_ref = statistics.fmean(ours_us), statistics.fmean(cublas_us)
        rows.append({
            "class": name, "shape": [m, n, k],
            "schedule": {"tile_m": cfg.tile_m, "tile_n": cfg.tile_n, "tile_k": cfg.tile_k, "stages": cfg.stages,
                         "k_splits": max(1, cfg.k_splits),
                         "flags": [nm for nm, bit in FLAG_NAMES if cfg.flags & bit]},
            "median_us": statistics.median(ours_us), "cublas_median_us": statistics.median(cublas_us),
            "mean_us": mean, "cublas_mean_us": mean_ref, "speedup": mean_ref / mean,
            "tflops": 2.0 * m * n * k / (mean * 1e-6) / 1e12,
            "parity_vs_cublas": {"success": parity.success, "max_ulp": parity.max_ulp},
        })
        del a, b, c, c_ref
    return rows


def skinny_gemms(device, stream, flush, steps: int = 60) -> dict:
    """HBM-bound shapes (north_star: HBM GB/s for the skinny shapes).  Our
    call with a NULL config (the library's shape selection: split K here)
    against same-run cuBLAS, L2 flushed, interleaved.  GB/s = the minimum
    bytes (A and B read once, C written once) / median time, against the
    measured HBM copy bandwidth.  Means are reported beside the medians: the
    event clock steps about 1 us, which is 3% of these launches."""
    import torch

    from kernel_mcts_b200 import _native
    from kernel_mcts_b200 import gemm as kg

    peaks, kind = load_peaks()
    hbm = float(peaks["hbm_gbs"])
    rows = []
    for m, n, k in SKINNY_SHAPES:
        g = torch.Generator(device=device).manual_seed(0)
        a = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
        b = torch.randn((k, n), generator=g, device=device).to(torch.bfloat16)
        c = torch.empty((m, n), dtype=torch.bfloat16, device=device)
        c_ref = torch.empty_like(c)
        status = torch.zeros(1, dtype=torch.int32, device=device)

        def ours():
            kg.bf16_gemm(a, b, out=c, b_layout="row", stream=stream, status=status)

        def cublas():
            torch.matmul(a, b, out=c_ref)

        with torch.cuda.stream(stream):
            for _ in range(3):
                ours()
                cublas()
        ours_us, cublas_us = time_interleaved([ours, cublas], steps, stream, flush)
        if int(status.item()) != 0:
            raise RuntimeError(f"device status {int(status.item()):#x}")
        parity = kg.compare(c, c_ref, stream=stream)
        min_bytes = 2 * (m * k + k * n + m * n)
        med, med_ref = statistics.median(ours_us), statistics.median(cublas_us)
        mean, mean_ref = statistics.fmean(ours_us), statistics.fmean(cublas_us)
        cfg = _native.select_config(m, n, k, _native.B_ROW)
        rows.append({
            "shape": [m, n, k],
            "schedule": {"tile_m": cfg.tile_m, "tile_n": cfg.tile_n, "tile_k": cfg.tile_k, "stages": cfg.stages,
                         "k_splits": max(1, cfg.k_splits),
                         "splits_add_in_shared_memory": bool(cfg.flags & _native.FLAG_SPLIT_CLUSTER)},
            "median_us": med, "cublas_median_us": med_ref,
            "mean_us": mean, "cublas_mean_us": mean_ref,
            "frac_of_hbm_from_mean": min_bytes / (mean * 1e-6) / 1e9 / hbm,
            "gbs": min_bytes / (med * 1e-6) / 1e9, "cublas_gbs": min_bytes / (med_ref * 1e-6) / 1e9,
            "frac_of_hbm": min_bytes / (med * 1e-6) / 1e9 / hbm,
            "parity_vs_cublas": {"success": parity.success, "max_ulp": parity.max_ulp,
                                 "n_gt_1ulp": parity.ulp_hist[2] + parity.ulp_hist[3]},
        })
    return {"bound": "hbm", "peak_gbs": hbm, "peak_source": f"{kind} hbm_gbs (copy)",
            "timing": "per-launch CUDA events, L2 flushed, interleaved with cuBLAS, 60 launches each: medians "
                      "(and means)", "shapes": rows}


def evaluation_throughput(device, world: int, local_rank: int, layout: str, repeat: int) -> dict:
    """the 96-point schedule sweep, one evaluator per GPU
    (this rank's), reported as src/kernel_mcts/cute_tuning.py:136-226 reports
    it: every point's static legality first (rejections are recorded with
    their reasons and not charged to b_tune), then every legal point compiled
    (for a prebuilt schedule: legality and kernel selection, no nvcc),
    correctness-checked against cuBLAS and timed with the harness protocol
    (10 warm-ups, 30 event-timed launches); best, default and their ratios to
    this run's cuBLAS median.  The legal points run ``repeat`` times so the
    batch keeps the GPU busy; evals/sec = all ranks' evaluations / the slowest
    rank's wall time."""
    import torch
    import torch.distributed as dist

    from kernel_mcts_b200.domain import BenchmarkResult
    from kernel_mcts_b200.evaluation import BackendKernelEvaluator, EvaluationContext
    from kernel_mcts_b200.inprocess import InProcessSm100Backend
    from kernel_mcts_b200.sweep import run_schedule_sweep, schedule_grid
    from kernel_mcts_b200.workloads import gemm_workload

    workload = gemm_workload("bf16_gemm_4096_randn_b200", M, N, K, b_layout=layout, inputs="randn")
    backend = InProcessSm100Backend(warmup_count=10, measurement_count=30)
    evaluator = BackendKernelEvaluator(backend=backend, root_benchmark=BenchmarkResult((100.0,), 100.0),
                                       context=EvaluationContext(f"rank{local_rank}", "bench", {}, {}))
    evaluator.prepare(workload)
    cublas_us = cublas_protocol_median(device, layout, warmups=10, measurements=30)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize(device)
    cublas = {"benchmark": {"median_us": cublas_us},
              "protocol": "torch.matmul under the evaluations' protocol (10 warm-ups, 30 event-timed launches, "
                          "no L2 flush), on this GPU"}
    report = run_schedule_sweep(evaluator, workload, cublas, schedules=schedule_grid(96, 0), repeat=repeat)
    torch.cuda.synchronize(device)
    wall = torch.tensor([report["wall_seconds"]], dtype=torch.float64, device=device)
    valid = torch.tensor([sum(t.get("status") == "VALID" for t in report["trials"]) * repeat],
                         dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(wall, op=dist.ReduceOp.MAX)
        dist.all_reduce(valid, op=dist.ReduceOp.SUM)
    total = report["evaluations"] * world
    rejected: dict[str, int] = {}
    for trial in report["trials"]:
        if trial.get("status") == "STATICALLY_REJECTED":
            for reason in trial["reasons"]:
                rejected[reason] = rejected.get(reason, 0) + 1
    return {
        "value": total / float(wall.item()),
        "unit": "evaluations/s",
        "evaluations": total,
        "valid": int(valid.item()),
        "wall_s": float(wall.item()),
        "per_evaluation": "compile (static legality + kernel selection: prebuilt schedules run no nvcc) + "
                          "correctness vs cuBLAS + 10 warm-up and 30 event-timed launches",
        "grid_points": report["candidate_count"],
        "legal": report["b_tune"],
        "statically_rejected": report["candidate_count"] - report["b_tune"],
        "rejection_reasons": rejected,
        "best": report["best"],
        "default": report["default"],
        "comparison": report["comparison"],
        "cublas_median_us": cublas_us,
        "repeat": repeat,
        "gpus": world,
    }


def cublas_protocol_median(device, layout: str, warmups: int, measurements: int) -> float:
    """Same-run cuBLAS (torch.matmul) at 4096^3 N(0,1) under the evaluation
    protocol of kmcts_time_gemm: warm-ups, one synchronise, then per launch an
    event pair and a synchronise.  Median in microseconds."""
    import torch

    g = torch.Generator(device=device).manual_seed(1)
    a = torch.randn((M, K), generator=g, device=device).to(torch.bfloat16)
    b = torch.randn((K, N) if layout == "row" else (N, K), generator=g, device=device).to(torch.bfloat16)
    b_op = b if layout == "row" else b.T
    c = torch.empty((M, N), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmups):
        torch.matmul(a, b_op, out=c)
    torch.cuda.synchronize(device)
    times = []
    for _ in range(measurements):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        torch.matmul(a, b_op, out=c)
        stop.record(stream)
        stop.synchronize()
        times.append(start.elapsed_time(stop) * 1e3)
    return statistics.median(times)


def sharded_gemm(device, world: int, local_rank: int, steps: int = 5, warmup: int = 2) -> dict:
    """8192x28672x8192, N(0, 0.02^2) BF16, B and C sharded by
    N columns over the ranks.  The fused kernel (GEMM + all-gather of C over
    NVLink peer stores), the copy-engine all-gather (row-block GEMMs whose
    finished rows the copy engines send to every rank's C) and the same GEMM
    followed by NCCL all_gather and a re-layout; aggregate TFLOP/s = 2MNK /
    max-over-ranks median time.

    Outside the timed region every rank checks its full C, on the first and
    last 256 rows (the first and last row tiles) and all columns, bit for bit
    against the single-GPU kernel run on those rows of the whole problem;
    ``bit_identical`` is the AND over ranks and paths."""
    import torch
    import torch.distributed as dist

    from kernel_mcts_b200 import gemm as kg
    from kernel_mcts_b200.sharded import ShardedGemm

    m, n, k = 8192, 28672, 8192
    if world == 1:
        dist_owned = False
        if not dist.is_initialized():
            dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29555", rank=0, world_size=1)
            dist_owned = True
    g = torch.Generator(device=device).manual_seed(0)  # the same A and B on every rank
    a = (torch.randn((m, k), generator=g, device=device) * 0.02).to(torch.bfloat16)
    b_full = (torch.randn((k, n), generator=g, device=device) * 0.02).to(torch.bfloat16)
    sg = ShardedGemm(m, n, k, b_layout="row")
    b_shard = b_full[:, sg.col0:sg.col1].contiguous()
    rows = torch.cat([torch.arange(0, 256, device=device), torch.arange(m - 256, m, device=device)])
    single = kg.bf16_gemm(a[rows].contiguous(), b_full, b_layout="row", config=sg.config)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    out = {"workload": "8192x28672x8192 N(0,0.02) bf16, B/C sharded by N", "gpus": world}
    identical = True
    try:
        for name, fn in (("fused", sg.run), ("copy_engines", sg.run_copy_engines), ("nccl", sg.run_nccl)):
            if world == 1 and name != "fused":
                continue
            for _ in range(warmup):
                fn(a, b_shard)
                sg.finish()
            times = []
            for _ in range(steps):
                if world > 1:
                    dist.barrier(device_ids=[local_rank])
                torch.cuda.synchronize(device)
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record(stream)
                fn(a, b_shard)
                s1.record(stream)
                sg.finish()
                times.append(s0.elapsed_time(s1) * 1e3)
            med = torch.tensor([statistics.median(times)], dtype=torch.float64, device=device)
            if world > 1:
                dist.all_reduce(med, op=dist.ReduceOp.MAX)
            out[f"{name}_median_us"] = float(med.item())
            out[f"{name}_tflops"] = 2.0 * m * n * k / (float(med.item()) * 1e-6) / 1e12
            # Untimed: this rank's full C (every rank's columns) on the sampled
            # rows against the single-GPU kernel; AND over ranks.
            same = torch.tensor([1 if torch.equal(sg.c[rows].view(torch.int16), single.view(torch.int16)) else 0],
                                dtype=torch.int32, device=device)
            if world > 1:
                dist.all_reduce(same, op=dist.ReduceOp.MIN)
            out[f"{name}_bit_identical"] = bool(same.item())
            identical = identical and bool(same.item())
        out["bit_identical"] = identical
        out["bit_identity_check"] = ("every rank's full C, rows [0,256) and [8192-256,8192), all 28672 columns, "
                                     "against the single-GPU kernel on those rows of the whole problem")
    finally:
        sg.close()
        if world == 1 and dist_owned:
            dist.destroy_process_group()
    return out


def run_ours(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))

    from kernel_mcts_b200 import _native
    from kernel_mcts_b200 import gemm as kg
    from oracle import oracle

    layout = args.b_layout
    a_cpu, b_cpu = oracle.randn_inputs(M, N, K, seed=0, b_layout=layout)
    a, b = a_cpu.to(device), b_cpu.to(device)
    c = torch.empty((M, N), dtype=torch.bfloat16, device=device)
    c_ref = torch.empty_like(c)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)
    cfg = _native.default_config()
    plan = _native.plan(cfg, M, N, K, _native.B_ROW if layout == "row" else _native.B_COL)
    status = torch.zeros(1, dtype=torch.int32, device=device)

    def ours():
        kg.bf16_gemm(a, b, out=c, b_layout=layout, config=cfg, stream=stream, status=status)

    b_for_torch = b if layout == "row" else b.T

    def cublas():
        torch.matmul(a, b_for_torch, out=c_ref)

    # Warm-up (untimed).
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            ours()
            cublas()
    stream.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    with ClockSampler(local_rank) as clocks:
        barrier()
        launches0 = _native.launch_count()
        ours_us, cublas_us = time_interleaved([ours, cublas], args.steps, stream, flush)
        launches = _native.launch_count() - launches0
        barrier()
    if int(status.item()) != 0:
        raise RuntimeError(f"device status {int(status.item()):#x}")

    # Untimed correctness of the measured kernel against same-run cuBLAS.
    parity = kg.compare(c, c_ref, stream=stream).as_dict()

    med_ours = statistics.median(ours_us)
    med_cublas = statistics.median(cublas_us)
    mean_ours = statistics.fmean(ours_us)
    t = torch.tensor([med_ours, med_cublas, mean_ours], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    med_ours, med_cublas, mean_ours = (float(v) for v in t.tolist())

    # End-to-end through the public API with host buffers: pinned H2D of A and
    # B, the GEMM, D2H of C — all inside the event-timed region.
    e2e = None
    if not args.no_e2e:
        ha = a_cpu.pin_memory()
        hb = b_cpu.pin_memory()
        hc = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()

        def end_to_end():
            # The public host-buffer call: A row blocks and B column blocks
            # alternate on the link; each C block's GEMM and copy back overlap
            # the rest of the copies in.
            kg.bf16_gemm_host(ha, hb, hc, a, b, c, b_layout=layout, stream=stream, status=status)

        with torch.cuda.stream(stream):
            for _ in range(3):
                end_to_end()
        stream.synchronize()
        e2e_steps = max(5, min(args.steps, 30))
        e2e_us = time_launches(end_to_end, e2e_steps, stream, flush)
        e2e_med = statistics.median(e2e_us)
        te = torch.tensor([e2e_med], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_med = float(te.item())
        e2e = {
            "value": world * FLOPS / (e2e_med * 1e-6) / 1e12,
            "unit": UNIT,
            "h2d_bytes_per_step": int(a.numel() * 2 + b.numel() * 2),
            "d2h_bytes_per_step": int(c.numel() * 2),
            "median_us": e2e_med,
            "steps": e2e_steps,
        }

    skinny = None
    if not args.no_skinny:
        skinny = skinny_gemms(device, stream, flush)
    classes = None
    if not args.no_shapes:
        classes = shape_classes(device, stream, flush)

    evaluations = None
    if not args.no_evals:
        evaluations = evaluation_throughput(device, world, local_rank, layout, args.eval_repeat)
    sharded = None
    if not args.no_sharded:
        sharded = sharded_gemm(device, world, local_rank)

    if rank == 0:
        peaks, peaks_kind = load_peaks()
        # Same median launch time as `value` (per GPU), so frac = value / (N * peak).
        achieved = FLOPS / (med_ours * 1e-6) / 1e12
        peak = float(peaks["bf16_tflops"])
        value = world * FLOPS / (med_ours * 1e-6) / 1e12
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu_info = cpu_matmul_tflops(seconds=12.0)
            cpu = {
                "value": cpu_info["value"],
                "unit": UNIT,
                "cores": cpu_info["cores"],
                "kind": "reference",
                "sample": (f"torch CPU BF16 matmul (the reference's CPU path) on rows [0,{cpu_info['rows']}) "
                           f"of the 4096^3 N(0,1) workload, median of {cpu_info['calls']} calls over ~12 s"),
            }
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": med_ours / 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: torch.randn seed 0 (CPU generator) cast to bf16",
            "config": {
                "workload": "bf16_gemm_4096 (BASELINE config 2: M=N=K=4096, N(0,1) seed 0)",
                "M": M, "N": N, "K": K,
                "b_layout": layout,
                "kernel": ("tcgen05 persistent %s %dx%dx%d, %d stages"
                           % ("CTA-pair (cta_group::2)" if cfg.tile_m == 256 else "1-CTA",
                              cfg.tile_m, cfg.tile_n, cfg.tile_k, cfg.stages)),
                "plan": plan,
                "parallelism": f"replicas x{world} (one evaluation per GPU, no collective)",
                "timing": "per-launch CUDA events on the launching stream, median; ours and cuBLAS interleaved step by step",
                "l2": "flushed before every timed launch (512 MiB write)",
            },
            "median_us": med_ours,
            "cublas_median_us": med_cublas,
            "speedup_vs_cublas": med_cublas / med_ours,
            "pct_bf16_peak": 100.0 * (FLOPS / (med_ours * 1e-6) / 1e12) / peak,
            "parity_vs_cublas": parity,
            "roofline": {
                "bound": "tensor",
                "achieved": achieved,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "traffic": profiled_traffic(),
                "peak_source": f"{peaks_kind} bf16_tflops (burst; kernel timed alone)",
                "algorithmic_flops_per_launch": FLOPS,
                "launch_time": "median of the event-timed launches (as value)",
                "achieved_from_mean": FLOPS / (mean_ours * 1e-6) / 1e12,
            },
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "evaluations": evaluations,
            "sharded_gemm": sharded,
            "skinny_hbm": skinny,
            "shape_classes": classes,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
