"""Schedule sweep: the 96-point B200 grid, evaluated in parallel over GPUs.

Semantics follow the reference's schedule tuning
(src/kernel_mcts/cute_tuning.py:136-226 and cute_schedule.py:41-88):
* a deterministic grid; a seeded subsample when fewer points are asked for;
* static legality first: statically rejected points are recorded with their
  reasons and are not charged to the tuning budget ``b_tune``;
* every legal point is a charged trial, VALID (with correctness and benchmark)
  or FAILED (with the failure), retained in the report;
* the report carries the best and default schedules and their ratios to a
  same-run cuBLAS measurement.

The grid is BASELINE's: CTA tile M in {128, 256} x N in {128, 256} x K in
{64, 128} x stages in {3, 4, 5, 6} x cluster in {1x1, 2x1, 2x2} = 96 points.
tile_m 256 is a CTA pair (cluster 2x1); 2x2 clusters are rejected statically
because they only pay with multicast loads, which this library never issues.

Run: ``python -m kernel_mcts_b200.sweep --devices 0,1,2,3 --out sweep.json``.
"""

from __future__ import annotations

import argparse
import hashlib
import itertools
import json
import random
import statistics
import sys
import time
from pathlib import Path
from typing import Any, Mapping, Sequence

from . import _native
from .backend import schedule_program
from .domain import ProposalStatus, WorkloadContract
from .serialization import serialize_benchmark
from .workloads import gemm_workload

TILE_M = (128, 256)
TILE_N = (128, 256)
TILE_K = (64, 128)
STAGES = (3, 4, 5, 6)
CLUSTERS = ((1, 1), (2, 1), (2, 2))
DEFAULT_SCHEDULE = {"tile_m": 256, "tile_n": 256, "tile_k": 128, "stages": 3, "cluster_m": 2, "cluster_n": 1}


def schedule_grid(count: int = 96, seed: int = 0) -> list[dict[str, int]]:
    full = [
        {"tile_m": m, "tile_n": n, "tile_k": k, "stages": s, "cluster_m": cm, "cluster_n": cn}
        for m, n, k, s, (cm, cn) in itertools.product(TILE_M, TILE_N, TILE_K, STAGES, CLUSTERS)
    ]
    if count >= len(full):
        return full
    keep = sorted(random.Random(seed).sample(range(len(full)), count))
    return [full[i] for i in keep]


def schedule_id(schedule: Mapping[str, int]) -> str:
    return hashlib.sha256(json.dumps(dict(schedule), sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def static_reasons(schedule: Mapping[str, int], workload: WorkloadContract) -> list[str]:
    shape = workload.shapes[0].dimensions
    layout = _native.B_ROW if workload.metadata.get("b_layout") == "row" else _native.B_COL
    cfg = _native.make_config(**schedule, kernel=_native.KERNEL_TCGEN05)
    code, why = _native.config_legal(cfg, int(shape["M"]), int(shape["N"]), int(shape["K"]), layout)
    return [] if code == _native.KMCTS_OK else [why]


def run_schedule_sweep(
    evaluator: Any,
    workload: WorkloadContract,
    cublas: Mapping[str, Any],
    *,
    schedules: Sequence[Mapping[str, int]] | None = None,
    default: Mapping[str, int] = DEFAULT_SCHEDULE,
    repeat: int = 1,
) -> dict[str, Any]:
    """``evaluator`` has ``evaluate_many`` (an EvaluationPool) or ``evaluate``.
    ``repeat`` > 1 evaluates every legal point that many times (the trial keeps
    the first result; throughput counts them all), to measure evaluations per
    second on a batch large enough to keep every GPU busy."""
    candidates = [dict(s) for s in (schedules if schedules is not None else schedule_grid())]
    trials: list[dict[str, Any]] = []
    legal: list[int] = []
    for ordinal, schedule in enumerate(candidates, 1):
        reasons = static_reasons(schedule, workload)
        trial: dict[str, Any] = {"ordinal": ordinal, "schedule": schedule, "schedule_id": schedule_id(schedule)}
        if reasons:
            trial.update(status="STATICALLY_REJECTED", charged_to_b_tune=False, reasons=reasons)
        else:
            legal.append(len(trials))
        trials.append(trial)

    programs = [schedule_program(**trials[i]["schedule"]) for i in legal]
    prepare = getattr(evaluator, "prepare", None)
    if callable(prepare):
        prepare(workload)  # per-workload state is built before the clock starts
    started = time.monotonic()
    batch = programs * max(1, repeat)
    if hasattr(evaluator, "evaluate_many"):
        results = evaluator.evaluate_many(batch, workload)
    else:
        results = [evaluator.evaluate(p, workload) for p in batch]
    wall = time.monotonic() - started

    attempted = 0
    best = default_trial = None
    for index in range(len(trials)):
        trial = trials[index]
        if trial.get("status") == "STATICALLY_REJECTED":
            trial["b_tune"] = attempted
            continue
        attempted += 1
        result = results[legal.index(index)]
        trial.update(charged_to_b_tune=True, b_tune=attempted)
        if result.status == ProposalStatus.VALID:
            trial.update(status="VALID", result={
                "correctness": {"success": True,
                                "maximum_error": result.correctness.maximum_error if result.correctness else None,
                                "mean_error": result.correctness.mean_error if result.correctness else None},
                "benchmark": serialize_benchmark(result.benchmark),
                "reward": result.reward,
            })
            if best is None or _median(trial) < _median(best):
                best = trial
        else:
            trial.update(status="FAILED", error_type=str(result.invalid_reason or result.status.value),
                         error=str(result.metadata.get("reason", result.metadata.get("error_type", ""))))
        if _same(trial["schedule"], default):
            default_trial = trial

    cublas_median = float(cublas["benchmark"]["median_us"]) if cublas.get("benchmark") else None
    best_median = _median(best) if best else None
    default_median = _median(default_trial) if default_trial and default_trial["status"] == "VALID" else None
    return {
        "status": "ok" if best is not None else "no_valid_schedule",
        "benchmark_id": workload.benchmark_id,
        "method": "deterministic_grid",
        "b_tune": attempted,
        "candidate_count": len(candidates),
        "cublas": dict(cublas),
        "trials": trials,
        "best": _summary(best),
        "default": _summary(default_trial),
        "comparison": {
            "best_latency_ratio_vs_cublas": (best_median / cublas_median
                                             if best_median and cublas_median else None),
            "best_speedup_vs_default": (default_median / best_median
                                        if default_median and best_median else None),
        },
        "evaluations": len(batch),
        "wall_seconds": wall,
        "evaluations_per_second": len(batch) / wall if wall > 0 else None,
    }


def _same(a: Mapping[str, int], b: Mapping[str, int]) -> bool:
    return all(a.get(k) == v for k, v in b.items())


def _median(trial: Mapping[str, Any]) -> float:
    return float(trial["result"]["benchmark"]["median_us"])


def _summary(trial: Mapping[str, Any] | None) -> dict[str, Any] | None:
    if trial is None:
        return None
    out = {k: trial[k] for k in ("status", "schedule", "schedule_id", "b_tune")}
    if trial["status"] == "VALID":
        out["median_us"] = _median(trial)
    return out


def main(argv: Sequence[str] | None = None) -> None:
    from .backend import CudaSm100Backend, CudaSm100Config
    from .pool import EvaluationPool, WorkerSpec
    from .vendor_baselines import VendorBaselineSuite

    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--devices", default="0", help="comma-separated GPU indices, one worker each")
    p.add_argument("--M", type=int, default=4096)
    p.add_argument("--N", type=int, default=4096)
    p.add_argument("--K", type=int, default=4096)
    p.add_argument("--b-layout", choices=("col", "row"), default="row")
    p.add_argument("--inputs", choices=("uniform", "randn", "int"), default="randn")
    p.add_argument("--count", type=int, default=96)
    p.add_argument("--repeat", type=int, default=1, help="evaluate every legal point this many times")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--warmups", type=int, default=20)
    p.add_argument("--measurements", type=int, default=100)
    p.add_argument("--artifact-root", default="/tmp/kmcts-sweep")
    p.add_argument("--subprocess", action="store_true",
                   help="evaluate schedules through the harness executable instead of in process")
    p.add_argument("--out", default=None)
    args = p.parse_args(argv)

    workload = gemm_workload(f"bf16_gemm_{args.M}x{args.N}x{args.K}_b200", args.M, args.N, args.K,
                             b_layout=args.b_layout, inputs=args.inputs)
    devices = [d for d in args.devices.split(",") if d]
    # Same-run cuBLAS on the first device (a harness subprocess; this process
    # never creates a CUDA context).
    import os

    os.environ.setdefault("CUDA_VISIBLE_DEVICES", devices[0])
    vendor_backend = CudaSm100Backend(CudaSm100Config(artifact_root=Path(args.artifact_root) / "vendor",
                                                      warmup_count=args.warmups, measurement_count=args.measurements,
                                                      device_index=int(devices[0])))
    cublas = VendorBaselineSuite(vendor_backend).run(workload)["cublas"]
    cublas_json = {"correctness": cublas.get("correctness"),
                   "benchmark": serialize_benchmark(cublas["benchmark"]) if "benchmark" in cublas else None}
    root_us = cublas["benchmark"].median_us if "benchmark" in cublas else 1.0
    spec = WorkerSpec("kernel_mcts_b200.pool:sm100_evaluator",
                      {"artifact_root": args.artifact_root, "root_us": root_us, "warmup_count": args.warmups,
                       "measurement_count": args.measurements, "inprocess": not args.subprocess})
    with EvaluationPool(devices, spec) as pool:
        report = run_schedule_sweep(pool, workload, cublas_json, schedules=schedule_grid(args.count, args.seed),
                                    repeat=args.repeat)
    report["devices"] = devices
    if args.out:
        Path(args.out).write_text(json.dumps(report, indent=1))
    summary = {k: report[k] for k in ("status", "b_tune", "candidate_count", "best", "default", "comparison",
                                      "evaluations", "wall_seconds", "evaluations_per_second", "devices")}
    summary["cublas_median_us"] = cublas_json["benchmark"]["median_us"] if cublas_json["benchmark"] else None
    print(json.dumps(summary))


if __name__ == "__main__":
    main(sys.argv[1:])
