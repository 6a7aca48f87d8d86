"""The schedule sweep's grid, static legality and report schema (CPU: the
host-only legality check and a fake evaluator; no GPU)."""

from __future__ import annotations

from kernel_mcts_b200.domain import BenchmarkResult, EvaluationResult, InvalidReason, ProposalStatus
from kernel_mcts_b200.sweep import DEFAULT_SCHEDULE, run_schedule_sweep, schedule_grid, static_reasons
from kernel_mcts_b200.workloads import BF16_GEMM_4096_RANDN
from kernel_mcts_b200.backend import schedule_from_source


class FakeEvaluator:
    def __init__(self):
        self.calls = []

    def evaluate_many(self, programs, workload):
        out = []
        for p in programs:
            s = schedule_from_source(p.source)
            self.calls.append(s)
            if s["tile_n"] == 128 and s["stages"] == 6 and s["tile_m"] == 128:
                out.append(EvaluationResult(status=ProposalStatus.INVALID, program=p,
                                            invalid_reason=InvalidReason.LAUNCH_FAILURE))
                continue
            median = 100.0 - s["tile_k"] / 10 - (5 if s["tile_m"] == 256 else 0) + s["stages"] * 0.01
            out.append(EvaluationResult(status=ProposalStatus.VALID, program=p, state_key="k", reward=0.1,
                                        benchmark=BenchmarkResult((median,), median)))
        return out


def test_grid_is_the_96_point_baseline_grid():
    grid = schedule_grid()
    assert len(grid) == 96 and len({tuple(sorted(g.items())) for g in grid}) == 96
    assert schedule_grid(96, seed=123) == grid  # the seeded subsample of 96 is the identity
    sub = schedule_grid(10, seed=1)
    assert len(sub) == 10 and all(s in grid for s in sub) and sub == schedule_grid(10, seed=1)


def test_static_legality_rejects_what_cannot_run():
    w = BF16_GEMM_4096_RANDN
    assert static_reasons(DEFAULT_SCHEDULE, w) == []
    # cluster 2x2: two CTA pairs sharing A over distributed shared memory,
    # compiled for the default tile only; one-CTA 2x2 would need a multicast
    assert static_reasons({**DEFAULT_SCHEDULE, "cluster_n": 2}, w) == []
    assert "cluster_n 2" in static_reasons({**DEFAULT_SCHEDULE, "cluster_n": 2, "tile_k": 64, "stages": 6}, w)[0]
    assert "multicast" in static_reasons({"tile_m": 128, "tile_n": 256, "tile_k": 64, "stages": 4, "cluster_m": 1,
                                          "cluster_n": 2}, w)[0]
    assert "shared memory" in static_reasons({**DEFAULT_SCHEDULE, "stages": 6}, w)[0]
    assert static_reasons({"tile_m": 128, "tile_n": 256, "tile_k": 64, "stages": 4, "cluster_m": 1,
                           "cluster_n": 1}, w) == []


def test_report_schema_charging_and_best():
    fake = FakeEvaluator()
    cublas = {"correctness": {"success": True}, "benchmark": {"median_us": 95.0}}
    report = run_schedule_sweep(fake, BF16_GEMM_4096_RANDN, cublas)
    assert report["candidate_count"] == 96
    statuses = [t["status"] for t in report["trials"]]
    legal = [t for t in report["trials"] if t["status"] != "STATICALLY_REJECTED"]
    assert len(fake.calls) == len(legal) == report["b_tune"] == 19
    assert statuses.count("FAILED") == 1
    rejected = [t for t in report["trials"] if t["status"] == "STATICALLY_REJECTED"]
    assert all(not t["charged_to_b_tune"] and t["reasons"] for t in rejected)
    # b_tune counts charged trials in ordinal order
    charged = [t["b_tune"] for t in legal]
    assert charged == list(range(1, len(legal) + 1))
    assert report["best"]["schedule"]["tile_m"] == 256 and report["best"]["schedule"]["tile_k"] == 128
    assert report["default"]["schedule"] == {**DEFAULT_SCHEDULE}
    assert report["comparison"]["best_latency_ratio_vs_cublas"] == report["best"]["median_us"] / 95.0
    assert report["status"] == "ok" and report["evaluations"] == 19
    assert run_schedule_sweep(FakeEvaluator(), BF16_GEMM_4096_RANDN, cublas, repeat=3)["evaluations"] == 57
