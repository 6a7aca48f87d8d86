"""Evaluator stand-ins for the pool tests: run in spawned CPU worker
processes, touch no GPU, and fail on the host when a test asks them to."""

from __future__ import annotations

import os
import time
from pathlib import Path

from kernel_mcts_b200.domain import BenchmarkResult, EvaluationResult, ProposalStatus


class FakeEvaluator:
    def __init__(self, device_index: int, marker_dir: str, delay: float) -> None:
        self.device_index = device_index
        self.marker_dir = Path(marker_dir)
        self.delay = delay

    def evaluate(self, program, workload):
        source = program.source
        if "CRASH_ALWAYS" in source:
            os._exit(3)
        if "CRASH_ONCE" in source:
            marker = self.marker_dir / ("crashed-" + source.split(":")[-1])
            if not marker.exists():
                marker.write_text("x")
                os._exit(3)
        if "RAISE" in source:
            raise RuntimeError("backend exploded")
        started = time.time()
        time.sleep(float(source.split("sleep=")[1].split(";")[0]) if "sleep=" in source else self.delay)
        return EvaluationResult(
            status=ProposalStatus.VALID, program=program, state_key=f"key-{source}", reward=1.0,
            benchmark=BenchmarkResult((1.0,), 1.0),
            metadata={"pid": os.getpid(), "visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES"),
                      "device_index": self.device_index, "started": started},
        )


def make(device_index: int, *, marker_dir: str, delay: float = 0.0) -> FakeEvaluator:
    return FakeEvaluator(device_index, marker_dir, delay)


def _profile(self, evaluation, workload, metric_set="lightweight_v1"):
    """Profiles only what this worker evaluated: the lookup the real
    evaluator needs for its compiled artifact."""
    return {"metric_set": metric_set, "profiler": "fake", "pid": os.getpid(),
            "visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES"), "source": evaluation.program.source}


FakeEvaluator.lightweight_profile = _profile
