"""PoolAutotuner and PoolDriftMonitor on CPU (fake evaluators, no GPU).

The trial order, budget, skip rule, best choice and events follow the
reference's PostSearchAutotuner (src/kernel_mcts/autotuning.py:133-211); when
the reference source tree is present the two are compared trial by trial.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

from kernel_mcts_b200.autotune import (
    PoolAutotuner,
    PoolDriftMonitor,
    TuningConfig,
    drift,
    parse_tuning_parameters,
    render_configuration,
)
from kernel_mcts_b200.backend import schedule_program
from kernel_mcts_b200.domain import BenchmarkResult, EvaluationResult, KernelProgram, ProposalStatus
from kernel_mcts_b200.pool import EvaluationPool, WorkerSpec
from kernel_mcts_b200.workloads import gemm_workload

WORKLOAD = gemm_workload("tune_test", 256, 256, 256)

SOURCE = """
// KERNEL_MCTS_TUNE BLOCK_M = 64, 128, 256
// KERNEL_MCTS_TUNE STAGES = 2, 3, 4
#define BLOCK_M 128
#define STAGES 3
extern "C" __global__ void bf16_gemm_root(const void* A, const void* B, void* C, int M, int N, int K) {}
"""


def defines(source: str) -> dict[str, int]:
    out = {}
    for line in source.splitlines():
        parts = line.split()
        if len(parts) == 3 and parts[0] == "#define":
            out[parts[1]] = int(parts[2])
    return out


def valid(program: KernelProgram, reward: float) -> EvaluationResult:
    return EvaluationResult(ProposalStatus.VALID, program=program, state_key=f"k{hash(program.source)}",
                            reward=reward, benchmark=BenchmarkResult((1.0,), 1.0))


class Batch:
    """Records each evaluate_many call; reward = BLOCK_M / 64 + STAGES / 10."""

    def __init__(self) -> None:
        self.calls: list[list[KernelProgram]] = []

    def evaluate_many(self, programs, workload):
        self.calls.append(list(programs))
        return [valid(p, d["BLOCK_M"] / 64 + d["STAGES"] / 10) for p, d in ((p, defines(p.source)) for p in programs)]

    def evaluate(self, program, workload):
        return self.evaluate_many([program], workload)[0]


class Events:
    def __init__(self) -> None:
        self.seen: list[tuple[str, dict]] = []

    def emit(self, kind, payload):
        self.seen.append((kind, dict(payload)))


def test_all_trials_go_to_one_batch_and_the_best_is_kept():
    batch, events = Batch(), Events()
    baseline = valid(KernelProgram(SOURCE), 128 / 64 + 0.3)
    result = PoolAutotuner(batch, WORKLOAD, TuningConfig(budget=5, method="random", seed=3), events).run(baseline)
    assert len(batch.calls) == 1 and len(batch.calls[0]) == 5
    assert result.used == 5 and len({json.dumps(t.parameters, sort_keys=True) for t in result.trials}) == 5
    assert all(t.parameters != {"BLOCK_M": 128, "STAGES": 3} for t in result.trials)  # current config dropped
    best_trial = max((t for t in result.trials), key=lambda t: t.evaluation.reward)
    if best_trial.evaluation.reward > baseline.reward:
        assert result.best is best_trial.evaluation and result.best_parameters == best_trial.parameters
        assert result.improved
    kinds = [k for k, _ in events.seen]
    assert kinds == ["tuning_started"] + ["tuning_trial"] * 5 + ["tuning_completed"]
    assert events.seen[0][1]["configuration_count"] == 5
    assert [p["trial"] for k, p in events.seen if k == "tuning_trial"] == [1, 2, 3, 4, 5]


def test_grid_order_and_budget():
    tuner = PoolAutotuner(Batch(), WORKLOAD, TuningConfig(budget=3, method="grid"))
    _, plan = tuner.plan(KernelProgram(SOURCE))
    assert plan == [{"BLOCK_M": 64, "STAGES": 2}, {"BLOCK_M": 64, "STAGES": 3}, {"BLOCK_M": 64, "STAGES": 4}]


def test_unannotated_program_is_skipped():
    events = Events()
    result = PoolAutotuner(Batch(), WORKLOAD, TuningConfig(budget=4), events).run(
        valid(KernelProgram("__global__ void bf16_gemm_root() {}"), 1.0))
    assert result.skipped_reason and result.used == 0 and events.seen[0][0] == "tuning_skipped"


def test_annotation_errors():
    with pytest.raises(ValueError):
        parse_tuning_parameters(KernelProgram("// KERNEL_MCTS_TUNE X = 1, 2\n"))  # no define
    with pytest.raises(ValueError):
        parse_tuning_parameters(KernelProgram("// KERNEL_MCTS_TUNE X = 1, 2\n// KERNEL_MCTS_TUNE X = 3, 4\n"
                                              "#define X 1\n"))
    with pytest.raises(ValueError):
        render_configuration(KernelProgram("#define X 1\n"), {"Y": 2})


def test_schedule_programs_tune_schedule_fields():
    program = schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3)
    names = [p.name for p in parse_tuning_parameters(program)]
    assert names == ["tile_n", "tile_k", "stages", "raster_group"]
    tuner = PoolAutotuner(Batch(), WORKLOAD, TuningConfig(budget=200, method="grid"))
    _, plan = tuner.plan(program)
    assert len(plan) == 2 * 2 * 4 * 5 - 1  # every combination but the current one (raster_group 8)
    rendered = json.loads(render_configuration(program, {"tile_n": 128, "stages": 4}).source)
    assert rendered == {"tile_m": 256, "cluster_m": 2, "tile_n": 128, "tile_k": 128, "stages": 4}


def test_trial_order_matches_the_reference_autotuner():
    from reference_tree import REFERENCE_SRC as ref_root

    if not ref_root.exists():
        pytest.skip("reference source tree not present")
    sys.path.insert(0, str(ref_root))
    try:
        from kernel_mcts import autotuning as ref
        from kernel_mcts import domain as ref_domain
    except Exception as error:  # the reference needs packages this image may lack
        pytest.skip(f"reference autotuner not importable: {error}")
    finally:
        sys.path.remove(str(ref_root))

    class Sequential:
        def __init__(self):
            self.order = []

        def evaluate(self, program, workload):
            self.order.append(defines(program.source))
            return ref_domain.EvaluationResult(ref_domain.ProposalStatus.INVALID,
                                               invalid_reason=ref_domain.InvalidReason.OTHER)

    class Sink:
        def emit(self, *_):
            pass

    for method, seed, budget in (("random", 0, 4), ("random", 7, 8), ("grid", 0, 6)):
        seq = Sequential()
        baseline = ref_domain.EvaluationResult(ref_domain.ProposalStatus.INVALID,
                                               program=ref_domain.KernelProgram(SOURCE),
                                               invalid_reason=ref_domain.InvalidReason.OTHER)
        ref.PostSearchAutotuner(seq, None, ref.TuningConfig(budget, method, seed), Sink()).run(baseline)
        _, plan = PoolAutotuner(Batch(), WORKLOAD, TuningConfig(budget, method, seed)).plan(KernelProgram(SOURCE))
        assert plan == seq.order, (method, seed)


def test_autotuner_fans_out_over_a_cpu_pool(tmp_path):
    """Through a real EvaluationPool with two spawned CPU workers."""
    source = SOURCE.replace("extern", "// sleep=0.05;\nextern")
    with EvaluationPool([0, 1], WorkerSpec("pool_fakes:make", {"marker_dir": str(tmp_path)})) as pool:
        result = PoolAutotuner(pool, WORKLOAD, TuningConfig(budget=6, method="grid")).run(
            valid(KernelProgram(source), 0.5))
        monitor = PoolDriftMonitor(pool)
        again = monitor.remeasure(result.trials[0].evaluation, WORKLOAD)
    assert result.used == 6 and all(t.evaluation.status == ProposalStatus.VALID for t in result.trials)
    assert {t.evaluation.metadata["visible_devices"] for t in result.trials} == {"0", "1"}
    assert monitor.calls == 1 and again.status == ProposalStatus.VALID
    assert drift(result.trials[0].evaluation, again) == pytest.approx(0.0)

