"""Post-search autotuning over the evaluation pool, and drift re-measurement.

The reference tunes the final best kernel one trial at a time
(src/kernel_mcts/autotuning.py:133-211, ``PostSearchAutotuner``): it reads the
``// KERNEL_MCTS_TUNE NAME = a, b, c`` annotations and their ``#define NAME
v`` lines (:80-101), renders each configuration by rewriting the defines
(:104-130), drops the current one, shuffles (``random``) or keeps grid order,
cuts to the budget, evaluates each trial and keeps the best reward, emitting
``tuning_skipped`` / ``tuning_started`` / ``tuning_trial`` /
``tuning_completed`` events.

:class:`PoolAutotuner` keeps that contract (same annotation format, same
trial order, same events and result types) but renders every trial first and
submits them in one ``evaluate_many`` call, so an :class:`~.pool.EvaluationPool`
runs them one per GPU.  Schedule programs (backend ``kmcts_sm100``) tune the
library kernel's schedule fields instead of defines.

:class:`PoolDriftMonitor` is the reference's ``WorkerMeasurementDriftMonitor``
(src/kernel_mcts/orchestration.py:160-173) on a pool: ``remeasure``
re-evaluates a program on the pool it was given (typically a one-GPU pool on a
spare device, so drift probes never queue behind search evaluations).
"""

from __future__ import annotations

import itertools
import json
import re
from dataclasses import dataclass
from random import Random
from typing import Any, Mapping, Protocol, Sequence

from .backend import SCHEDULE_BACKEND, schedule_from_source
from .domain import EvaluationResult, InvalidReason, KernelProgram, ProposalStatus, WorkloadContract
from .serialization import serialize_evaluation

_ANNOTATION = re.compile(
    r"^\s*//\s*KERNEL_MCTS_TUNE\s+([A-Z][A-Z0-9_]*)\s*=\s*([0-9]+(?:\s*,\s*[0-9]+)+)\s*$", re.MULTILINE)

#: Schedule fields a schedule program is tuned over, with their choices (the
#: library's compiled pair and 1-CTA variants; illegal combinations come back
#: as statically rejected trials, as in the sweep).
SCHEDULE_CHOICES: Mapping[str, tuple[int, ...]] = {
    "tile_n": (128, 256),
    "tile_k": (64, 128),
    "stages": (3, 4, 5, 6),
    "raster_group": (1, 2, 4, 8, 16),
}


class EventSink(Protocol):
    def emit(self, event_type: str, payload: Mapping[str, object]) -> None: ...


class NullEventSink:
    def emit(self, event_type: str, payload: Mapping[str, object]) -> None:
        return None


class BatchEvaluator(Protocol):
    def evaluate_many(self, programs: Sequence[KernelProgram], workload: WorkloadContract) -> list[EvaluationResult]: ...


@dataclass(frozen=True, slots=True)
class TuningParameter:
    name: str
    choices: tuple[int, ...]


@dataclass(frozen=True, slots=True)
class TuningConfig:
    budget: int
    method: str = "random"
    seed: int = 0

    def __post_init__(self) -> None:
        if self.budget < 1:
            raise ValueError("tuning budget must be positive")
        if self.method not in ("random", "grid"):
            raise ValueError("tuning method must be 'random' or 'grid'")


@dataclass(frozen=True, slots=True)
class TuningTrial:
    number: int
    parameters: Mapping[str, int]
    evaluation: EvaluationResult


@dataclass(frozen=True, slots=True)
class TuningResult:
    parameters: tuple[TuningParameter, ...]
    trials: tuple[TuningTrial, ...]
    best: EvaluationResult | None
    best_parameters: Mapping[str, int] | None
    baseline_reward: float | None = None
    skipped_reason: str | None = None

    @property
    def used(self) -> int:
        return len(self.trials)

    @property
    def improved(self) -> bool:
        return (self.best is not None and self.best.reward is not None and self.baseline_reward is not None
                and self.best.reward > self.baseline_reward)


def _define(name: str) -> re.Pattern[str]:
    return re.compile(rf"^(\s*#define\s+{re.escape(name)}\s+)([0-9]+)(\s*)$", re.MULTILINE)


def parse_tuning_parameters(program: KernelProgram) -> tuple[TuningParameter, ...]:
    """The tunable parameters of a program: annotated defines of a CUDA
    source, or the schedule fields of a schedule program."""
    if program.backend == SCHEDULE_BACKEND:
        schedule_from_source(program.source)  # validates the program
        return tuple(TuningParameter(name, choices) for name, choices in SCHEDULE_CHOICES.items())
    found: list[TuningParameter] = []
    for match in _ANNOTATION.finditer(program.source):
        name = match.group(1)
        if any(p.name == name for p in found):
            raise ValueError(f"duplicate tuning parameter {name}")
        choices = tuple(dict.fromkeys(int(v) for v in match.group(2).split(",")))
        if len(choices) < 2:
            raise ValueError(f"invalid choices for tuning parameter {name}")
        if not _define(name).search(program.source):
            raise ValueError(f"tuning parameter {name} has no integer #define")
        found.append(TuningParameter(name, choices))
    return tuple(found)


def current_configuration(program: KernelProgram, parameters: Sequence[TuningParameter]) -> dict[str, int]:
    if program.backend == SCHEDULE_BACKEND:
        from . import _native

        resolved = _native.make_config(**schedule_from_source(program.source)).as_dict()
        return {p.name: int(resolved[p.name]) for p in parameters}
    current = {}
    for p in parameters:
        match = _define(p.name).search(program.source)
        if match is None:
            raise ValueError(f"tuning parameter {p.name} has no integer #define")
        current[p.name] = int(match.group(2))
    return current


def render_configuration(program: KernelProgram, values: Mapping[str, int]) -> KernelProgram:
    """The program with each parameter set to ``values[name]``."""
    if program.backend == SCHEDULE_BACKEND:
        schedule = schedule_from_source(program.source)
        schedule.update({k: int(v) for k, v in values.items()})
        return KernelProgram(json.dumps(schedule, sort_keys=True), program.backend)
    source = program.source
    for name, value in values.items():
        source, count = _define(name).subn(rf"\g<1>{int(value)}\g<3>", source, count=1)
        if count != 1:
            raise ValueError(f"tuning parameter {name} has no unique integer #define")
    return KernelProgram(source, program.backend)


def configurations(parameters: Sequence[TuningParameter]) -> list[dict[str, int]]:
    names = [p.name for p in parameters]
    return [dict(zip(names, values)) for values in itertools.product(*(p.choices for p in parameters))]


class PoolAutotuner:
    """Tunes a program's parameters with every trial submitted to one
    ``evaluate_many`` call (one trial per pool worker at a time)."""

    def __init__(self, evaluator: BatchEvaluator, workload: WorkloadContract, config: TuningConfig,
                 events: EventSink | None = None) -> None:
        self._evaluator = evaluator
        self._workload = workload
        self._config = config
        self._events = events or NullEventSink()

    def plan(self, program: KernelProgram) -> tuple[tuple[TuningParameter, ...], list[dict[str, int]]]:
        """The parameters and the trial configurations, in trial order."""
        parameters = parse_tuning_parameters(program)
        if not parameters:
            return parameters, []
        current = current_configuration(program, parameters)
        trials = [c for c in configurations(parameters) if c != current]
        if self._config.method == "random":
            Random(self._config.seed).shuffle(trials)
        return parameters, trials[: self._config.budget]

    def run(self, baseline: EvaluationResult) -> TuningResult:
        if baseline.program is None:
            raise ValueError("autotuning requires a program")
        parameters, trials_plan = self.plan(baseline.program)
        if not parameters:
            reason = "final best kernel has no KERNEL_MCTS_TUNE annotations"
            self._events.emit("tuning_skipped", {"reason": reason})
            return TuningResult((), (), None, None, baseline.reward, reason)
        self._events.emit("tuning_started", {
            "budget": self._config.budget, "method": self._config.method, "seed": self._config.seed,
            "parameters": [{"name": p.name, "choices": list(p.choices)} for p in parameters],
            "configuration_count": len(trials_plan),
        })
        # Render everything first; statically unrenderable trials never reach a GPU.
        rendered: list[KernelProgram | EvaluationResult] = []
        for values in trials_plan:
            try:
                rendered.append(render_configuration(baseline.program, values))
            except ValueError as error:
                rendered.append(EvaluationResult(ProposalStatus.INVALID, invalid_reason=InvalidReason.OTHER,
                                                 metadata={"error_type": "static_tuning_rejection",
                                                           "message": str(error)}))
        programs = [r for r in rendered if isinstance(r, KernelProgram)]
        evaluated = iter(self._evaluator.evaluate_many(programs, self._workload) if programs else [])
        trials: list[TuningTrial] = []
        best: EvaluationResult | None = baseline
        best_values: Mapping[str, int] | None = None
        for number, (values, item) in enumerate(zip(trials_plan, rendered), 1):
            evaluation = next(evaluated) if isinstance(item, KernelProgram) else item
            trials.append(TuningTrial(number, values, evaluation))
            if (evaluation.status == ProposalStatus.VALID and evaluation.reward is not None
                    and (best.reward is None or evaluation.reward > best.reward)):
                best, best_values = evaluation, values
            self._events.emit("tuning_trial", {"trial": number, "b_tune": number, "parameters": dict(values),
                                               "evaluation": serialize_evaluation(evaluation)})
        self._events.emit("tuning_completed", {
            "b_tune": len(trials), "best_parameters": dict(best_values or {}),
            "baseline_reward": baseline.reward,
            "best_evaluation": serialize_evaluation(best) if best else None,
        })
        return TuningResult(parameters, tuple(trials), best, best_values, baseline.reward)


class PoolDriftMonitor:
    """``remeasure`` re-evaluates an evaluated program on its own pool."""

    def __init__(self, evaluator: Any) -> None:
        self._evaluator = evaluator
        self.calls = 0

    def remeasure(self, evaluation: EvaluationResult, workload: WorkloadContract) -> EvaluationResult:
        if evaluation.program is None:
            raise ValueError("drift remeasurement requires an evaluated program")
        self.calls += 1
        return self._evaluator.evaluate(evaluation.program, workload)


def drift(first: EvaluationResult, again: EvaluationResult) -> float | None:
    """Relative change of the median between two measurements of a program."""
    if first.benchmark is None or again.benchmark is None or first.benchmark.median_us <= 0:
        return None
    return again.benchmark.median_us / first.benchmark.median_us - 1.0


__all__ = [
    "NullEventSink",
    "PoolAutotuner",
    "PoolDriftMonitor",
    "SCHEDULE_CHOICES",
    "TuningConfig",
    "TuningParameter",
    "TuningResult",
    "TuningTrial",
    "configurations",
    "current_configuration",
    "drift",
    "parse_tuning_parameters",
    "render_configuration",
]
