"""Nsight Compute metric sets and CSV parsing for the lightweight profile.

``lightweight_v1`` keeps the reference's metric names and summary aliases
(src/kernel_mcts/profiling.py:8-37) because profile payloads are part of the
worker's wire format.  ``sm100_v1`` adds the B200 evidence this path is judged
on: tensor-pipe utilisation against elapsed cycles, SM activity (wave
quantisation), DRAM and L2->SM bytes (re-reads), and the kernel's duration.
Every metric in it was read back from ncu on a B200 with driver 580.
"""

from __future__ import annotations

import csv
import math
from dataclasses import dataclass
from typing import Mapping, Sequence

LIGHTWEIGHT_V1_METRICS = (
    "launch__registers_per_thread",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "l1tex__throughput.avg.pct_of_peak_sustained_active",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
    "smsp__inst_executed.sum",
)

LIGHTWEIGHT_V1_ALIASES = {
    "launch__registers_per_thread": "registers_per_thread",
    "sm__warps_active.avg.pct_of_peak_sustained_active": "achieved_occupancy_pct",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed": "sm_throughput_pct",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": "dram_throughput_pct",
    "lts__throughput.avg.pct_of_peak_sustained_elapsed": "l2_throughput_pct",
    "l1tex__throughput.avg.pct_of_peak_sustained_active": "l1tex_throughput_pct",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": "tensor_pipe_utilization_pct",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio": "long_scoreboard_warps_per_issue",
    "smsp__inst_executed.sum": "instructions_executed",
}

SM100_V1_METRICS = (
    "gpu__time_duration.sum",
    "launch__registers_per_thread",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__cycles_active.avg",
    "sm__cycles_elapsed.avg",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "lts__t_sector_hit_rate.pct",
    "l1tex__m_xbar2l1tex_read_bytes.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
)

SM100_V1_ALIASES = {
    "gpu__time_duration.sum": "duration",
    "launch__registers_per_thread": "registers_per_thread",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed": "tensor_pipe_active_pct_of_elapsed",
    "sm__cycles_active.avg": "sm_cycles_active",
    "sm__cycles_elapsed.avg": "sm_cycles_elapsed",
    "dram__bytes_read.sum": "dram_bytes_read",
    "dram__bytes_write.sum": "dram_bytes_written",
    "lts__t_sector_hit_rate.pct": "l2_sector_hit_rate_pct",
    "l1tex__m_xbar2l1tex_read_bytes.sum": "l2_to_sm_bytes",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": "dram_throughput_pct",
}

# Kernel-name patterns (ncu --kernel-name regex:...) per artifact ABI.
_KERNEL_PATTERNS = {
    "root": "bf16_gemm_root",
    "library": "gemm_bf16_tcgen05|gemm_bf16_simt",
    "schedule": "gemm_bf16_tcgen05",
    "vendor:cublas": "nvjet|gemm|sm100",
    "vendor:cutlass_sm80": "cutlass|Kernel",
}


@dataclass(frozen=True, slots=True)
class ProfileMetricSet:
    id: str
    schema_version: int
    architecture: str
    metrics: tuple[str, ...]
    aliases: Mapping[str, str]

    def kernel_regex(self, abi: str) -> str:
        return _KERNEL_PATTERNS.get(abi, ".*")


_METRIC_SETS = {
    ("lightweight_v1", "*"): ProfileMetricSet("lightweight_v1", 1, "*", LIGHTWEIGHT_V1_METRICS, LIGHTWEIGHT_V1_ALIASES),
    ("sm100_v1", "sm_100a"): ProfileMetricSet("sm100_v1", 1, "sm_100a", SM100_V1_METRICS, SM100_V1_ALIASES),
}

PROFILE_METRIC_SET_IDS = ("lightweight_v1", "sm100_v1")

# Launch attributes that ncu collects but does not list among queryable
# metrics (the reference exempts the same one, src/kernel_mcts/profiling.py:22-24).
NCU_QUERY_VALIDATION_EXEMPT_METRICS = frozenset({"launch__registers_per_thread"})


def metrics_missing_from_query(definition: "ProfileMetricSet", query_output: str) -> list[str]:
    """Metrics of ``definition`` that ``ncu --query-metrics-mode all`` output
    does not list (the check of src/kernel_mcts/cuda_backend.py:413-461:
    every token containing "__" is an available metric name)."""
    available = {token.strip(" ,:\"'") for token in query_output.split() if "__" in token}
    return [m for m in definition.metrics if m not in available and m not in NCU_QUERY_VALIDATION_EXEMPT_METRICS]


def resolve_metric_set(metric_set_id: str, architecture: str) -> ProfileMetricSet:
    definition = _METRIC_SETS.get((metric_set_id, architecture)) or _METRIC_SETS.get((metric_set_id, "*"))
    if definition is None:
        raise ValueError(f"profile metric set {metric_set_id!r} is unavailable for {architecture!r}")
    return definition


class ProfileParseError(ValueError):
    """ncu's CSV did not carry the requested metrics."""


def _number(text: str) -> float:
    value = float(text.replace(",", ""))
    if not math.isfinite(value):
        raise ProfileParseError("Nsight Compute returned a non-finite metric")
    return value


def parse_ncu_csv(text: str, required: Sequence[str]) -> dict[str, dict[str, object]]:
    """Parses ncu ``--csv --page raw`` output in either layout: one metric per
    row ("Metric Name"/"Metric Unit"/"Metric Value") or one metric per column
    (header row, unit row, value rows).  Takes the first launch."""
    rows = list(csv.reader(text.splitlines()))
    long_header = next((i for i, r in enumerate(rows)
                        if "Metric Name" in r and "Metric Unit" in r and "Metric Value" in r), None)
    metrics: dict[str, dict[str, object]] = {}
    if long_header is not None:
        header = rows[long_header]
        name_i, unit_i, value_i = (header.index(k) for k in ("Metric Name", "Metric Unit", "Metric Value"))
        for row in rows[long_header + 1:]:
            if len(row) <= max(name_i, unit_i, value_i) or row[name_i] not in required or row[name_i] in metrics:
                continue
            try:
                metrics[row[name_i]] = {"value": _number(row[value_i]), "unit": row[unit_i]}
            except ValueError as error:
                raise ProfileParseError("Nsight Compute returned a non-numeric metric") from error
    else:
        wide_header = next((i for i, r in enumerate(rows) if all(m in r for m in required)), None)
        if wide_header is None or wide_header + 2 >= len(rows):
            raise ProfileParseError("Nsight Compute returned malformed CSV")
        header, units = rows[wide_header], rows[wide_header + 1]
        columns = {m: header.index(m) for m in required}
        for row in rows[wide_header + 2:]:
            if len(row) <= max(columns.values()):
                continue
            try:
                metrics = {m: {"value": _number(row[c]), "unit": units[c] if c < len(units) else ""}
                           for m, c in columns.items()}
            except ValueError:
                continue
            break
    missing = [m for m in required if m not in metrics]
    if missing:
        raise ProfileParseError(f"Nsight Compute did not return {missing[:4]}")
    return {m: metrics[m] for m in required}
