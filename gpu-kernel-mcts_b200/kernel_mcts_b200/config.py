"""Search configuration files in the reference's schema
(src/kernel_mcts/config.py:10-41): strategies and workloads as YAML or JSON.

``configs/strategies_sm100.yaml`` holds strategies for generated candidates on
B200, and ``configs/bf16_gemm_4096_b200.json`` the reference contract's
workload on B200; the reference's own loader reads both.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

from .domain import ShapeCase, Strategy, WorkloadContract

CONFIG_DIR = Path(__file__).resolve().parent / "configs"
SM100_STRATEGIES = CONFIG_DIR / "strategies_sm100.yaml"
B200_WORKLOAD = CONFIG_DIR / "bf16_gemm_4096_b200.json"


def load_data(path: str | Path) -> dict[str, Any]:
    text = Path(path).read_text()
    if Path(path).suffix == ".json":
        value = json.loads(text)
    else:
        import yaml

        value = yaml.safe_load(text)
    if not isinstance(value, dict):
        raise ValueError("configuration root must be a mapping")
    return value


def parse_strategies(data: dict[str, Any]) -> tuple[Strategy, ...]:
    return tuple(Strategy(item["id"], item["description"], dict(item["prompts"])) for item in data["strategies"])


def parse_workload(data: dict[str, Any]) -> WorkloadContract:
    item = data["workload"]
    return WorkloadContract(
        benchmark_id=item["benchmark_id"],
        operation=item["operation"],
        dtype=item["dtype"],
        shapes=tuple(ShapeCase(dict(s["dimensions"]), float(s["weight"])) for s in item["shapes"]),
        rtol=float(item["rtol"]),
        atol=float(item["atol"]),
        metadata=item.get("metadata", {}),
    )


def sm100_strategies() -> tuple[Strategy, ...]:
    return parse_strategies(load_data(SM100_STRATEGIES))
