"""Search configuration files (CPU): the B200 strategies and workload load with
this package's loader and, when the reference tree is present, with the
reference's own (src/kernel_mcts/config.py)."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

from kernel_mcts_b200.backend import CudaSm100Backend
from kernel_mcts_b200.config import B200_WORKLOAD, SM100_STRATEGIES, load_data, parse_workload, sm100_strategies
from kernel_mcts_b200.domain import KernelProgram
from kernel_mcts_b200.workloads import BF16_GEMM_4096_B200

from reference_tree import REFERENCE_SRC


def test_sm100_strategies_load_and_have_cuda_prompts():
    strategies = sm100_strategies()
    assert len(strategies) >= 6 and len({s.id for s in strategies}) == len(strategies)
    for s in strategies:
        assert s.prompt_for("cuda_cpp").strip()
    launcher = [s for s in strategies if "bf16_gemm_launch" in s.prompt_for("cuda_cpp")]
    assert launcher, "at least one strategy asks for the host-launcher ABI"
    assert "multicast" not in SM100_STRATEGIES.read_text()


def test_b200_workload_config_is_the_package_contract():
    workload = parse_workload(load_data(B200_WORKLOAD))
    assert workload.shapes == BF16_GEMM_4096_B200.shapes
    assert workload.metadata["entry_point"] == "bf16_gemm_root"
    CudaSm100Backend._validate_contract(KernelProgram("", "cuda_cpp"), workload)  # accepted as is


def test_reference_loader_reads_the_b200_configs():
    if not REFERENCE_SRC.exists():
        pytest.skip("reference source tree not present")
    sys.path.insert(0, str(REFERENCE_SRC))
    try:
        from kernel_mcts import config as ref_config
    except Exception as error:
        pytest.skip(f"reference config loader not importable: {error}")
    finally:
        sys.path.remove(str(REFERENCE_SRC))
    ref_strategies = ref_config.parse_strategies(ref_config.load_data(SM100_STRATEGIES))
    assert [s.id for s in ref_strategies] == [s.id for s in sm100_strategies()]
    ref_workload = ref_config.parse_workload(ref_config.load_data(B200_WORKLOAD))
    assert ref_workload.benchmark_id == "bf16_gemm_4096_b200"
