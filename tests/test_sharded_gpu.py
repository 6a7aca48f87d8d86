"""The fused N-sharded GEMM + all-gather on 2 GPUs (skipped with fewer): every
rank's full C is bit-identical to the single-GPU kernel on the full problem,
for the fused kernel, the copy-engine all-gather and the NCCL baseline."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

PACKAGE_ROOT = Path(__file__).resolve().parent.parent / "gpu-kernel-mcts_b200"


@pytest.mark.parametrize("layout", ["row", "col"])
def test_fused_allgather_matches_single_gpu_bit_for_bit(cuda_device, layout):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={29700 + (0 if layout == 'row' else 1)}",
           "-m", "kernel_mcts_b200.sharded", "--M", "2048", "--N", "4096", "--K", "1024",
           "--b-layout", layout, "--steps", "3", "--warmup", "1", "--check"]
    out = subprocess.run(cmd, cwd=PACKAGE_ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    line = [l for l in out.stdout.splitlines() if l.startswith("{")][-1]
    result = json.loads(line)
    assert result["fused_bit_identical"] and result["nccl_bit_identical"], result
    assert result["copy_engines_bit_identical"], result
