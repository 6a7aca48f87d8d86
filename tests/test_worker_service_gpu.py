"""The worker service end to end on a B200: build_application calibrates the
root program and the vendor columns through the harness on GPU 0, then serves
the reference worker's HTTP protocol from a pool lane on that GPU; a schedule
and a candidate source evaluate over HTTP, a repeated request is served from
the idempotency cache, and /profile runs ncu with the sm100_v1 set."""

from __future__ import annotations

import json
import shutil
import subprocess
import threading
import urllib.error
import urllib.request

import pytest

from kernel_mcts_b200.backend import CudaSm100Backend, CudaSm100Config, schedule_program
from kernel_mcts_b200.serialization import serialize_workload
from kernel_mcts_b200.worker_service import build_application, make_server
from kernel_mcts_b200.workloads import BF16_GEMM_4096_B200

pytestmark = pytest.mark.gpu

TOKEN = "gpu-test-token"
LAUNCHER = r"""
#include <cuda_runtime.h>
#include "kmcts_gemm.h"
extern "C" int bf16_gemm_launch(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
    return kmcts_bf16_gemm_ex(A, B, C, M, N, K, KMCTS_B_COL, nullptr, s, nullptr);
}
"""


def _http(address, method, path, payload=None):
    body = json.dumps(payload, sort_keys=True).encode() if payload is not None else None
    request = urllib.request.Request(address + path, data=body, method=method,
                                     headers={"Authorization": f"Bearer {TOKEN}", "Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(request, timeout=600) as response:
            return response.status, json.loads(response.read())
    except urllib.error.HTTPError as error:
        return error.code, json.loads(error.read())


def _evaluate(address, evaluation_id, source, backend):
    return _http(address, "POST", "/evaluate", {
        "evaluation_id": evaluation_id, "program": {"source": source, "backend": backend},
        "workload": serialize_workload(BF16_GEMM_4096_B200), "profile_level": "tier0"})


def test_worker_service_serves_evaluations_on_a_b200(cuda_device, tmp_path):
    env = {"KERNEL_MCTS_WORKER_TOKEN": TOKEN, "KERNEL_MCTS_WORKER_ID": "b200-test", "KERNEL_MCTS_GPU_POOL": "0",
           "KERNEL_MCTS_ARTIFACT_ROOT": str(tmp_path)}
    app = build_application(env)
    server = make_server(app.handle, "127.0.0.1", 0)
    threading.Thread(target=server.serve_forever, daemon=True).start()
    address = f"http://127.0.0.1:{server.server_address[1]}"
    try:
        status, calibration = _http(address, "GET", "/calibration")
        assert status == 200 and calibration["backend"] == "cuda_sm100" and calibration["gpu_pool"] == [0]
        assert calibration["correctness"]["success"] and calibration["benchmark"]["median_us"] > 0
        assert "cublas" in calibration["vendor_baselines"]
        status, manifest = _http(address, "GET", "/manifest")
        assert status == 200 and "B200" in manifest["gpu_model"] and manifest["gpu_count"] == 1

        schedule = schedule_program(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3)
        status, first = _evaluate(address, "sched-1", schedule.source, schedule.backend)
        assert status == 200 and first["status"] == "VALID", first
        assert first["reward"] > 0  # faster than the CUDA-core root
        assert _evaluate(address, "sched-1", schedule.source, schedule.backend) == (200, first)
        status, candidate = _evaluate(address, "cand-1", LAUNCHER, "cuda_cpp")
        assert status == 200 and candidate["status"] == "VALID", candidate

        if shutil.which("ncu") is None:
            return
        # ncu runs the harness on this schedule for one launch; the same
        # command runs once without ncu first and must exit 0.
        probe = CudaSm100Backend(CudaSm100Config(artifact_root=tmp_path / "probe"))
        compiled = probe.compile(schedule, BF16_GEMM_4096_B200)
        target = probe.profile_target_command(compiled.artifact, BF16_GEMM_4096_B200)
        plain = subprocess.run(target, capture_output=True, text=True, timeout=300,
                               env=dict(probe.config.subprocess_environment))
        assert plain.returncode == 0, plain.stdout[-1000:] + plain.stderr[-1000:]
        status, profile = _http(address, "POST", "/profile",
                                {"evaluation_id": "sched-1", "profile_level": "lightweight", "metric_set": "sm100_v1"})
        assert status == 200 and profile["metric_set"] == "sm100_v1", profile
        assert profile["summary"]["tensor_pipe_active_pct_of_elapsed"] > 0
    finally:
        server.shutdown()
        server.server_close()
        app.dispatcher.close()
