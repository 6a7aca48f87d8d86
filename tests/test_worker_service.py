"""The worker service on CPU: the reference's worker protocol over the sm_100a
backend, and this package's pooled worker (per-GPU dispatch) with fake GPU
lanes, fake spawned pool workers and a real HTTP server on 127.0.0.1.
Nothing here touches a GPU."""

from __future__ import annotations

import json
import sys
import threading
import time

import pytest

from kernel_mcts_b200.domain import BenchmarkResult, EvaluationResult, KernelProgram, ProposalStatus
from kernel_mcts_b200.serialization import serialize_workload
from kernel_mcts_b200.worker_service import (
    EnvironmentManifest,
    GpuDispatcher,
    PooledWorkerApplication,
    WorkerBootstrap,
    build_application,
    gpu_pool,
    make_server,
)
from kernel_mcts_b200.workloads import gemm_workload
from reference_tree import REFERENCE_SRC

WORKLOAD = gemm_workload("worker_test", 256, 256, 256)
TOKEN = "secret-token"
AUTH = {"Authorization": f"Bearer {TOKEN}"}
MANIFEST = EnvironmentManifest(worker_id="w0", provider="local", gpu_model="NVIDIA B200", compute_capability="10.0",
                               captured_at="2026-01-01T00:00:00+00:00", gpu_count=2)


def request(evaluation_id: str, source: str = "candidate", profile_level: str = "tier0") -> bytes:
    return json.dumps({"evaluation_id": evaluation_id, "program": {"source": source, "backend": "cuda_cpp"},
                       "workload": serialize_workload(WORKLOAD), "profile_level": profile_level},
                      sort_keys=True).encode()


def valid(program: KernelProgram, lane: int) -> EvaluationResult:
    return EvaluationResult(status=ProposalStatus.VALID, program=program, reward=1.0, state_key=f"k-{program.source}",
                            benchmark=BenchmarkResult((1.0,), 1.0), metadata={"lane": lane})


class Lane:
    """One fake GPU: records what ran on it; optionally meets a barrier, so
    a test fails if two evaluations cannot be inside lanes at the same time."""

    def __init__(self, index: int, barrier: threading.Barrier | None = None, delay: float = 0.0) -> None:
        self.index, self.barrier, self.delay = index, barrier, delay
        self.evaluated: list[str] = []
        self.profiled: list[str] = []

    def evaluate(self, program, workload):
        self.evaluated.append(program.source)
        if "RAISE" in program.source:
            raise RuntimeError("lane failed")
        if self.barrier is not None:
            self.barrier.wait()
        time.sleep(self.delay)
        return valid(program, self.index)

    def lightweight_profile(self, evaluation, workload, metric_set):
        self.profiled.append(evaluation.program.source)
        return {"metric_set": metric_set, "lane": self.index}


def app_with(lanes) -> PooledWorkerApplication:
    return PooledWorkerApplication(auth_token=TOKEN, manifest=MANIFEST, dispatcher=GpuDispatcher(lanes),
                                   calibration={"backend": "cuda_sm100"})


def post(app, path, body):
    return app.handle("POST", path, AUTH, body)


def test_concurrent_requests_run_on_separate_gpus():
    barrier = threading.Barrier(2, timeout=10)  # both evaluations must be in flight at once
    lanes = [Lane(0, barrier), Lane(1, barrier)]
    app = app_with(lanes)
    out = {}
    threads = [threading.Thread(target=lambda i=i: out.__setitem__(i, post(app, "/evaluate", request(f"e{i}", f"c{i}"))))
               for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(20)
    assert [out[i].status for i in range(2)] == [200, 200]
    assert sorted(len(l.evaluated) for l in lanes) == [1, 1]
    assert {out[i].payload["metadata"]["lane"] for i in range(2)} == {0, 1}


def test_one_gpu_runs_one_evaluation_at_a_time():
    lane = Lane(0, delay=0.3)
    app = app_with([lane])
    start = time.monotonic()
    threads = [threading.Thread(target=post, args=(app, "/evaluate", request(f"e{i}", f"c{i}"))) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(20)
    assert time.monotonic() - start >= 0.6  # the second waited for the GPU
    assert sorted(lane.evaluated) == ["c0", "c1"]


def test_idempotency_conflict_and_concurrent_duplicates():
    lane = Lane(0, delay=0.3)
    app = app_with([lane])
    body = request("same", "cand")
    results = []
    threads = [threading.Thread(target=lambda: results.append(post(app, "/evaluate", body))) for _ in range(3)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(20)
    assert [r.status for r in results] == [200, 200, 200]
    assert lane.evaluated == ["cand"]  # one evaluation for three requests
    assert post(app, "/evaluate", body).payload == results[0].payload
    assert post(app, "/evaluate", request("same", "other")).status == 409


def test_protocol_errors_match_the_reference():
    app = app_with([Lane(0)])
    assert app.handle("GET", "/health", {}).status == 401
    assert app.handle("GET", "/health", {"authorization": f"Bearer {TOKEN}"}).payload == {"status": "ready"}
    assert app.handle("GET", "/nowhere", AUTH).status == 404
    assert post(app, "/evaluate", b"x" * 2_000_001).status == 413
    assert post(app, "/evaluate", b"{not json").payload == {"error": "invalid_request"}
    assert post(app, "/evaluate", request("e", profile_level="full")).payload == {"error": "unsupported_profile_level"}
    assert app.handle("GET", "/calibration", AUTH).payload == {"backend": "cuda_sm100"}
    manifest = app.handle("GET", "/manifest", AUTH).payload
    assert manifest["manifest_id"] == MANIFEST.manifest_id and manifest["gpu_count"] == 2


def test_a_failed_evaluation_is_not_cached():
    lane = Lane(0)
    app = app_with([lane])
    assert post(app, "/evaluate", request("r", "RAISE")).status == 500
    assert post(app, "/evaluate", request("r", "RAISE")).status == 500
    assert lane.evaluated == ["RAISE", "RAISE"]  # retried, not served from the cache


def test_profile_runs_on_the_lane_that_evaluated_and_is_cached():
    lanes = [Lane(0), Lane(1)]
    app = app_with(lanes)
    first = post(app, "/evaluate", request("p", "cand")).payload["metadata"]["lane"]
    body = json.dumps({"evaluation_id": "p", "profile_level": "lightweight", "metric_set": "sm100_v1"}).encode()
    profile = post(app, "/profile", body)
    assert profile.status == 200 and profile.payload == {"metric_set": "sm100_v1", "lane": first}
    assert post(app, "/profile", body).payload == profile.payload
    assert lanes[first].profiled == ["cand"] and lanes[1 - first].profiled == []
    unknown = json.dumps({"evaluation_id": "zz", "profile_level": "lightweight"}).encode()
    assert post(app, "/profile", unknown).payload == {"error": "evaluation_not_found"}
    bad_set = json.dumps({"evaluation_id": "p", "profile_level": "lightweight", "metric_set": "nope"}).encode()
    assert post(app, "/profile", bad_set).payload == {"error": "unsupported_metric_set"}
    artifact = json.dumps({"evaluation_id": "p", "sha256": "0" * 64}).encode()
    assert post(app, "/compiler-artifact", artifact).payload == {"error": "artifact_not_found"}


def test_bootstrap_reports_starting_then_failed_or_delegates():
    boot = WorkerBootstrap(TOKEN)
    assert boot.handle("GET", "/health", AUTH).status == 503
    boot.initialize(lambda progress: (_ for _ in ()).throw(RuntimeError("no GPU")))
    assert boot.handle("GET", "/health", AUTH).payload == {"status": "failed", "stage": "starting",
                                                           "error_code": "RuntimeError"}
    ready = WorkerBootstrap(TOKEN)
    ready.initialize(lambda progress: app_with([Lane(0)]))
    assert ready.handle("GET", "/health", AUTH).payload == {"status": "ready"}


def test_gpu_pool_from_the_environment():
    assert gpu_pool({"KERNEL_MCTS_GPU_POOL": "0,2,5"}) == [0, 2, 5]
    assert gpu_pool({"KERNEL_MCTS_GPU_COUNT": "4"}) == [0, 1, 2, 3]
    assert gpu_pool({}) == [0]
    with pytest.raises(RuntimeError):
        gpu_pool({"KERNEL_MCTS_GPU_POOL": "1,1"})


def test_build_application_calibrates_then_builds_one_lane_per_gpu(tmp_path):
    from test_backend import FakeRunner, make_backend

    runner = FakeRunner()
    backend = make_backend(tmp_path, runner)
    built = {}

    def backend_factory(environ, devices):
        from kernel_mcts_b200.workloads import root_program

        return "cuda_sm100", backend, root_program(), lambda root_us: ("spec", root_us)

    def lanes(devices, spec):
        built["devices"], built["spec"] = list(devices), spec
        return [Lane(d) for d in devices]

    def tools(command):
        if command[0] == "nvidia-smi":
            return "NVIDIA B200, GPU-1234, 10.0, 183359"
        return "Cuda compilation tools, release 12.9, V12.9.86" if command[0] == "nvcc" else "ncu 2025.2"

    stages = []
    env = {"KERNEL_MCTS_WORKER_TOKEN": TOKEN, "KERNEL_MCTS_WORKER_ID": "w1", "KERNEL_MCTS_GPU_POOL": "3,4"}
    app = build_application(env, stages.append, manifest_runner=tools, lane_factory=lanes,
                            backend_factory=backend_factory)
    assert stages == ["environment_manifest", "root_compile", "root_correctness", "root_benchmark",
                      "vendor_baselines", "gpu_lanes"]
    assert built["devices"] == [3, 4] and built["spec"] == ("spec", 11.0)  # the root's median reward denominator
    calibration = app.handle("GET", "/calibration", AUTH).payload
    assert calibration["backend"] == "cuda_sm100" and calibration["gpu_pool"] == [3, 4]
    assert calibration["benchmark"]["median_us"] == 11.0 and "cublas" in calibration["vendor_baselines"]
    manifest = app.handle("GET", "/manifest", AUTH).payload
    assert manifest["gpu_count"] == 2 and manifest["gpu_model"] == "NVIDIA B200"
    assert manifest["toolchain_versions"]["nvcc"] == "12.9"
    with pytest.raises(RuntimeError):
        build_application({"KERNEL_MCTS_WORKER_ID": "w1"}, manifest_runner=tools, lane_factory=lanes,
                          backend_factory=backend_factory)


def test_pool_lanes_evaluate_concurrently_in_spawned_workers(tmp_path):
    """Lanes backed by single-GPU EvaluationPools (spawned CPU workers pinned
    by CUDA_VISIBLE_DEVICES): two requests overlap, and a profile goes back
    to the worker process that evaluated the program."""
    from kernel_mcts_b200.pool import EvaluationPool, WorkerSpec

    spec = WorkerSpec("pool_fakes:make", {"marker_dir": str(tmp_path), "delay": 0.0})
    lanes = [EvaluationPool([d], spec) for d in (0, 1)]
    app = app_with(lanes)
    try:
        out = {}
        start = time.monotonic()
        threads = [threading.Thread(target=lambda i=i: out.__setitem__(
            i, post(app, "/evaluate", request(f"e{i}", f"sleep=1.0;c{i}")))) for i in range(2)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(60)
        elapsed = time.monotonic() - start
        assert [out[i].status for i in range(2)] == [200, 200]
        assert elapsed < 1.9, elapsed  # serialised they would take >= 2 s
        devices = {out[i].payload["metadata"]["visible_devices"] for i in range(2)}
        assert devices == {"0", "1"}
        body = json.dumps({"evaluation_id": "e0", "profile_level": "lightweight"}).encode()
        profile = post(app, "/profile", body).payload
        assert profile["visible_devices"] == out[0].payload["metadata"]["visible_devices"]
        assert profile["source"] == "sleep=1.0;c0"
    finally:
        app.dispatcher.close()


def test_http_server_with_the_reference_transport():
    """A real threading HTTP server on 127.0.0.1; the reference's own
    HTTPWorkerTransport (when its source tree is present) reads the manifest,
    evaluates and profiles over it."""
    lanes = [Lane(0), Lane(1)]
    server = make_server(app_with(lanes).handle, "127.0.0.1", 0)
    thread = threading.Thread(target=server.serve_forever, daemon=True)
    thread.start()
    address = f"http://127.0.0.1:{server.server_address[1]}"
    try:
        if not (REFERENCE_SRC / "kernel_mcts" / "worker_protocol.py").exists():
            import urllib.request

            req = urllib.request.Request(address + "/evaluate", data=request("h", "cand"), headers=AUTH, method="POST")
            with urllib.request.urlopen(req, timeout=30) as response:
                assert json.loads(response.read())["status"] == "VALID"
            return
        sys.path.insert(0, str(REFERENCE_SRC))
        try:
            from kernel_mcts.domain import KernelProgram as RefProgram
            from kernel_mcts.providers import WorkerEndpoint
            from kernel_mcts.serialization import deserialize_workload as ref_workload
            from kernel_mcts.worker_protocol import HTTPWorkerTransport
        except Exception as error:  # the reference needs packages this image may lack
            pytest.skip(f"reference transport not importable: {error}")
        finally:
            sys.path.remove(str(REFERENCE_SRC))
        transport = HTTPWorkerTransport(WorkerEndpoint(worker_id="w0", address=address, auth_token=TOKEN),
                                        timeout_seconds=30)
        manifest = transport.get_environment_manifest()
        assert manifest.gpu_count == 2 and manifest.manifest_id == MANIFEST.manifest_id
        result = transport.evaluate("h1", RefProgram("cand", "cuda_cpp"), ref_workload(serialize_workload(WORKLOAD)),
                                    "tier0")
        assert result.status.value == "VALID" and result.reward == 1.0
        profile = transport.profile("h1", "lightweight", "lightweight_v1")
        assert profile["metric_set"] == "lightweight_v1"
    finally:
        server.shutdown()
        server.server_close()


@pytest.mark.skipif(not (REFERENCE_SRC / "kernel_mcts" / "worker_protocol.py").exists(),
                    reason="reference tree not present")
def test_reference_worker_application_over_the_sm100_backend(tmp_path):
    """What a cuda_sm100 branch of the reference's _build_backend
    (src/kernel_mcts/worker_service.py:113-147) yields: the reference's own
    WorkerApplication and BackendKernelEvaluator over CudaSm100Backend (fake
    command runner), evaluating and profiling over its handler."""
    from test_backend import FakeRunner, ROOT_SOURCE, _wide_csv, make_backend
    from kernel_mcts_b200.profiling import LIGHTWEIGHT_V1_METRICS

    sys.path.insert(0, str(REFERENCE_SRC))
    try:
        from kernel_mcts.domain import BenchmarkResult as RefBenchmark
        from kernel_mcts.evaluation import BackendKernelEvaluator as RefEvaluator
        from kernel_mcts.evaluation import EvaluationContext as RefContext
        from kernel_mcts.providers import EnvironmentManifest as RefManifest
        from kernel_mcts.serialization import deserialize_evaluation as ref_deserialize
        from kernel_mcts.worker_protocol import WorkerApplication
    except Exception as error:
        pytest.skip(f"reference worker not importable: {error}")
    finally:
        sys.path.remove(str(REFERENCE_SRC))
    runner = FakeRunner()
    runner.ncu_stdout = _wide_csv(LIGHTWEIGHT_V1_METRICS)
    backend = make_backend(tmp_path, runner)
    manifest = RefManifest(worker_id="w0", provider="local", gpu_model="NVIDIA B200", compute_capability="10.0",
                           captured_at="2026-01-01T00:00:00+00:00")
    evaluator = RefEvaluator(backend=backend, root_benchmark=RefBenchmark((20.0,), 20.0),
                             context=RefContext("w0", manifest.manifest_id, {}, {"gpu_model": "B200"}))
    app = WorkerApplication(auth_token=TOKEN, manifest=manifest, evaluator=evaluator, profiler=evaluator)
    body = json.dumps({"evaluation_id": "r1", "program": {"source": ROOT_SOURCE, "backend": "cuda_cpp"},
                       "workload": serialize_workload(WORKLOAD), "profile_level": "tier0"}).encode()
    response = app.handle("POST", "/evaluate", AUTH, body)
    assert response.status == 200, response.payload
    result = ref_deserialize(response.payload)
    assert result.status.value == "VALID" and result.benchmark.median_us == 11.0
    assert result.reward == pytest.approx(__import__("math").log(20.0 / 11.0))
    profile = app.handle("POST", "/profile", AUTH,
                         json.dumps({"evaluation_id": "r1", "profile_level": "lightweight"}).encode())
    assert profile.status == 200 and profile.payload["metric_set"] == "lightweight_v1"


def test_in_process_schedule_profiles_through_the_harness(tmp_path):
    """A schedule evaluated in process (its artifact carries the resolved
    config, launch fields included) is profiled as the same schedule run by
    the harness under ncu."""
    from test_backend import FakeRunner, _wide_csv, make_backend

    from kernel_mcts_b200 import _native
    from kernel_mcts_b200.inprocess import HybridSm100Backend, ScheduleArtifact
    from kernel_mcts_b200.profiling import SM100_V1_METRICS

    class Query(FakeRunner):
        def __call__(self, command, *, timeout, env):
            if command[0].endswith("ncu") and "--query-metrics-mode" in command:
                return __import__("subprocess").CompletedProcess(command, 0, "\n".join(SM100_V1_METRICS), "")
            return super().__call__(command, timeout=timeout, env=env)

    runner = Query()
    runner.ncu_stdout = _wide_csv(SM100_V1_METRICS)
    hybrid = HybridSm100Backend(make_backend(tmp_path, runner), None)
    resolved = _native.make_config(tile_m=256, cluster_m=2, tile_n=256, tile_k=128, stages=3).as_dict()
    profile = hybrid.lightweight_profile(ScheduleArtifact("id", resolved), WORKLOAD, "sm100_v1")
    assert profile["metric_set"] == "sm100_v1"
    profiled = [c[0] for c in runner.calls if "--metrics" in c[0]]
    assert len(profiled) == 1 and "--tile-m=256" in profiled[0] and "--kernel=tcgen05" in profiled[0]
