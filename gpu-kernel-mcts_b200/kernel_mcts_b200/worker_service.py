"""The kernel_mcts worker service on B200: the reference worker's HTTP
protocol over this package's evaluator, with one evaluation per GPU at a time
instead of one evaluation per worker.

Reference behaviour kept (paths relative to the reference project):

* ``build_application`` (src/kernel_mcts/worker_service.py:28-110): token and
  worker id required; environment manifest; root program compiled, checked
  and benchmarked (its median is the reward denominator); vendor baselines;
  the calibration document served at ``/calibration``.
* ``build_backend`` is the ``_build_backend`` selection (:113-147) with a
  ``cuda_sm100`` branch: ``KERNEL_MCTS_BACKEND=cuda_sm100`` and
  ``KERNEL_MCTS_GPU_POOL=0,1,...`` (the GPUs this worker drives).  The root
  program is ``KERNEL_MCTS_ROOT_SOURCE`` (e.g. the reference's
  bf16_gemm_root.cu) or the library's CUDA-core kernel, which keeps the
  root's arithmetic.
* ``WorkerBootstrap`` (:150-194): ``/health`` answers 503 "starting" (or 500
  "failed") while the application is built.
* ``PooledWorkerApplication.handle`` keeps the routes, authentication,
  request-size limit, ``profile_level`` checks, idempotency cache (same
  ``evaluation_id`` and body: cached answer; different body: 409) and profile
  cache of ``WorkerApplication`` (src/kernel_mcts/worker_protocol.py:82-236),
  and its response payloads, so ``HTTPWorkerTransport`` and the CLIs above it
  run unchanged.

What changes:

* The reference holds one lock across each whole evaluation
  (worker_protocol.py:124-135), so a worker runs one evaluation at a time on
  device 0.  Here the lock guards only the caches; the evaluation runs on
  whichever GPU of the pool is idle (``GpuDispatcher``), so concurrent
  requests run on different GPUs.  A request whose ``evaluation_id`` is
  already being evaluated waits for that evaluation instead of starting a
  second one.
* Requests are served by a threading HTTP server (one thread per request).
* ``/compiler-artifact`` serves compiler-written PTX in the reference; this
  backend keeps none (reading the PTX of its own builds is not done here), so
  it answers 404 ``artifact_not_found`` for every request.
"""

from __future__ import annotations

import hashlib
import hmac
import json
import os
import queue
import re
import shutil
import subprocess
import threading
from dataclasses import dataclass, field
from datetime import datetime, timezone
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from typing import Any, Callable, Mapping, Sequence

from .domain import EvaluationResult, KernelProgram, ProposalStatus, WorkloadContract
from .evaluation import EvaluationInfrastructureError
from .profiling import PROFILE_METRIC_SET_IDS
from .serialization import deserialize_workload, json_value, serialize_benchmark, serialize_evaluation

BACKEND_NAME = "cuda_sm100"


# ------------------------------------------------------------------ manifest


@dataclass(frozen=True)
class EnvironmentManifest:
    """The worker's environment record, with the field names, identity
    payload and id hash of src/kernel_mcts/providers.py:28-93 and :540-542
    (controllers recompute the id from these fields)."""

    worker_id: str
    provider: str
    gpu_model: str
    compute_capability: str
    captured_at: str
    pod_id: str | None = None
    gpu_count: int = 1
    gpu_uuid: str | None = None
    sm_count: int | None = None
    total_memory_bytes: int | None = None
    form_factor: str | None = None
    mig_configuration: Mapping[str, object] = field(default_factory=dict)
    toolchain_versions: Mapping[str, str] = field(default_factory=dict)
    profiler_versions: Mapping[str, str] = field(default_factory=dict)
    library_versions: Mapping[str, str] = field(default_factory=dict)
    host_information: Mapping[str, object] = field(default_factory=dict)
    container_image: str | None = None
    container_digest: str | None = None
    container_runtime: str | None = None
    operating_state: Mapping[str, object] = field(default_factory=dict)
    project_git_commit: str | None = None
    dirty_tree: bool | None = None
    config_hashes: Mapping[str, str] = field(default_factory=dict)
    backend_implementation_hash: str | None = None

    _IDENTITY = ("worker_id", "provider", "pod_id", "gpu_model", "gpu_count", "gpu_uuid", "compute_capability",
                 "sm_count", "total_memory_bytes", "form_factor", "mig_configuration", "toolchain_versions",
                 "profiler_versions", "library_versions", "host_information", "container_image",
                 "container_digest", "container_runtime", "operating_state", "project_git_commit", "dirty_tree",
                 "config_hashes", "backend_implementation_hash")

    def __post_init__(self) -> None:
        if self.gpu_count < 1:
            raise ValueError("manifest gpu_count must be positive")

    def identity_payload(self) -> dict[str, object]:
        return {name: (dict(v) if isinstance(v := getattr(self, name), Mapping) else v) for name in self._IDENTITY}

    @property
    def manifest_id(self) -> str:
        encoded = json.dumps(self.identity_payload(), sort_keys=True, separators=(",", ":")).encode("utf-8")
        return hashlib.sha256(encoded).hexdigest()

    def as_dict(self) -> dict[str, object]:
        return {"manifest_id": self.manifest_id, "captured_at": self.captured_at, **self.identity_payload()}


ToolRunner = Callable[[Sequence[str]], str]


def _run_tool(command: Sequence[str]) -> str:
    resolved = shutil.which(command[0]) or command[0]
    result = subprocess.run([resolved, *command[1:]], capture_output=True, text=True, timeout=30, check=False,
                            env={"PATH": os.environ.get("PATH", os.defpath), "LANG": "C", "LC_ALL": "C"})
    if result.returncode != 0:
        raise RuntimeError(f"required worker tool {command[0]!r} failed")
    return " ".join(result.stdout.split())


def capture_environment_manifest(environ: Mapping[str, str], devices: Sequence[int],
                                 run: ToolRunner = _run_tool) -> EnvironmentManifest:
    """nvidia-smi, nvcc and ncu facts about the first GPU of the pool, as
    src/kernel_mcts/worker_service.py:202-262 gathers them; ``gpu_count`` is
    the pool's size."""
    worker_id = environ.get("KERNEL_MCTS_WORKER_ID") or environ.get("RUNPOD_POD_ID")
    if not worker_id:
        raise RuntimeError("KERNEL_MCTS_WORKER_ID is required")
    line = run(["nvidia-smi", "--query-gpu=name,uuid,compute_cap,memory.total", "--format=csv,noheader,nounits",
                f"--id={devices[0]}"])
    gpu_model, gpu_uuid, compute_capability, memory_mib = (item.strip() for item in line.split(",", 3))
    match = re.search(r"\brelease\s+([0-9]+(?:\.[0-9]+)+)", run(["nvcc", "--version"]), re.IGNORECASE)
    if match is None:
        raise RuntimeError("could not parse nvcc version")
    profilers = {}
    try:
        profilers["ncu"] = run(["ncu", "--version"])
    except (OSError, RuntimeError, subprocess.TimeoutExpired):
        pass
    return EnvironmentManifest(
        worker_id=worker_id, provider=environ.get("KERNEL_MCTS_PROVIDER", "local"), pod_id=worker_id,
        gpu_model=gpu_model, gpu_count=len(devices), gpu_uuid=gpu_uuid, compute_capability=compute_capability,
        total_memory_bytes=int(float(memory_mib) * 1024 * 1024),
        form_factor="SXM" if "b200" in gpu_model.casefold() else None,
        captured_at=datetime.now(timezone.utc).isoformat(),
        toolchain_versions={"nvcc": match.group(1), "cuda_toolkit": environ.get("CUDA_VERSION", "unknown")},
        profiler_versions=profilers,
        host_information={"gpu_pool": list(devices)},
        project_git_commit=environ.get("KERNEL_MCTS_GIT_COMMIT") or None,
    )


# ---------------------------------------------------------------- dispatch


class GpuDispatcher:
    """Hands each evaluation to an idle GPU lane.  A lane is one GPU's
    evaluator (for instance a single-device ``EvaluationPool``) with
    ``evaluate(program, workload)`` and ``lightweight_profile(evaluation,
    workload, metric_set)``; each lane runs one evaluation at a time, and
    callers on different threads run on different lanes at once."""

    def __init__(self, lanes: Sequence[Any]) -> None:
        if not lanes:
            raise ValueError("the dispatcher needs at least one GPU lane")
        self.lanes = list(lanes)
        self._idle: queue.Queue[int] = queue.Queue()
        for index in range(len(self.lanes)):
            self._idle.put(index)
        self._locks = [threading.Lock() for _ in self.lanes]

    def evaluate(self, program: KernelProgram, workload: WorkloadContract) -> tuple[EvaluationResult, int]:
        index = self._idle.get()
        try:
            with self._locks[index]:
                return self.lanes[index].evaluate(program, workload), index
        finally:
            self._idle.put(index)

    def lightweight_profile(self, lane: int, evaluation: EvaluationResult, workload: WorkloadContract,
                            metric_set: str) -> Mapping[str, object]:
        """Profiles on the lane that evaluated (it holds the compiled
        artifact); waits for that lane if it is busy."""
        with self._locks[lane]:
            return self.lanes[lane].lightweight_profile(evaluation, workload, metric_set)

    def close(self) -> None:
        for lane in self.lanes:
            close = getattr(lane, "close", None)
            if callable(close):
                close()


# ------------------------------------------------------------- application


@dataclass(frozen=True)
class WorkerResponse:
    status: int
    payload: Mapping[str, object]


class _Pending:
    """An evaluation in flight: later requests for its id wait on it."""

    def __init__(self, request_hash: str) -> None:
        self.request_hash = request_hash
        self.done = threading.Event()
        self.response: WorkerResponse | None = None


class PooledWorkerApplication:
    """Authenticated, idempotent worker protocol whose evaluations run
    concurrently, one per GPU (see the module docstring)."""

    def __init__(self, *, auth_token: str, manifest: EnvironmentManifest, dispatcher: GpuDispatcher,
                 calibration: Mapping[str, object] | None = None, max_request_bytes: int = 2_000_000) -> None:
        if not auth_token:
            raise ValueError("worker authentication token is required")
        self._auth_token = auth_token
        self._manifest = manifest
        self._dispatcher = dispatcher
        self._calibration = dict(calibration or {})
        self._max_request_bytes = max_request_bytes
        self._lock = threading.Lock()
        self._evaluations: dict[str, _Pending] = {}
        self._results: dict[str, tuple[EvaluationResult, WorkloadContract, int]] = {}
        self._profiles: dict[tuple[str, str, str], dict[str, object]] = {}

    @property
    def dispatcher(self) -> GpuDispatcher:
        return self._dispatcher

    def handle(self, method: str, path: str, headers: Mapping[str, str], body: bytes = b"") -> WorkerResponse:
        if not self._authorized(headers):
            return WorkerResponse(401, {"error": "unauthorized"})
        if method == "GET" and path == "/health":
            return WorkerResponse(200, {"status": "ready"})
        if method == "GET" and path == "/manifest":
            return WorkerResponse(200, json_value(self._manifest.as_dict()))
        if method == "GET" and path == "/calibration":
            return WorkerResponse(200, self._calibration)
        if method == "POST" and path == "/profile":
            return self._handle_profile(body)
        if method == "POST" and path == "/compiler-artifact":
            return self._handle_compiler_artifact(body)
        if method != "POST" or path != "/evaluate":
            return WorkerResponse(404, {"error": "not_found"})
        if len(body) > self._max_request_bytes:
            return WorkerResponse(413, {"error": "request_too_large"})
        try:
            payload = json.loads(body)
            evaluation_id = payload["evaluation_id"]
            program_value = payload["program"]
            if not isinstance(evaluation_id, str) or not evaluation_id or not isinstance(program_value, Mapping):
                raise ValueError
            program = KernelProgram(str(program_value["source"]), str(program_value["backend"]))
            workload = deserialize_workload(payload["workload"])
            if payload.get("profile_level") != "tier0":
                return WorkerResponse(400, {"error": "unsupported_profile_level"})
        except (KeyError, TypeError, ValueError, json.JSONDecodeError):
            return WorkerResponse(400, {"error": "invalid_request"})

        request_hash = hashlib.sha256(body).hexdigest()
        with self._lock:
            pending = self._evaluations.get(evaluation_id)
            owner = pending is None
            if owner:
                pending = _Pending(request_hash)
                self._evaluations[evaluation_id] = pending
        if pending.request_hash != request_hash:
            return WorkerResponse(409, {"error": "evaluation_id_conflict"})
        if not owner:
            pending.done.wait()
            return pending.response
        try:
            result, lane = self._dispatcher.evaluate(program, workload)
            response = WorkerResponse(200, serialize_evaluation(result))
            with self._lock:
                self._results[evaluation_id] = (result, workload, lane)
        except Exception:
            # The evaluation itself failed (not the candidate): forget the id
            # so a retry with it runs again, as an infrastructure retry would.
            with self._lock:
                self._evaluations.pop(evaluation_id, None)
            response = WorkerResponse(500, {"error": "evaluation_failed"})
        pending.response = response
        pending.done.set()
        return response

    def _handle_compiler_artifact(self, body: bytes) -> WorkerResponse:
        if len(body) > self._max_request_bytes:
            return WorkerResponse(413, {"error": "request_too_large"})
        try:
            payload = json.loads(body)
            if not isinstance(payload["evaluation_id"], str) or not isinstance(payload["sha256"], str):
                raise ValueError
        except (KeyError, TypeError, ValueError, json.JSONDecodeError):
            return WorkerResponse(400, {"error": "invalid_request"})
        with self._lock:
            known = self._results.get(payload["evaluation_id"])
        if known is None or known[0].status != ProposalStatus.VALID:
            return WorkerResponse(404, {"error": "evaluation_not_found"})
        return WorkerResponse(404, {"error": "artifact_not_found"})

    def _handle_profile(self, body: bytes) -> WorkerResponse:
        if len(body) > self._max_request_bytes:
            return WorkerResponse(413, {"error": "request_too_large"})
        try:
            payload = json.loads(body)
            evaluation_id = payload["evaluation_id"]
            profile_level = payload["profile_level"]
            metric_set = payload.get("metric_set", "lightweight_v1")
            if not isinstance(evaluation_id, str) or not evaluation_id:
                raise ValueError
            if profile_level != "lightweight":
                return WorkerResponse(400, {"error": "unsupported_profile_level"})
            if not isinstance(metric_set, str) or not metric_set:
                raise ValueError
            if metric_set not in PROFILE_METRIC_SET_IDS:
                return WorkerResponse(400, {"error": "unsupported_metric_set"})
        except (KeyError, TypeError, ValueError, json.JSONDecodeError):
            return WorkerResponse(400, {"error": "invalid_request"})
        key = (evaluation_id, profile_level, metric_set)
        with self._lock:
            cached = self._profiles.get(key)
            known = self._results.get(evaluation_id)
        if cached is not None:
            return WorkerResponse(200, cached)
        if known is None:
            return WorkerResponse(404, {"error": "evaluation_not_found"})
        evaluation, workload, lane = known
        try:
            profile = dict(self._dispatcher.lightweight_profile(lane, evaluation, workload, metric_set))
        except Exception as error:
            failure: dict[str, object] = {"error": "profiling_failed", "error_type": type(error).__name__}
            if isinstance(error, EvaluationInfrastructureError):
                failure["diagnostic"] = str(error)[:2_000]
            return WorkerResponse(500, failure)
        if profile.get("metric_set") != metric_set:
            return WorkerResponse(500, {"error": "profiling_failed", "error_type": "ProfileMetricSetMismatch"})
        with self._lock:
            self._profiles[key] = profile
        return WorkerResponse(200, profile)

    def _authorized(self, headers: Mapping[str, str]) -> bool:
        authorization = next((v for k, v in headers.items() if k.casefold() == "authorization"), "")
        return hmac.compare_digest(authorization, f"Bearer {self._auth_token}")


class WorkerBootstrap:
    """Answers /health while the application is being built
    (src/kernel_mcts/worker_service.py:150-194)."""

    def __init__(self, auth_token: str) -> None:
        self._auth_token = auth_token
        self._lock = threading.Lock()
        self._stage = "starting"
        self._application: PooledWorkerApplication | None = None
        self._failure_code: str | None = None

    def initialize(self, factory: Callable[[Callable[[str], None]], PooledWorkerApplication]) -> None:
        try:
            application = factory(self.set_stage)
        except Exception as error:
            with self._lock:
                self._failure_code = type(error).__name__
            return
        with self._lock:
            self._application = application
            self._stage = "ready"

    def set_stage(self, stage: str) -> None:
        with self._lock:
            self._stage = stage

    def handle(self, method: str, path: str, headers: Mapping[str, str], body: bytes = b"") -> WorkerResponse:
        authorization = next((v for k, v in headers.items() if k.casefold() == "authorization"), "")
        if not hmac.compare_digest(authorization, f"Bearer {self._auth_token}"):
            return WorkerResponse(401, {"error": "unauthorized"})
        with self._lock:
            application, stage, failure = self._application, self._stage, self._failure_code
        if application is not None:
            return application.handle(method, path, headers, body)
        if method == "GET" and path == "/health":
            if failure is not None:
                return WorkerResponse(500, {"status": "failed", "stage": stage, "error_code": failure})
            return WorkerResponse(503, {"status": "starting", "stage": stage})
        return WorkerResponse(503, {"error": "worker_starting", "stage": stage})


# ------------------------------------------------------------ construction


def gpu_pool(environ: Mapping[str, str]) -> list[int]:
    """``KERNEL_MCTS_GPU_POOL`` ("0,1,2"), else the first
    ``KERNEL_MCTS_GPU_COUNT`` devices, else device 0."""
    pool = environ.get("KERNEL_MCTS_GPU_POOL", "").strip()
    if pool:
        devices = [int(item) for item in pool.split(",") if item.strip()]
    else:
        devices = list(range(int(environ.get("KERNEL_MCTS_GPU_COUNT", "1"))))
    if not devices or len(set(devices)) != len(devices) or min(devices) < 0:
        raise RuntimeError(f"invalid GPU pool {pool!r}")
    return devices


def build_backend(environ: Mapping[str, str], devices: Sequence[int]):
    """The ``cuda_sm100`` branch of the reference's backend selection
    (worker_service.py:113-147): the subprocess backend that compiles and
    runs the root and vendor programs on the pool's first GPU, the root
    program, and the worker spec each GPU lane builds its evaluator from."""
    from .backend import CudaSm100Backend, CudaSm100Config
    from .pool import WorkerSpec
    from .workloads import root_program

    name = environ.get("KERNEL_MCTS_BACKEND", BACKEND_NAME)
    if name != BACKEND_NAME:
        raise RuntimeError(f"unsupported worker backend {name!r} (this worker builds {BACKEND_NAME!r})")
    artifact_root = Path(environ.get("KERNEL_MCTS_ARTIFACT_ROOT", "/tmp/kernel-mcts-artifacts"))
    env = {key: value for key, value in os.environ.items() if key in ("PATH", "LANG", "LC_ALL", "LD_LIBRARY_PATH",
                                                                        "HOME")}
    env["CUDA_VISIBLE_DEVICES"] = str(devices[0])
    calibration_backend = CudaSm100Backend(CudaSm100Config(artifact_root=artifact_root / "calibration",
                                                           device_index=devices[0], subprocess_environment=env))

    def lane_spec(root_us: float) -> WorkerSpec:
        return WorkerSpec("kernel_mcts_b200.pool:sm100_evaluator",
                          {"artifact_root": str(artifact_root), "root_us": root_us,
                           "worker_id": environ.get("KERNEL_MCTS_WORKER_ID")})

    return name, calibration_backend, root_program(environ.get("KERNEL_MCTS_ROOT_SOURCE")), lane_spec


def _default_lanes(devices: Sequence[int], spec) -> list[Any]:
    from .pool import EvaluationPool

    return [EvaluationPool([device], spec) for device in devices]


def build_application(environ: Mapping[str, str] | None = None, progress: Callable[[str], None] | None = None, *,
                      manifest_runner: ToolRunner = _run_tool,
                      lane_factory: Callable[[Sequence[int], Any], list[Any]] = _default_lanes,
                      backend_factory=build_backend) -> PooledWorkerApplication:
    """src/kernel_mcts/worker_service.py:28-110 for B200: root calibration on
    the pool's first GPU, then one evaluator lane per GPU of the pool."""
    from .vendor_baselines import VendorBaselineSuite
    from .workloads import BF16_GEMM_4096_B200

    environ = os.environ if environ is None else environ
    token = environ.get("KERNEL_MCTS_WORKER_TOKEN")
    worker_id = environ.get("KERNEL_MCTS_WORKER_ID") or environ.get("RUNPOD_POD_ID")
    if not token or not worker_id:
        raise RuntimeError("worker token and worker ID are required")
    devices = gpu_pool(environ)

    def stage(name: str) -> None:
        if progress is not None:
            progress(name)

    stage("environment_manifest")
    manifest = capture_environment_manifest(environ, devices, manifest_runner)
    backend_name, backend, root, lane_spec = backend_factory(environ, devices)
    workload = BF16_GEMM_4096_B200
    stage("root_compile")
    compiled = backend.compile(root, workload)
    if not compiled.success or compiled.artifact is None:
        raise RuntimeError("fixed root kernel failed to compile on the worker")
    stage("root_correctness")
    correctness = backend.check_correctness(compiled.artifact, workload)
    if not correctness.success:
        raise RuntimeError("fixed root kernel failed correctness on the worker")
    stage("root_benchmark")
    root_benchmark = backend.benchmark(compiled.artifact, workload)
    stage("vendor_baselines")
    vendor = VendorBaselineSuite(backend).run(workload)
    stage("gpu_lanes")
    dispatcher = GpuDispatcher(lane_factory(devices, lane_spec(root_benchmark.median_us)))
    calibration = {
        "benchmark_id": workload.benchmark_id,
        "backend": backend_name,
        "gpu_pool": list(devices),
        "compile": {"success": compiled.success, "duration_seconds": compiled.duration_seconds,
                    "artifact_id": compiled.artifact.artifact_id},
        "correctness": {"success": correctness.success, "maximum_error": correctness.maximum_error,
                        "mean_error": correctness.mean_error, "failed_test_id": correctness.failed_test_id,
                        "reference_metadata": json_value(dict(correctness.reference_metadata))},
        "benchmark": serialize_benchmark(root_benchmark),
        "vendor_baselines": {
            name: ({"correctness": result["correctness"], "benchmark": serialize_benchmark(result["benchmark"])}
                   if "benchmark" in result else json_value(dict(result)))
            for name, result in vendor.items()
        },
    }
    return PooledWorkerApplication(auth_token=token, manifest=manifest, dispatcher=dispatcher,
                                   calibration=calibration)


# ------------------------------------------------------------------ server


def make_server(handler: Callable[..., WorkerResponse], host: str = "127.0.0.1", port: int = 8000
                ) -> ThreadingHTTPServer:
    """A threading HTTP server for ``handler`` (one thread per request; the
    reference's handler class, worker_service.py:271-293, on a threading
    server so that requests for different GPUs overlap)."""

    class Handler(BaseHTTPRequestHandler):
        def do_GET(self):
            self._dispatch()

        def do_POST(self):
            self._dispatch()

        def _dispatch(self):
            length = int(self.headers.get("Content-Length", "0"))
            body = self.rfile.read(length) if length else b""
            response = handler(self.command, self.path, self.headers, body)
            encoded = json.dumps(response.payload, separators=(",", ":")).encode()
            self.send_response(response.status)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(encoded)))
            self.end_headers()
            self.wfile.write(encoded)

        def log_message(self, format, *args):
            return

    server = ThreadingHTTPServer((host, port), Handler)
    server.daemon_threads = True
    return server


def main() -> None:
    port = int(os.environ.get("KERNEL_MCTS_WORKER_PORT", "8000"))
    token = os.environ.get("KERNEL_MCTS_WORKER_TOKEN")
    if not token:
        raise RuntimeError("worker token is required")
    bootstrap = WorkerBootstrap(token)
    threading.Thread(target=bootstrap.initialize, args=(lambda progress: build_application(progress=progress),),
                     daemon=True).start()
    make_server(bootstrap.handle, os.environ.get("KERNEL_MCTS_WORKER_HOST", "0.0.0.0"), port).serve_forever()


if __name__ == "__main__":
    main()
