"""Parallel candidate evaluation: one worker process per GPU.

The reference serialises every evaluation behind one lock on device 0
(src/kernel_mcts/worker_protocol.py:124-135; cuda_backend.py:264 ``--id=0``).
Candidate and schedule evaluations are independent units, so here each GPU
gets its own worker process (spawned, ``CUDA_VISIBLE_DEVICES`` pinned before
anything touches CUDA) with its own backend and evaluator, and jobs are handed
to whichever worker is idle.  There is no collective: the path shards by
evaluation.

Failure handling (host side only; nothing here touches a GPU):
* a worker that dies or stops answering has its in-flight job re-queued on
  another worker and is restarted;
* a job whose attempts all end in dead workers comes back as an
  INFRASTRUCTURE_FAILURE result, as an infrastructure retry in the reference
  would report it (src/kernel_mcts/orchestration.py:256-272).

A ``HostCompilePool`` builds candidate sources with nvcc on host cores ahead
of the GPU workers: ``evaluate_many(..., compile_ahead=pool)`` submits every
candidate's build at once and hands a candidate to a GPU only when its build
is done, so the GPU evaluates candidate i while nvcc builds i+1, i+2, ...;
the workers find the builds in the shared candidate cache.

``evaluate_many`` keeps the KernelEvaluator call shape
(src/kernel_mcts/interfaces.py:8-9) for a batch; ``evaluate`` is the single
call, so MCTS runs unchanged on top.  ``lightweight_profile`` keeps the
NodeProfiler call shape: the worker that evaluated a program profiles it,
from the compiled artifact it still holds.
"""

from __future__ import annotations

import importlib
import multiprocessing as mp
import os
import queue
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping, Sequence

from .domain import EvaluationResult, KernelProgram, ProposalStatus, WorkloadContract
from .serialization import deserialize_evaluation, deserialize_workload, serialize_evaluation, serialize_workload


@dataclass(frozen=True)
class WorkerSpec:
    """How a worker builds its evaluator: ``factory`` is "module:function",
    called as ``function(device_index, **options)`` inside the worker and
    returning an object with ``evaluate(program, workload)``."""

    factory: str
    options: Mapping[str, Any] = field(default_factory=dict)


def _resolve(factory: str) -> Callable[..., Any]:
    module, _, name = factory.partition(":")
    return getattr(importlib.import_module(module), name)


def _worker_main(slot: int, device: str, spec: WorkerSpec, jobs: "mp.Queue", results: "mp.Queue") -> None:
    # Pin the GPU before any CUDA context can exist in this process.
    os.environ["CUDA_VISIBLE_DEVICES"] = device
    try:
        evaluator = _resolve(spec.factory)(int(device) if device.isdigit() else 0, **dict(spec.options))
    except Exception:  # the worker could not start: report and exit
        results.put(("startup_error", slot, None, traceback.format_exc()))
        return
    results.put(("ready", slot, None, None))
    # This worker's latest result per (program source, workload id): a later
    # profile request for that evaluation needs its compiled artifact.
    evaluated: dict[tuple[str, str], EvaluationResult] = {}
    while True:
        item = jobs.get()
        if item is None:
            return
        if item[0] == "profile":
            _, job_id, program_value, workload_value, metric_set = item
            workload = deserialize_workload(workload_value)
            evaluation = evaluated.get((program_value["source"], workload.benchmark_id))
            try:
                if evaluation is None:
                    raise LookupError("this worker holds no evaluation of that program and workload")
                profile = dict(evaluator.lightweight_profile(evaluation, workload, metric_set))
                results.put(("profiled", slot, job_id, profile))
            except Exception as error:
                results.put(("profile_error", slot, job_id, (type(error).__name__, str(error)[-2000:])))
            continue
        if item[0] == "prepare":
            # Warm this worker for a workload (inputs, references) before timing starts.
            try:
                prepare = getattr(evaluator, "prepare", None)
                if callable(prepare):
                    prepare(deserialize_workload(item[1]))
                results.put(("prepared", slot, None, None))
            except Exception:
                results.put(("prepared", slot, None, traceback.format_exc()))
            continue
        job_id, program_value, workload_value = item
        program = KernelProgram(program_value["source"], program_value["backend"])
        workload = deserialize_workload(workload_value)
        try:
            evaluation = evaluator.evaluate(program, workload)
            evaluated[(program.source, workload.benchmark_id)] = evaluation
            results.put(("result", slot, job_id, serialize_evaluation(evaluation)))
        except Exception:
            results.put(("error", slot, job_id, traceback.format_exc()))


@dataclass
class _Worker:
    slot: int
    device: str
    process: Any
    jobs: Any
    job: int | None = None
    started_at: float = 0.0
    ready: bool = False


class EvaluationPool:
    """Fans evaluations out over GPUs, one worker process per device."""

    def __init__(
        self,
        devices: Sequence[int | str],
        spec: WorkerSpec,
        *,
        job_timeout_seconds: float = 1800.0,
        max_attempts: int = 2,
        startup_timeout_seconds: float = 600.0,
    ) -> None:
        if not devices:
            raise ValueError("the pool needs at least one device")
        self.devices = [str(d) for d in devices]
        self.spec = spec
        self.job_timeout = job_timeout_seconds
        self.max_attempts = max_attempts
        self.startup_timeout = startup_timeout_seconds
        self._ctx = mp.get_context("spawn")
        self._results = self._ctx.Queue()
        self._workers: list[_Worker] = []
        self._ran_on: dict[tuple[str, str], int] = {}  # (source, workload id) -> slot that evaluated it
        self._profile_jobs = 0
        self.restarts = 0
        for slot, device in enumerate(self.devices):
            self._workers.append(self._start(slot, device))
        self._await_ready()

    # ------------------------------------------------------------- lifecycle

    def _start(self, slot: int, device: str) -> _Worker:
        jobs = self._ctx.Queue()
        process = self._ctx.Process(target=_worker_main, args=(slot, device, self.spec, jobs, self._results),
                                    daemon=True, name=f"kmcts-eval-gpu{device}")
        process.start()
        return _Worker(slot, device, process, jobs)

    def _await_ready(self) -> None:
        deadline = time.monotonic() + self.startup_timeout
        while not all(w.ready for w in self._workers):
            try:
                kind, slot, _, payload = self._results.get(timeout=max(0.1, deadline - time.monotonic()))
            except queue.Empty as error:
                self.close()
                raise RuntimeError("evaluation workers did not start in time") from error
            if kind == "startup_error":
                self.close()
                raise RuntimeError(f"evaluation worker {slot} failed to start:\n{payload}")
            if kind == "ready":
                self._workers[slot].ready = True

    def close(self) -> None:
        for w in self._workers:
            if w.process.is_alive():
                try:
                    w.jobs.put(None)
                except (OSError, ValueError):
                    pass
        for w in self._workers:
            w.process.join(timeout=10)
            if w.process.is_alive():
                w.process.kill()
                w.process.join(timeout=5)

    def __enter__(self) -> "EvaluationPool":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    @property
    def size(self) -> int:
        return len(self._workers)

    def worker_pids(self) -> list[int]:
        return [w.process.pid for w in self._workers]

    # ------------------------------------------------------------ evaluation

    def prepare(self, workload: WorkloadContract, timeout_seconds: float = 600.0) -> None:
        """Has every worker build its per-workload state (device inputs, the
        reference output) now, so later evaluations measure only evaluation."""
        value = serialize_workload(workload)
        for w in self._workers:
            w.jobs.put(("prepare", value))
        waiting = {w.slot for w in self._workers}
        deadline = time.monotonic() + timeout_seconds
        while waiting:
            try:
                kind, slot, _, payload = self._results.get(timeout=max(0.1, deadline - time.monotonic()))
            except queue.Empty as error:
                raise RuntimeError("workers did not finish preparing in time") from error
            if kind == "prepared":
                if payload:
                    raise RuntimeError(f"worker {slot} failed to prepare:\n{payload}")
                waiting.discard(slot)
            elif kind == "ready":
                self._workers[slot].ready = True

    def evaluate(self, program: KernelProgram, workload: WorkloadContract) -> EvaluationResult:
        return self.evaluate_many([program], workload)[0]

    def evaluate_many(self, programs: Sequence[KernelProgram], workload: WorkloadContract, *,
                      compile_ahead: "HostCompilePool | None" = None) -> list[EvaluationResult]:
        workload_value = serialize_workload(workload)
        builds = ([compile_ahead.submit(p, workload) for p in programs] if compile_ahead is not None
                  else [None] * len(programs))
        pending = list(range(len(programs)))[::-1]  # pop() takes the lowest index first
        attempts = [0] * len(programs)
        out: list[EvaluationResult | None] = [None] * len(programs)
        done = 0

        def next_job() -> int | None:
            # The lowest pending job whose build (if any) has finished.
            for position in range(len(pending) - 1, -1, -1):
                build = builds[pending[position]]
                if build is None or build.done():
                    return pending.pop(position)
            return None

        while done < len(programs):
            for w in self._workers:
                if w.job is None and w.ready and pending:
                    job = next_job()
                    if job is None:
                        break
                    attempts[job] += 1
                    p = programs[job]
                    w.jobs.put((job, {"source": p.source, "backend": p.backend}, workload_value))
                    w.job, w.started_at = job, time.monotonic()
            try:
                # Short waits while builds are still running, so a finished
                # build reaches an idle GPU at once.
                waiting_builds = any(builds[j] is not None and not builds[j].done() for j in pending)
                kind, slot, job, payload = self._results.get(timeout=0.02 if waiting_builds else 0.5)
            except queue.Empty:
                kind = None
            if kind == "ready":
                self._workers[slot].ready = True
            elif kind in ("result", "error"):
                w = self._workers[slot]
                if w.job == job:
                    w.job = None
                if out[job] is None:
                    out[job] = (deserialize_evaluation(payload) if kind == "result"
                                else _infrastructure_failure(programs[job], f"worker raised:\n{payload}"))
                    if kind == "result":
                        self._ran_on[(programs[job].source, workload.benchmark_id)] = slot
                    done += 1
            elif kind == "startup_error":
                w = self._workers[slot]
                w.ready = False
            # Dead or stuck workers: re-queue their job and restart them.
            for w in self._workers:
                stuck = w.job is not None and time.monotonic() - w.started_at > self.job_timeout
                if w.process.is_alive() and not stuck:
                    continue
                if w.process.is_alive():
                    w.process.kill()
                w.process.join(timeout=5)
                job = w.job
                if job is not None and out[job] is None:
                    if attempts[job] < self.max_attempts:
                        pending.append(job)
                    else:
                        out[job] = _infrastructure_failure(
                            programs[job], f"worker on device {w.device} died {attempts[job]} time(s)")
                        done += 1
                self.restarts += 1
                self._ran_on = {key: s for key, s in self._ran_on.items() if s != w.slot}
                self._workers[w.slot] = self._start(w.slot, w.device)
        return [r for r in out if r is not None]


    def lightweight_profile(self, evaluation: EvaluationResult, workload: WorkloadContract,
                            metric_set: str = "lightweight_v1", timeout_seconds: float = 900.0) -> Mapping[str, Any]:
        """Profiles a valid evaluation this pool ran, on the worker that ran it
        (it holds the compiled artifact).  Raises EvaluationInfrastructureError
        when that worker has been restarted since, or profiling fails there."""
        from .evaluation import EvaluationInfrastructureError

        if evaluation.status != ProposalStatus.VALID or evaluation.program is None:
            raise ValueError("only valid evaluations can be profiled")
        slot = self._ran_on.get((evaluation.program.source, workload.benchmark_id))
        if slot is None:
            raise EvaluationInfrastructureError("no worker of this pool holds that evaluation")
        w = self._workers[slot]
        if not w.process.is_alive():
            raise EvaluationInfrastructureError("the worker that ran the evaluation has exited")
        self._profile_jobs += 1
        job = -self._profile_jobs  # negative ids never collide with evaluation jobs
        program = evaluation.program
        w.jobs.put(("profile", job, {"source": program.source, "backend": program.backend},
                    serialize_workload(workload), metric_set))
        deadline = time.monotonic() + timeout_seconds
        while True:
            try:
                kind, got_slot, got_job, payload = self._results.get(timeout=0.5)
            except queue.Empty:
                if not w.process.is_alive():
                    self._ran_on = {key: s for key, s in self._ran_on.items() if s != slot}
                    self.restarts += 1
                    self._workers[slot] = self._start(slot, w.device)
                    raise EvaluationInfrastructureError("the worker died while profiling") from None
                if time.monotonic() > deadline:
                    raise EvaluationInfrastructureError("profiling did not finish in time") from None
                continue
            if kind == "ready":
                self._workers[got_slot].ready = True
            elif got_slot == slot and got_job == job:
                if kind == "profiled":
                    return payload
                error_type, message = payload
                if error_type == "EvaluationInfrastructureError":
                    raise EvaluationInfrastructureError(message)
                # Any other failure in the worker is an infrastructure failure
                # to the caller; keep its type in the diagnostic.
                raise EvaluationInfrastructureError(f"{error_type}: {message}")


class HostCompilePool:
    """nvcc builds of candidate sources on host cores, into the candidate
    cache the GPU workers read (``CudaSm100Config.candidate_cache``).
    Schedule programs need no build and get no job."""

    def __init__(self, artifact_root: str | os.PathLike, *, jobs: int | None = None, runner: Any = None) -> None:
        from concurrent.futures import ThreadPoolExecutor
        from pathlib import Path

        from .backend import CudaSm100Backend, CudaSm100Config

        root = Path(artifact_root)
        self.backend = CudaSm100Backend(CudaSm100Config(artifact_root=root / "host-compile",
                                                        candidate_cache=candidate_cache(root)), runner=runner)
        self.jobs = jobs or max(1, (os.cpu_count() or 2) - 1)
        self._executor = ThreadPoolExecutor(max_workers=self.jobs, thread_name_prefix="kmcts-nvcc")

    def submit(self, program: KernelProgram, workload: WorkloadContract):
        from .backend import CANDIDATE_BACKEND

        if program.backend != CANDIDATE_BACKEND:
            return None
        return self._executor.submit(self.backend.compile, program, workload)

    def close(self) -> None:
        self._executor.shutdown(wait=True)

    def __enter__(self) -> "HostCompilePool":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def candidate_cache(artifact_root: str | os.PathLike):
    """The candidate build cache shared by a host compile pool and the GPU
    workers under one artifact root."""
    from pathlib import Path

    return Path(artifact_root) / "candidates"


def _infrastructure_failure(program: KernelProgram, reason: str) -> EvaluationResult:
    return EvaluationResult(status=ProposalStatus.INFRASTRUCTURE_FAILURE, program=program,
                            metadata={"error_type": "WorkerFailure", "reason": reason[-2000:]})


# --------------------------------------------------------------- factories


def sm100_evaluator(device_index: int, *, artifact_root: str, root_us: float, warmup_count: int = 10,
                    measurement_count: int = 30, flush_l2: bool = False, worker_id: str | None = None,
                    inprocess: bool = True):
    """The production worker: BackendKernelEvaluator on this worker's GPU over
    the hybrid backend (schedule programs in process, candidate sources
    through nvcc and the harness), rewarding against a root median of
    ``root_us``."""
    from pathlib import Path

    from .backend import CudaSm100Backend, CudaSm100Config
    from .domain import BenchmarkResult
    from .evaluation import BackendKernelEvaluator, EvaluationContext
    from .inprocess import HybridSm100Backend, InProcessSm100Backend

    subprocess_backend = CudaSm100Backend(CudaSm100Config(
        artifact_root=Path(artifact_root) / f"gpu{device_index}", warmup_count=warmup_count,
        measurement_count=measurement_count, device_index=device_index, flush_l2=flush_l2,
        candidate_cache=candidate_cache(artifact_root)))
    local = (InProcessSm100Backend(warmup_count=warmup_count, measurement_count=measurement_count,
                                   flush_l2=flush_l2, device_index=device_index) if inprocess else None)
    backend = HybridSm100Backend(subprocess_backend, local)
    context = EvaluationContext(worker_id or f"b200-gpu{device_index}", "kmcts-b200",
                                {"launcher": "kmcts_bf16_gemm_ex"}, {"gpu": "B200", "arch": "sm_100a"})
    return BackendKernelEvaluator(backend=backend, root_benchmark=BenchmarkResult((root_us,), root_us),
                                  context=context)


# ------------------------------------------------------------ measurement


def candidate_sources(count: int) -> list[KernelProgram]:
    """``count`` distinct host-launcher candidates (each runs the library's
    GEMM with its own raster group, so each is a separate build)."""
    template = (
        "#include <cuda_runtime.h>\n#include \"kmcts_gemm.h\"\n"
        "extern \"C\" int bf16_gemm_launch(const void* A, const void* B, void* C, int M, int N, int K,\n"
        "                                cudaStream_t s) {{\n"
        "    kmcts_gemm_config cfg;\n    kmcts_default_config(&cfg);\n    cfg.raster_group = {group};\n"
        "    return kmcts_bf16_gemm_ex(A, B, C, M, N, K, KMCTS_B_COL, &cfg, s, nullptr);\n}}\n")
    return [KernelProgram(template.format(group=1 + i), "cuda_cpp") for i in range(count)]


def _measure(argv: Sequence[str] | None = None) -> None:
    """Candidate-source evaluations per second through the pool, with and
    without the host compile pool ahead of it (fresh build caches each)."""
    import argparse
    import json
    import tempfile

    from .workloads import gemm_workload

    p = argparse.ArgumentParser(description=_measure.__doc__.split("\n")[0])
    p.add_argument("--devices", default="0")
    p.add_argument("--candidates", type=int, default=8)
    p.add_argument("--M", type=int, default=4096)
    p.add_argument("--N", type=int, default=4096)
    p.add_argument("--K", type=int, default=4096)
    p.add_argument("--jobs", type=int, default=None, help="host compile threads")
    args = p.parse_args(argv)
    devices = [d for d in args.devices.split(",") if d]
    workload = gemm_workload(f"bf16_gemm_{args.M}x{args.N}x{args.K}_b200", args.M, args.N, args.K)
    programs = candidate_sources(args.candidates)
    report: dict[str, Any] = {"candidates": len(programs), "devices": devices, "shape": [args.M, args.N, args.K]}
    for mode in ("worker_compiles", "compile_ahead"):
        with tempfile.TemporaryDirectory(prefix="kmcts-candidates-") as root:
            spec = WorkerSpec("kernel_mcts_b200.pool:sm100_evaluator", {"artifact_root": root, "root_us": 100.0})
            with EvaluationPool(devices, spec) as pool:
                pool.prepare(workload)
                compiler = HostCompilePool(root, jobs=args.jobs) if mode == "compile_ahead" else None
                started = time.monotonic()
                try:
                    results = pool.evaluate_many(programs, workload, compile_ahead=compiler)
                finally:
                    if compiler is not None:
                        compiler.close()
                wall = time.monotonic() - started
        valid = sum(r.status == ProposalStatus.VALID for r in results)
        report[mode] = {"wall_s": wall, "evaluations_per_second": len(programs) / wall, "valid": valid,
                        "host_compile_threads": (args.jobs or max(1, (os.cpu_count() or 2) - 1))
                        if mode == "compile_ahead" else 0}
    print(json.dumps(report))


if __name__ == "__main__":
    _measure()
