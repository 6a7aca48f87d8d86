"""The sm_100a evaluation backend (implements the KernelBackend protocol).

Mirrors the reference CUDA backend's contract (src/kernel_mcts/cuda_backend.py):
compile a candidate with the harness into one executable (:129-208), run it
as a subprocess in ``--mode=correctness`` and ``--mode=benchmark`` and parse
the last stdout line as JSON (:466-535), map statuses to the evaluation
exceptions (launch_failure -> CandidateLaunchError, benchmark_failure ->
CandidateBenchmarkError, anything else -> EvaluationInfrastructureError,
subprocess timeout -> CandidateTimeoutError), sample the GPU operating state
around the benchmark (:246-290) and fingerprint the binary (:292-324).

Differences, all B200-driven:
* target ``sm_100a``; the harness is this package's ``harness.cu`` linked
  against libkmcts_gemm_sm100.so (device-side correctness reduction);
* candidates may export the legacy ``bf16_gemm_root`` kernel (fixed 16x16
  launch) or a host launcher ``bf16_gemm_launch`` that owns its launch;
* ``KernelProgram(backend="kmcts_sm100", source=<schedule JSON>)`` selects a
  prebuilt schedule of the library kernel: "compiling" is a static legality
  check, so schedule sweeps pay no nvcc time;
* compiled executables are cached by (normalised source, flags, toolkit);
* the fingerprint hashes the executable bytes — no disassembly;
* workloads with several weighted shapes are evaluated shape by shape (the
  reference backend rejects them, cuda_backend.py:511-512).
"""

from __future__ import annotations

import csv
import hashlib
import json
import os
import re
import shutil
import statistics
import subprocess
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Mapping, Protocol, Sequence

from . import build as native_build
from .domain import BenchmarkResult, KernelProgram, WorkloadContract
from .evaluation import (
    CandidateBenchmarkError,
    CandidateLaunchError,
    CandidateTimeoutError,
    EvaluationInfrastructureError,
)
from .profiling import ProfileParseError, metrics_missing_from_query, parse_ncu_csv, resolve_metric_set

CANDIDATE_BACKEND = "cuda_cpp"
SCHEDULE_BACKEND = "kmcts_sm100"
SCHEDULE_FIELDS = ("tile_m", "tile_n", "tile_k", "stages", "cluster_m", "cluster_n", "persistent", "raster_group",
                   "k_splits")


class CommandRunner(Protocol):
    def __call__(self, command: Sequence[str], *, timeout: float, env: Mapping[str, str]) -> subprocess.CompletedProcess[str]: ...


def run_command(command: Sequence[str], *, timeout: float, env: Mapping[str, str]) -> subprocess.CompletedProcess[str]:
    return subprocess.run(list(command), timeout=timeout, env=dict(env), text=True, capture_output=True, check=False)


def _default_env() -> dict[str, str]:
    env = {"PATH": os.environ.get("PATH", os.defpath), "LANG": "C", "LC_ALL": "C"}
    for name in ("LD_LIBRARY_PATH", "CUDA_VISIBLE_DEVICES", "HOME"):
        if name in os.environ:
            env[name] = os.environ[name]
    return env


@dataclass(frozen=True, slots=True)
class CudaSm100Config:
    artifact_root: Path
    nvcc: str = "nvcc"
    ncu: str = "ncu"
    nvidia_smi: str | None = "nvidia-smi"
    architecture: str = "sm_100a"
    compile_timeout_seconds: float = 180.0
    execution_timeout_seconds: float = 120.0
    profile_timeout_seconds: float = 300.0
    warmup_count: int = 10
    measurement_count: int = 30
    seed: int = 0
    device_index: int = 0
    flush_l2: bool = False
    subprocess_environment: Mapping[str, str] = field(default_factory=_default_env)
    # Where candidate builds are cached (by source, ABI, harness and library);
    # None: under artifact_root.  Backends that share it (a host compile pool
    # and the GPU workers) build each candidate once.
    candidate_cache: Path | None = None

    def __post_init__(self) -> None:
        if min(self.compile_timeout_seconds, self.execution_timeout_seconds, self.profile_timeout_seconds) <= 0:
            raise ValueError("backend timeouts must be positive")
        if self.warmup_count < 0 or self.measurement_count < 1:
            raise ValueError("benchmark counts are invalid")
        if self.architecture != "sm_100a":
            raise ValueError("this backend builds for sm_100a only")


@dataclass(frozen=True, slots=True)
class Sm100Artifact:
    artifact_id: str
    executable: Path
    extra_args: tuple[str, ...] = ()
    abi: str = "library"


@dataclass(frozen=True, slots=True)
class Sm100CompilationResult:
    success: bool
    artifact: Sm100Artifact | None
    stdout: str
    stderr: str
    duration_seconds: float | None
    timed_out: bool = False
    compiler_context: Mapping[str, object] | None = None

    @property
    def artifact_paths(self) -> tuple[str, ...]:
        return (str(self.artifact.executable),) if self.artifact else ()


@dataclass(frozen=True, slots=True)
class Sm100CorrectnessResult:
    success: bool
    maximum_error: float | None
    mean_error: float | None
    failed_test_id: str | None = None
    reference_metadata: Mapping[str, object] = field(default_factory=dict)
    statistics: Mapping[str, object] = field(default_factory=dict)


_PTXAS_LINE = re.compile(
    r"ptxas info\s*:\s*Used (?P<registers>\d+) registers(?:, used (?P<barriers>\d+) barriers)?"
    r"(?:, (?P<smem>\d+) bytes smem)?"
)
_SPILL_LINE = re.compile(r"(?P<stack>\d+) bytes stack frame, (?P<stores>\d+) bytes spill stores, (?P<loads>\d+) bytes spill loads")
_FUNCTION_LINE = re.compile(r"Compiling entry function '(?P<name>[^']+)'")


def parse_ptxas_resources(output: str) -> list[dict[str, object]]:
    """Per-kernel registers / spills / static smem from ``-Xptxas -v`` output
    (the part of the reference's compiler context that reads no PTX/SASS,
    src/kernel_mcts/compiler_context.py:113-137)."""
    kernels: list[dict[str, object]] = []
    current: dict[str, object] | None = None
    for line in output.splitlines():
        if m := _FUNCTION_LINE.search(line):
            current = {"function": m.group("name")}
            kernels.append(current)
        elif current is not None and (m := _SPILL_LINE.search(line)):
            current.update(stack_bytes=int(m.group("stack")), spill_store_bytes=int(m.group("stores")),
                           spill_load_bytes=int(m.group("loads")))
        elif current is not None and (m := _PTXAS_LINE.search(line)):
            current["registers"] = int(m.group("registers"))
            if m.group("barriers"):
                current["barriers"] = int(m.group("barriers"))
            if m.group("smem"):
                current["static_smem_bytes"] = int(m.group("smem"))
    return kernels


def detect_candidate_abi(source: str) -> str:
    """``launcher`` if the candidate defines bf16_gemm_launch, else ``root``."""
    stripped = re.sub(r"//[^\n]*|/\*.*?\*/", " ", source, flags=re.S)
    if re.search(r"\bbf16_gemm_launch\s*\(", stripped):
        return "launcher"
    if re.search(r"\bbf16_gemm_root\s*\(", stripped):
        return "root"
    raise ValueError("candidate defines neither bf16_gemm_root nor bf16_gemm_launch")


# ------------------------------------------------------- multi-shape workloads
#
# A WorkloadContract may carry several weighted shapes (domain.py); the
# evaluator's reward already weights log(T_root / T) per shape
# (evaluation.py).  The backends evaluate shape by shape (the harness keeps
# one shape per run) and merge: correctness passes only if every shape passes,
# and the benchmark reports each shape's median under its shape key plus the
# weighted mean of the medians as ``median_us`` (the expected time of one
# call of the weighted mix).  Single-shape workloads are reported exactly as
# before (no per-shape map).


def shape_mnk(dimensions: Mapping[str, int]) -> tuple[int, int, int]:
    return int(dimensions["M"]), int(dimensions["N"]), int(dimensions["K"])


def merge_correctness(workload: WorkloadContract,
                      results: Sequence[Sm100CorrectnessResult]) -> Sm100CorrectnessResult:
    if len(results) == 1:
        return results[0]
    from .evaluation import shape_key

    keys = [shape_key(shape.dimensions) for shape in workload.shapes]
    sizes = [shape_mnk(shape.dimensions)[0] * shape_mnk(shape.dimensions)[1] for shape in workload.shapes]
    failed = next((key for key, result in zip(keys, results) if not result.success), None)
    maxima = [r.maximum_error for r in results if r.maximum_error is not None]
    means = [(r.mean_error, size) for r, size in zip(results, sizes) if r.mean_error is not None]
    per_shape = {key: dict(r.statistics, success=r.success, maximum_error=r.maximum_error, mean_error=r.mean_error)
                 for key, r in zip(keys, results)}
    metadata = dict(results[0].reference_metadata)
    metadata["per_shape"] = per_shape
    return Sm100CorrectnessResult(
        success=failed is None,
        maximum_error=max(maxima) if maxima else None,
        mean_error=(sum(m * n for m, n in means) / sum(n for _, n in means)) if means else None,
        failed_test_id=failed,
        reference_metadata=metadata,
        statistics={"per_shape": per_shape},
    )


def merge_benchmarks(workload: WorkloadContract, results: Sequence[BenchmarkResult],
                     gpu_operating_state: Mapping[str, object]) -> BenchmarkResult:
    if len(results) == 1:
        return results[0]
    from .evaluation import shape_key

    timings = tuple(t for r in results for t in r.timings_us)
    per_shape = {shape_key(shape.dimensions): r.median_us for shape, r in zip(workload.shapes, results)}
    return BenchmarkResult(
        timings_us=timings,
        median_us=sum(shape.weight * r.median_us for shape, r in zip(workload.shapes, results)),
        warmup_count=results[0].warmup_count,
        mean_us=statistics.fmean(timings),
        stddev_us=statistics.pstdev(timings),
        min_us=min(timings),
        max_us=max(timings),
        per_shape_median_us=per_shape,
        gpu_operating_state=gpu_operating_state,
    )


def schedule_from_source(source: str) -> dict[str, int]:
    try:
        value = json.loads(source)
    except json.JSONDecodeError as error:
        raise ValueError(f"schedule program is not JSON: {error}") from error
    if not isinstance(value, Mapping):
        raise ValueError("schedule program must be a JSON object")
    unknown = set(value) - set(SCHEDULE_FIELDS)
    if unknown:
        raise ValueError(f"unknown schedule fields {sorted(unknown)}")
    return {k: int(v) for k, v in value.items()}


def schedule_program(**schedule: int) -> KernelProgram:
    return KernelProgram(json.dumps(schedule, sort_keys=True), SCHEDULE_BACKEND)


class CudaSm100Backend:
    name = "cuda_sm100"

    def __init__(self, config: CudaSm100Config, *, runner: CommandRunner | None = None) -> None:
        self.config = config
        self._runner = runner or run_command
        self._compiler_output: dict[str, str] = {}
        self._validated_metric_sets: set[str] = set()

    # -------------------------------------------------------------- compile

    def normalize_program(self, program: KernelProgram) -> str:
        if program.backend == SCHEDULE_BACKEND:
            return json.dumps(schedule_from_source(program.source), sort_keys=True)
        without_comments = re.sub(r"//[^\n]*|/\*.*?\*/", " ", program.source, flags=re.S)
        return " ".join(without_comments.split())

    def compile(self, program: KernelProgram, workload: WorkloadContract) -> Sm100CompilationResult:
        self._validate_contract(program, workload)
        if program.backend == SCHEDULE_BACKEND:
            return self._select_schedule(program, workload)
        return self._compile_candidate(program, workload)

    def _select_schedule(self, program: KernelProgram, workload: WorkloadContract) -> Sm100CompilationResult:
        from . import _native

        started = time.monotonic()
        schedule = schedule_from_source(program.source)
        layout = 1 if workload.metadata.get("b_layout", "col") == "row" else 0
        cfg = _native.make_config(**schedule, kernel=_native.KERNEL_TCGEN05)
        for shape in workload.shapes:
            code, why = _native.config_legal(cfg, *shape_mnk(shape.dimensions), layout)
            if code != _native.KMCTS_OK:
                return Sm100CompilationResult(False, None, "", f"statically rejected: {why}",
                                              time.monotonic() - started)
        harness = native_build.build_harness()
        resolved = cfg.as_dict()
        args = tuple(
            f"--{name.replace('_', '-')}={resolved[name]}"
            for name in ("tile_m", "cluster_m", "cluster_n", "tile_n", "tile_k", "stages", "persistent", "raster_group",
                         "k_splits")
        ) + ("--kernel=tcgen05",)
        digest = hashlib.sha256()
        digest.update(harness.read_bytes())
        digest.update(native_build.LIBRARY.read_bytes())
        digest.update(json.dumps(args).encode())
        artifact = Sm100Artifact(digest.hexdigest(), harness, args, "schedule")
        return Sm100CompilationResult(True, artifact, "", "", time.monotonic() - started,
                                      compiler_context={"schedule": schedule, "smem_bytes": _native.config_smem_bytes(cfg, layout)})

    def candidate_key(self, program: KernelProgram) -> tuple[str, str]:
        """(ABI, cache key) of a candidate source's build."""
        abi = detect_candidate_abi(program.source)
        library = native_build.build_library()
        harness_src = native_build.CSRC / "harness.cu"
        key = hashlib.sha256(
            json.dumps([self.normalize_program(program), abi, self.config.architecture,
                        hashlib.sha256(harness_src.read_bytes()).hexdigest(),
                        hashlib.sha256(library.read_bytes()).hexdigest()]).encode()
        ).hexdigest()[:32]
        return abi, key

    def _cache_root(self) -> Path:
        return Path(self.config.candidate_cache or self.config.artifact_root)

    def _harness_object(self, abi: str) -> tuple[Path | None, str]:
        """The harness compiled once per ABI (relocatable device code), so a
        candidate build compiles only the candidate and links.  Returns the
        object, or None and the compiler output on failure."""
        harness_src = native_build.CSRC / "harness.cu"
        digest = hashlib.sha256(harness_src.read_bytes() + (native_build.INCLUDE / "kmcts_gemm.h").read_bytes()
                                + abi.encode() + self.config.architecture.encode()).hexdigest()[:24]
        obj = self._cache_root() / f"harness-{abi}-{digest}.o"
        if obj.exists():
            return obj, ""
        obj.parent.mkdir(parents=True, exist_ok=True)
        tmp = obj.with_name(f"{obj.name}.{os.getpid()}.{threading.get_ident()}.tmp")
        command = [
            _resolve_tool(self.config.nvcc), "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O3",
            "-rdc=true", "-DKMCTS_CANDIDATE_ROOT" if abi == "root" else "-DKMCTS_CANDIDATE_LAUNCHER",
            f"-I{native_build.INCLUDE}", "-c", str(harness_src), "-o", str(tmp),
        ]
        completed = self._runner(command, timeout=self.config.compile_timeout_seconds,
                                 env=self.config.subprocess_environment)
        if completed.returncode != 0 or not tmp.exists():
            return None, f"{completed.stdout}\n{completed.stderr}"
        os.replace(tmp, obj)  # atomic: concurrent builders leave one complete object
        return obj, ""

    def _compile_candidate(self, program: KernelProgram, workload: WorkloadContract) -> Sm100CompilationResult:
        """nvcc build of a candidate source against the evaluation harness
        (src/kernel_mcts/cuda_backend.py:129-208 builds candidate and harness
        in one nvcc call; here the harness is compiled once per ABI and each
        candidate is compiled alone, -rdc, and linked to it).  Builds are
        cached on disk by key, with their compiler output, so another
        process sharing ``candidate_cache`` reuses them."""
        try:
            abi, key = self.candidate_key(program)
        except ValueError as error:
            return Sm100CompilationResult(False, None, "", str(error), 0.0)
        artifact_dir = self._cache_root() / f"cand-{key}"
        executable = artifact_dir / "evaluate"
        log = artifact_dir / "compile.log"
        started = time.monotonic()
        if executable.exists() and (key in self._compiler_output or log.exists()):
            output = self._compiler_output.get(key)
            if output is None:
                output = log.read_text(encoding="utf-8", errors="replace")
                self._compiler_output[key] = output
            return self._compiled(executable, abi, "", output, time.monotonic() - started)
        artifact_dir.mkdir(parents=True, exist_ok=True)
        try:
            harness_obj, harness_output = self._harness_object(abi)
        except subprocess.TimeoutExpired as error:
            return Sm100CompilationResult(False, None, _bounded(_text(error.stdout)), _bounded(_text(error.stderr)),
                                          time.monotonic() - started, True)
        except OSError as error:
            raise EvaluationInfrastructureError("CUDA compiler could not be executed") from error
        if harness_obj is None:
            raise EvaluationInfrastructureError("the evaluation harness failed to compile: "
                                                + _bounded(harness_output, 2000))
        tag = f"{os.getpid()}.{threading.get_ident()}"
        candidate = artifact_dir / f"candidate.{tag}.cu"
        candidate.write_text(program.source, encoding="utf-8")
        candidate_obj = artifact_dir / f"candidate.{tag}.o"
        tmp_executable = artifact_dir / f"evaluate.{tag}.tmp"
        arch = ["-gencode", "arch=compute_100a,code=sm_100a"]
        compile_command = [
            _resolve_tool(self.config.nvcc), *arch, "-std=c++17", "-O3", "-rdc=true", "-Xptxas=-v",
            "-DKMCTS_CANDIDATE_ROOT" if abi == "root" else "-DKMCTS_CANDIDATE_LAUNCHER",
            f"-I{native_build.INCLUDE}", "-c", str(candidate), "-o", str(candidate_obj),
        ]
        link_command = [
            _resolve_tool(self.config.nvcc), *arch, "-rdc=true", str(candidate_obj), str(harness_obj),
            f"-L{native_build.LIB_DIR}", "-lkmcts_gemm_sm100", "-lcublas",
            "-Xlinker", f"-rpath={native_build.LIB_DIR}",
            "-o", str(tmp_executable),
        ]
        try:
            completed = self._runner(compile_command, timeout=self.config.compile_timeout_seconds,
                                     env=self.config.subprocess_environment)
            if completed.returncode == 0:
                linked = self._runner(link_command, timeout=self.config.compile_timeout_seconds,
                                      env=self.config.subprocess_environment)
                if linked.returncode != 0:
                    completed = subprocess.CompletedProcess(link_command, linked.returncode,
                                                            completed.stdout + linked.stdout,
                                                            completed.stderr + linked.stderr)
        except subprocess.TimeoutExpired as error:
            return Sm100CompilationResult(False, None, _bounded(_text(error.stdout)), _bounded(_text(error.stderr)),
                                          time.monotonic() - started, True)
        except OSError as error:
            raise EvaluationInfrastructureError("CUDA compiler could not be executed") from error
        finally:
            for leftover in (candidate_obj,):
                try:
                    leftover.unlink()
                except OSError:
                    pass
        duration = time.monotonic() - started
        if completed.returncode != 0 or not tmp_executable.exists():
            return Sm100CompilationResult(False, None, _bounded(completed.stdout), _bounded(completed.stderr), duration)
        output = f"{completed.stdout}\n{completed.stderr}"
        os.replace(candidate, artifact_dir / "candidate.cu")
        os.replace(tmp_executable, executable)  # atomic: a concurrent builder's copy is equivalent
        log.write_text(output, encoding="utf-8")
        self._compiler_output[key] = output
        return self._compiled(executable, abi, _bounded(completed.stdout), output, duration)

    def _compiled(self, executable: Path, abi: str, stdout: str, output: str, duration: float) -> Sm100CompilationResult:
        artifact_id = hashlib.sha256(executable.read_bytes()).hexdigest()
        context = {"architecture": self.config.architecture, "abi": abi,
                   "ptxas": parse_ptxas_resources(output)}
        return Sm100CompilationResult(True, Sm100Artifact(artifact_id, executable, ("--kernel=candidate",), abi),
                                      stdout, _bounded(output), duration, compiler_context=context)

    # ---------------------------------------------------------------- run

    def check_correctness(self, artifact: Sm100Artifact, workload: WorkloadContract) -> Sm100CorrectnessResult:
        results = []
        for shape in workload.shapes:
            payload = self._execute(artifact, workload, "correctness", shape.dimensions)
            extra = {k: payload[k] for k in ("max_ulp", "n_gt_1ulp", "ulp_hist", "n_nonfinite", "kernel")
                     if k in payload}
            results.append(Sm100CorrectnessResult(
                success=bool(payload["success"]),
                maximum_error=_optional_float(payload.get("maximum_error")),
                mean_error=_optional_float(payload.get("mean_error")),
                failed_test_id=payload.get("failed_test_id"),
                reference_metadata={**payload.get("reference_metadata", {}), **extra},
                statistics=extra,
            ))
        return merge_correctness(workload, results)

    def benchmark(self, artifact: Sm100Artifact, workload: WorkloadContract) -> BenchmarkResult:
        before = self.gpu_operating_state()
        payloads = [self._execute(artifact, workload, "benchmark", shape.dimensions) for shape in workload.shapes]
        after = self.gpu_operating_state()
        results = []
        for payload in payloads:
            timings = tuple(float(v) for v in payload["timings_us"])
            if len(timings) != self.config.measurement_count:
                raise EvaluationInfrastructureError("worker returned an unexpected timing count")
            results.append(BenchmarkResult(
                timings_us=timings,
                median_us=statistics.median(timings),
                warmup_count=self.config.warmup_count,
                mean_us=statistics.fmean(timings),
                stddev_us=statistics.pstdev(timings),
                min_us=min(timings),
                max_us=max(timings),
                gpu_operating_state={"before": before, "after": after},
            ))
        return merge_benchmarks(workload, results, {"before": before, "after": after})

    def _command(self, artifact: Sm100Artifact, workload: WorkloadContract, mode: str,
                 dimensions: Mapping[str, int] | None = None) -> list[str]:
        shape = dimensions if dimensions is not None else workload.shapes[0].dimensions
        command = [
            str(artifact.executable),
            f"--mode={mode}",
            f"--M={shape['M']}",
            f"--N={shape['N']}",
            f"--K={shape['K']}",
            f"--rtol={workload.rtol}",
            f"--atol={workload.atol}",
            f"--seed={self.config.seed}",
            f"--warmups={self.config.warmup_count}",
            f"--measurements={self.config.measurement_count}",
            f"--b-layout={workload.metadata.get('b_layout', 'col')}",
            f"--inputs={workload.metadata.get('inputs', 'uniform')}",
            f"--flush-l2={1 if self.config.flush_l2 else 0}",
        ]
        return command + list(artifact.extra_args)

    def _execute(self, artifact: Sm100Artifact, workload: WorkloadContract, mode: str,
                 dimensions: Mapping[str, int] | None = None) -> dict[str, object]:
        command = self._command(artifact, workload, mode, dimensions)
        try:
            result = self._runner(command, timeout=self.config.execution_timeout_seconds,
                                  env=self.config.subprocess_environment)
        except subprocess.TimeoutExpired as error:
            raise CandidateTimeoutError("candidate execution timed out") from error
        except OSError as error:
            raise EvaluationInfrastructureError("evaluation harness could not be executed") from error
        payload = parse_payload(result.stdout)
        status = payload.get("status")
        if status == "launch_failure":
            raise CandidateLaunchError(f"candidate launch failed ({payload.get('reason', 'unknown')})")
        if status == "benchmark_failure":
            raise CandidateBenchmarkError("candidate benchmark failed")
        if result.returncode != 0 or status != "ok":
            raise EvaluationInfrastructureError("evaluation harness failed")
        return payload

    # ------------------------------------------------------- observability

    def gpu_operating_state(self) -> Mapping[str, object]:
        if self.config.nvidia_smi is None:
            return {"status": "unavailable"}
        fields = ("temperature.gpu", "clocks.sm", "clocks.mem", "power.draw", "power.limit", "pstate",
                  "utilization.gpu", "utilization.memory", "clocks_event_reasons.active")
        command = [_resolve_tool(self.config.nvidia_smi), f"--query-gpu={','.join(fields)}",
                   "--format=csv,noheader,nounits", f"--id={self.config.device_index}"]
        try:
            result = self._runner(command, timeout=min(10.0, self.config.execution_timeout_seconds),
                                  env=self.config.subprocess_environment)
        except (OSError, subprocess.TimeoutExpired):
            return {"status": "unavailable"}
        rows = list(csv.reader(result.stdout.splitlines())) if result.returncode == 0 else []
        if len(rows) != 1 or len(rows[0]) != len(fields):
            return {"status": "unavailable"}
        values: dict[str, object] = {"status": "observed"}
        for name, raw in zip(fields, rows[0]):
            raw = raw.strip()
            if name in ("pstate", "clocks_event_reasons.active"):
                values[name] = raw
            else:
                try:
                    values[name] = float(raw)
                except ValueError:
                    values[name] = None
        return values

    def binary_fingerprint(self, artifact: Sm100Artifact, launch_config: Mapping[str, object]) -> str:
        digest = hashlib.sha256(Path(artifact.executable).read_bytes())
        digest.update(json.dumps(list(artifact.extra_args)).encode())
        return digest.hexdigest()

    def evaluation_metadata(self, artifact: Sm100Artifact) -> Mapping[str, object]:
        return {"backend": self.name, "architecture": self.config.architecture, "abi": artifact.abi,
                "schedule_args": list(artifact.extra_args)}

    def profile_target_command(self, artifact: Sm100Artifact, workload: WorkloadContract) -> list[str]:
        """The harness command a lightweight profile runs under ncu: one
        benchmark launch, no warm-ups (as src/kernel_mcts/cuda_backend.py:345-368)."""
        command = self._command(artifact, workload, "benchmark")
        return [command[0], *[arg for arg in command[1:] if not arg.startswith(("--warmups=", "--measurements="))],
                "--warmups=0", "--measurements=1"]

    def validate_metric_set(self, definition) -> None:
        """Checks once per metric set that this GPU's ncu offers every metric
        in it (``ncu --query-metrics-mode all --devices 0``, the device the
        harness runs on), as src/kernel_mcts/cuda_backend.py:413-461 does for
        non-default sets.  Raises EvaluationInfrastructureError naming what is
        missing."""
        if definition.id == "lightweight_v1" or definition.id in self._validated_metric_sets:
            return
        command = [_resolve_tool(self.config.ncu), "--query-metrics-mode", "all", "--devices", "0"]
        try:
            result = self._runner(command, timeout=self.config.profile_timeout_seconds,
                                  env=self.config.subprocess_environment)
        except (OSError, subprocess.TimeoutExpired) as error:
            raise EvaluationInfrastructureError("Nsight Compute metric validation could not be completed") from error
        if result.returncode != 0:
            raise EvaluationInfrastructureError(
                "Nsight Compute metric validation failed: " + _bounded(result.stderr + result.stdout, 2000))
        missing = metrics_missing_from_query(definition, f"{result.stdout}\n{result.stderr}")
        if missing:
            preview = ", ".join(missing[:8]) + (", ..." if len(missing) > 8 else "")
            raise EvaluationInfrastructureError(
                f"Nsight Compute metric set {definition.id!r} is unavailable; missing: {preview}")
        self._validated_metric_sets.add(definition.id)

    def lightweight_profile(self, artifact: Sm100Artifact, workload: WorkloadContract,
                            metric_set: str = "lightweight_v1") -> Mapping[str, object]:
        try:
            definition = resolve_metric_set(metric_set, self.config.architecture)
        except ValueError as error:
            raise EvaluationInfrastructureError(str(error)) from error
        self.validate_metric_set(definition)
        command = [
            _resolve_tool(self.config.ncu), "--csv", "--page", "raw", "--log-file", "stdout",
            "--clock-control", "none", "--kernel-name-base", "function",
            "--kernel-name", f"regex:{definition.kernel_regex(artifact.abi)}",
            "--launch-count", "1", "--metrics", ",".join(definition.metrics),
            *self.profile_target_command(artifact, workload),
        ]
        try:
            result = self._runner(command, timeout=self.config.profile_timeout_seconds,
                                  env=self.config.subprocess_environment)
        except (OSError, subprocess.TimeoutExpired) as error:
            raise EvaluationInfrastructureError("Nsight Compute profiling could not be completed") from error
        if result.returncode != 0:
            raise EvaluationInfrastructureError("Nsight Compute profiling failed: " + _bounded(result.stderr + result.stdout, 2000))
        metrics = None
        for text in (result.stdout, result.stderr):
            try:
                metrics = parse_ncu_csv(text, definition.metrics)
                break
            except ProfileParseError:
                continue
        if metrics is None:
            raise EvaluationInfrastructureError("Nsight Compute returned malformed CSV")
        return {
            "schema_version": definition.schema_version,
            "profiler": "ncu",
            "metric_set": definition.id,
            "target": {"architecture": self.config.architecture},
            "resolved_metrics": list(definition.metrics),
            "artifact_id": artifact.artifact_id,
            "summary": {alias: metrics[name]["value"] for name, alias in definition.aliases.items()},
            "metrics": metrics,
        }

    def full_profile(self, artifact: Sm100Artifact, workload: WorkloadContract) -> Mapping[str, object]:
        raise NotImplementedError("full profiles are taken with ncu --set full outside the evaluator")

    @staticmethod
    def _validate_contract(program: KernelProgram, workload: WorkloadContract) -> None:
        if program.backend not in (CANDIDATE_BACKEND, SCHEDULE_BACKEND):
            raise ValueError(f"unsupported program backend {program.backend!r}")
        if workload.operation != "gemm" or workload.dtype != "bfloat16":
            raise ValueError("CudaSm100Backend supports only BF16 GEMM")
        if workload.metadata.get("entry_point") != "bf16_gemm_root":
            raise ValueError("BF16 GEMM workload must use the bf16_gemm_root entry point")


def parse_payload(stdout: str) -> dict[str, object]:
    try:
        value = json.loads(stdout.strip().splitlines()[-1])
    except (IndexError, json.JSONDecodeError) as error:
        raise EvaluationInfrastructureError("worker returned malformed JSON") from error
    if not isinstance(value, dict):
        raise EvaluationInfrastructureError("worker JSON payload must be an object")
    return value


def _optional_float(value: object) -> float | None:
    return None if value is None else float(value)


def _text(value: object) -> str:
    if value is None:
        return ""
    return value.decode(errors="replace") if isinstance(value, bytes) else str(value)


def _bounded(value: str, limit: int = 64_000) -> str:
    return value[-limit:]


def _resolve_tool(command: str) -> str:
    if os.sep in command:
        return command
    return shutil.which(command) or command
