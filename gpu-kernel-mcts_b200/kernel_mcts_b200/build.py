"""Builds the native parts of kernel_mcts_b200 in-tree with nvcc (sm_100a).

Outputs (git-ignored, shipped with the source tree):
  _lib/libkmcts_gemm_sm100.so   the C-ABI GEMM library (include/kmcts_gemm.h)
  _lib/kmcts_bf16_eval          the evaluation harness executable built on it

Run as ``python -m kernel_mcts_b200.build`` (with gpu-kernel-mcts_b200/ on
sys.path) or call :func:`build_all`.  Rebuilds only what is older than its
sources.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent.parent
CSRC = PACKAGE_DIR / "csrc"
LIB_DIR = PACKAGE_DIR / "_lib"
INCLUDE = REPO_ROOT / "include"
OBJ_DIR = LIB_DIR / "obj"

LIBRARY = LIB_DIR / "libkmcts_gemm_sm100.so"
HARNESS = LIB_DIR / "kmcts_bf16_eval"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}"]

LIBRARY_SOURCES = ("gemm_tcgen05.cu", "gemm_tcgen05_pair.cu", "gemm_tcgen05_stream.cu", "gemm_simt.cu", "compare.cu",
                   "capi.cu", "ipc.cu", "selftest.cu", "workspace.cu", "host_gemm.cu")
HEADERS = ("ptx_sm100.cuh", "gemm_common.cuh", "kmcts_internal.h")


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the sm_100a build needs the CUDA toolkit")
    return found


def _newest(paths) -> float:
    return max(Path(p).stat().st_mtime for p in paths)


def _stale(target: Path, deps) -> bool:
    return not target.exists() or target.stat().st_mtime < _newest(deps)


def _run(command: list[str]) -> None:
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(
            "build step failed:\n" + " ".join(command) + "\n" + result.stdout + result.stderr
        )


def build_library(verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "kmcts_gemm.h"]
    jobs = []
    objects = []
    for name in LIBRARY_SOURCES:
        src = CSRC / name
        obj = OBJ_DIR / (Path(name).stem + ".o")
        objects.append(obj)
        if _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append([nvcc(), *COMMON_FLAGS, "-Xcompiler", "-fPIC", "-c", str(src), "-o", str(obj)])
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=len(jobs)) as pool:
            for cmd, fut in [(cmd, pool.submit(_run, cmd)) for cmd in jobs]:
                if verbose:
                    print(" ".join(cmd), file=sys.stderr)
                fut.result()
    if _stale(LIBRARY, objects):
        _run([nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIBRARY), *map(str, objects)])
    return LIBRARY


def cutlass_include() -> Path | None:
    """CUTLASS headers vendored in this image (flashinfer's copy), if present.
    Used only for the CUTLASS column of the vendor baselines."""
    import importlib.util

    spec = importlib.util.find_spec("flashinfer")
    if spec is None or spec.origin is None:
        return None
    path = Path(spec.origin).parent / "data" / "cutlass" / "include"
    return path if (path / "cutlass" / "gemm" / "device" / "gemm.h").exists() else None


def build_harness(verbose: bool = False) -> Path:
    src = CSRC / "harness.cu"
    if not src.exists():
        return HARNESS
    lib = build_library(verbose)
    sources = [src]
    flags = ["-DKMCTS_HAVE_CUTLASS=0"]
    cutlass = cutlass_include()
    if cutlass is not None:
        sources.append(CSRC / "vendor_cutlass.cu")
        flags = ["-DKMCTS_HAVE_CUTLASS=1", f"-I{cutlass}"]
    if _stale(HARNESS, [*sources, lib, INCLUDE / "kmcts_gemm.h", Path(__file__)]):
        cmd = [
            nvcc(), *COMMON_FLAGS, *flags, *map(str, sources), "-o", str(HARNESS),
            f"-L{LIB_DIR}", "-lkmcts_gemm_sm100", "-lcublas",
            "-Xlinker", f"-rpath={LIB_DIR}", "-Xlinker", "-rpath=$ORIGIN",
        ]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        _run(cmd)
    return HARNESS


def build_all(verbose: bool = False) -> None:
    build_library(verbose)
    build_harness(verbose)


if __name__ == "__main__":
    build_all(verbose=True)
    print(LIBRARY)
