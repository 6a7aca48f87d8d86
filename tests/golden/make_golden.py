"""Generates the golden fixtures that pin the CPU oracle to the reference.

Two steps, because the reference's GEMM is GPU code:

1. ``python tests/golden/make_golden.py inputs`` (any machine with the
   reference tree): runs the reference's own input generator, compiled from
   src/kernel_mcts/benchmarks/kernels/bf16_input_generator.cu by oracle/Makefile
   into oracle/_ref/bf16_input_generator, and stores its A/B streams
   (full arrays for small cases, SHA-256 digests for large ones) in
   ``reference_inputs.npz``.

2. ``python tests/golden/make_golden.py outputs --out DIR`` (on a B200): runs
   the reference's own root kernel (bf16_gemm_root.cu, built for sm_100a into
   oracle/_ref/libref_root.so) and the reference's cuBLAS entry point
   (bf16_reference.cu, oracle/_ref/libkernel_mcts_bf16_reference.so) on those
   inputs and writes ``reference_outputs.npz`` to DIR; copy it next to this
   script.

The fixtures are data only; the tests never run the reference.
"""

from __future__ import annotations

import argparse
import ctypes
import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import oracle  # noqa: E402

# (name, M, N, K, seed, store_full_arrays)
CASES = (
    ("m16n16k16_s0", 16, 16, 16, 0, True),
    ("m37n29k53_s7", 37, 29, 53, 7, True),
    ("m64n48k40_s3", 64, 48, 40, 3, True),
    ("m128n96k256_s0", 128, 96, 256, 0, True),
    ("m256n256k256_s0", 256, 256, 256, 0, False),
    ("m512n384k320_s11", 512, 384, 320, 11, False),
)

# Integer-valued cases (torch.randint in {-2..2}, seed given), run through the
# reference root kernel too: FP32 accumulation is exact, so every FP32
# summation order gives these bits.
INT_CASES = (
    ("int_m64n64k64_s0", 64, 64, 64, 0),
    ("int_m96n80k200_s5", 96, 80, 200, 5),
)


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def make_inputs() -> None:
    oracle.build(reference=True)
    if not oracle.REF_GENERATOR.exists():
        raise SystemExit("reference generator not built (is the reference tree present?)")
    payload: dict[str, np.ndarray] = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, m, n, k, seed, full in CASES:
            a, b = oracle.reference_generator_inputs(m, n, k, seed, Path(tmp))
            payload[f"{name}.shape"] = np.array([m, n, k, seed], dtype=np.int64)
            if full:
                payload[f"{name}.A"] = a
                payload[f"{name}.B"] = b
            payload[f"{name}.A_sha256"] = np.array(sha256(a))
            payload[f"{name}.B_sha256"] = np.array(sha256(b))
    np.savez_compressed(HERE / "reference_inputs.npz", **payload)
    print("wrote", HERE / "reference_inputs.npz")


def make_outputs(out_dir: Path) -> None:
    import torch

    root = ctypes.CDLL(str(oracle.REF_ROOT_LIB))
    root.kmcts_ref_root_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    root.kmcts_ref_root_gemm.restype = ctypes.c_int
    cublas = ctypes.CDLL(str(oracle.REF_CUBLAS_LIB))
    cublas.kernel_mcts_bf16_reference.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    cublas.kernel_mcts_bf16_reference.restype = ctypes.c_int

    def run(fn, a_bits: np.ndarray, b_bits: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        a = torch.from_numpy(a_bits.view(np.int16).copy()).cuda()
        b = torch.from_numpy(b_bits.view(np.int16).copy()).cuda()
        c = torch.zeros((m, n), dtype=torch.int16, device="cuda")
        rc = fn(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k)
        torch.cuda.synchronize()
        if rc != 0:
            raise RuntimeError(f"reference call failed with {rc}")
        return c.cpu().numpy().view(np.uint16)

    payload: dict[str, np.ndarray] = {}
    for name, m, n, k, seed, full in CASES:
        a, b = oracle.uniform_inputs(m, n, k, seed)
        c_root = run(root.kmcts_ref_root_gemm, a, b, m, n, k)
        c_cublas = run(cublas.kernel_mcts_bf16_reference, a, b, m, n, k)
        if full:
            payload[f"{name}.C_root"] = c_root
            payload[f"{name}.C_cublas"] = c_cublas
        payload[f"{name}.C_root_sha256"] = np.array(sha256(c_root))
        payload[f"{name}.C_cublas_sha256"] = np.array(sha256(c_cublas))
    for name, m, n, k, seed in INT_CASES:
        a_t, b_t = oracle.integer_inputs(m, n, k, seed)
        a, b = oracle.torch_bits(a_t), oracle.torch_bits(b_t)
        payload[f"{name}.shape"] = np.array([m, n, k, seed], dtype=np.int64)
        payload[f"{name}.C_root"] = run(root.kmcts_ref_root_gemm, a, b, m, n, k)
        payload[f"{name}.C_cublas"] = run(cublas.kernel_mcts_bf16_reference, a, b, m, n, k)
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "reference_outputs.npz", **payload)
    print("wrote", out_dir / "reference_outputs.npz")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("step", choices=("inputs", "outputs"))
    parser.add_argument("--out", type=Path, default=HERE)
    args = parser.parse_args()
    if args.step == "inputs":
        make_inputs()
    else:
        make_outputs(args.out)


if __name__ == "__main__":
    main()
