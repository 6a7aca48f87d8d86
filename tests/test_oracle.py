"""The CPU oracle against the reference's own golden vectors and known answers."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def _golden_inputs():
    return np.load(GOLDEN / "reference_inputs.npz")


def _case_names(data) -> list[str]:
    return sorted({key.split(".")[0] for key in data.files if key.endswith(".shape")})


def test_mt19937_known_answer():
    # The 10000th output of a default-seeded (5489) mt19937 is fixed by the
    # C++ standard ([rand.predef]): 4123659995.
    words = oracle.mt19937_words(5489, 10000)
    assert int(words[-1]) == 4123659995


def test_uniform_inputs_match_reference_generator_fixtures():
    data = _golden_inputs()
    names = _case_names(data)
    assert len(names) >= 6
    for name in names:
        m, n, k, seed = (int(v) for v in data[f"{name}.shape"])
        a, b = oracle.uniform_inputs(m, n, k, seed)
        assert oracle.__dict__  # oracle module loaded
        if f"{name}.A" in data.files:
            np.testing.assert_array_equal(a, data[f"{name}.A"])
            np.testing.assert_array_equal(b, data[f"{name}.B"])
        import hashlib

        assert hashlib.sha256(a.tobytes()).hexdigest() == str(data[f"{name}.A_sha256"])
        assert hashlib.sha256(b.tobytes()).hexdigest() == str(data[f"{name}.B_sha256"])


def test_uniform_inputs_range_and_grid():
    a, b = oracle.uniform_inputs(64, 64, 64, 0)
    af = oracle.bf16_bits_to_float(a)
    assert af.min() >= -0.25 and af.max() <= 0.25
    # Every value is a BF16 rounding of a float in range: re-rounding is identity.
    np.testing.assert_array_equal(oracle.float_to_bf16_bits(af), a)


@pytest.mark.skipif(not (GOLDEN / "reference_outputs.npz").exists(), reason="root outputs not generated yet")
def test_root_gemm_matches_reference_root_kernel_bit_exact():
    inputs = _golden_inputs()
    outputs = np.load(GOLDEN / "reference_outputs.npz")
    import hashlib

    for name in _case_names(inputs):
        m, n, k, seed = (int(v) for v in inputs[f"{name}.shape"])
        a, b = oracle.uniform_inputs(m, n, k, seed)
        c = oracle.root_gemm(a, b, "col")
        if f"{name}.C_root" in outputs.files:
            np.testing.assert_array_equal(c, outputs[f"{name}.C_root"])
        assert hashlib.sha256(c.tobytes()).hexdigest() == str(outputs[f"{name}.C_root_sha256"])


@pytest.mark.skipif(not (GOLDEN / "reference_outputs.npz").exists(), reason="root outputs not generated yet")
def test_integer_cases_match_reference_root_and_cublas():
    outputs = np.load(GOLDEN / "reference_outputs.npz")
    names = sorted({key.split(".")[0] for key in outputs.files if key.startswith("int_") and key.endswith(".shape")})
    assert names
    for name in names:
        m, n, k, seed = (int(v) for v in outputs[f"{name}.shape"])
        a_t, b_t = oracle.integer_inputs(m, n, k, seed)
        c = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(b_t), "col")
        np.testing.assert_array_equal(c, outputs[f"{name}.C_root"])
        assert np.all(oracle.ulp_distance(c, outputs[f"{name}.C_cublas"]) == 0)


def test_root_gemm_integer_inputs_exact():
    a_t, b_t = oracle.integer_inputs(48, 40, 96, seed=3)
    c = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(b_t), "col")
    exact = a_t.double().numpy() @ b_t.double().numpy().T
    np.testing.assert_array_equal(oracle.bf16_bits_to_float(c).astype(np.float64), exact)


def test_root_gemm_row_layout_equals_col_layout():
    a, b = oracle.uniform_inputs(33, 24, 70, 5)
    c_col = oracle.root_gemm(a, b, "col")
    c_row = oracle.root_gemm(a, np.ascontiguousarray(b.T), "row")
    np.testing.assert_array_equal(c_col, c_row)


def test_root_gemm_known_answers():
    # identity: C = A exactly
    import torch

    a_t, _ = oracle.integer_inputs(32, 32, 32, seed=1)
    eye = torch.eye(32, dtype=torch.bfloat16)
    c = oracle.root_gemm(oracle.torch_bits(a_t), oracle.torch_bits(eye), "col")
    np.testing.assert_array_equal(c, oracle.torch_bits(a_t))
    # all-zero B: C == 0 (as values)
    zb = np.zeros((16, 32), dtype=np.uint16)
    c0 = oracle.root_gemm(oracle.torch_bits(a_t), zb, "col")
    assert np.all(oracle.bf16_bits_to_float(c0) == 0.0)
    # rank-1 integer outer product via K=1
    u = torch.tensor([[1.0], [-2.0], [3.0]], dtype=torch.bfloat16)
    v = torch.tensor([[2.0], [5.0]], dtype=torch.bfloat16)
    c1 = oracle.root_gemm(oracle.torch_bits(u), oracle.torch_bits(v), "col")
    np.testing.assert_array_equal(oracle.bf16_bits_to_float(c1), np.array([[2, 5], [-4, -10], [6, 15]], np.float32))


def test_float_to_bf16_rne_ties():
    # 1 + 2^-8 is exactly halfway between 1 and 1 + 2^-7: ties to even (1.0).
    # 1 + 3*2^-8 is halfway between 1+2^-7 and 1+2^-6: ties to even (1 + 2^-6).
    vals = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -(1.0 + 2.0 ** -8), 1.0 + 2.0 ** -8 + 2.0 ** -20], np.float32)
    bits = oracle.float_to_bf16_bits(vals)
    assert list(bits) == [0x3F80, 0x3F82, 0xBF80, 0x3F81]
    lib = oracle.load()
    assert [lib.kmcts_oracle_float_to_bf16(float(v)) for v in vals] == list(bits)
    assert oracle.float_to_bf16_bits(np.array([np.nan], np.float32))[0] == 0x7FFF


def test_ulp_distance_properties():
    assert oracle.ulp_distance(np.array([0x0000]), np.array([0x8000]))[0] == 0  # +0 vs -0
    assert oracle.ulp_distance(np.array([0x3F80]), np.array([0x3F81]))[0] == 1
    assert oracle.ulp_distance(np.array([0x0001]), np.array([0x8001]))[0] == 2  # across zero
    assert oracle.ulp_distance(np.array([0x7FC0]), np.array([0x3F80]))[0] == 65535
    lib = oracle.load()
    assert lib.kmcts_oracle_ulp_distance(0x0001, 0x8001) == 2


def test_harness_check_semantics():
    ref = oracle.float_to_bf16_bits(np.array([1.0, -2.0, 0.0, 100.0], np.float32))
    same = oracle.harness_check(ref, ref)
    assert same == {"success": True, "maximum_error": 0.0, "mean_error": 0.0}
    # error 0.03 > 0.02 + 0.02*0 at ref 0 -> fail
    c = oracle.float_to_bf16_bits(np.array([1.0, -2.0, 0.03125, 100.0], np.float32))
    res = oracle.harness_check(c, ref)
    assert not res["success"] and res["maximum_error"] == pytest.approx(0.03125)
    # non-finite output fails even when the reference matches
    inf = oracle.float_to_bf16_bits(np.array([np.inf, -2.0, 0.0, 100.0], np.float32))
    assert not oracle.harness_check(inf, inf)["success"]


def test_parity_report_accepts_reordered_fp32_sums():
    import torch

    a, b = oracle.randn_inputs(64, 64, 512, seed=0)
    ref32 = oracle.torch_bits(oracle.torch_reference(a, b))
    ref64, mag = oracle.fp64_reference(a, b)
    # a different FP32 summation order: reversed K
    alt = torch.matmul(a.float().flip(1), b.float().flip(1).T).to(torch.bfloat16)
    report = oracle.parity_report(oracle.torch_bits(alt), ref32, ref64, mag, 512)
    assert report["passed"], report
    # a planted 3-ulp error on a large element is caught
    bad = oracle.torch_bits(alt).copy()
    idx = np.unravel_index(np.argmax(np.abs(ref64)), ref64.shape)
    bad[idx] = np.uint16(int(bad[idx]) + 3)
    assert not oracle.parity_report(bad, ref32, ref64, mag, 512)["passed"]
