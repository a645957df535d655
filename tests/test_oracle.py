"""The oracle, pinned against outputs of the reference itself.

tests/golden/gemm_cases.npz holds inputs and outputs of the reference's Triton
kernels (kernels/grouped_gemm.py:321-482, kernels/matmul.py:223-273) executed
by the Triton CPU interpreter (tests/golden/make_golden.py).  The oracle must
reproduce them within the output type's rounding: the reference accumulates
in fp32 and casts once, the oracle sums in float64 and casts once.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gemm as oracle
from tests.golden_data import load_gemm_cases

CASES = load_gemm_cases()


def _tolerance(dtype: str) -> tuple[float, float]:
    # fp16: one output ulp at |C| ~ 1 plus fp32-vs-fp64 accumulation order;
    # fp32: accumulation-order differences only.
    return (2e-3, 2e-3) if dtype == "fp16" else (1e-5, 1e-6)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_reproduces_reference_outputs(case):
    if case["kind"] == "single_strided":
        a = case["a_base"][:, ::2].astype(np.float64)
        b = case["b_base"][:, ::2].astype(np.float64)
        expected = oracle.matmul(a, b, "fp32")
        got = case["c_base"][:, ::2].astype(np.float64)
        # The reference ran with input_precision="tf32"; the interpreter's dot
        # keeps fp32 products, so the fp32 oracle agrees to TF32's tolerance.
        np.testing.assert_allclose(got, expected, rtol=2e-3, atol=2e-3)
        assert np.isnan(case["c_base"][:, 1::2]).all(), "reference wrote outside the strided view"
        return
    rtol, atol = _tolerance(case["dtype"])
    for e, (a, b, c) in enumerate(zip(case["a"], case["b"], case["c"])):
        if case["kind"] == "gate_up":
            expected = oracle.gate_up(a.astype(np.float64), b.astype(np.float64), case["dtype"])
        else:
            expected = oracle.matmul(a.astype(np.float64), b.astype(np.float64), case["dtype"])
        got = c.astype(np.float64)
        assert np.isfinite(got).all(), f"{case['name']}: reference left unwritten outputs"
        np.testing.assert_allclose(got, expected, rtol=rtol, atol=atol, err_msg=f"{case['name']} problem {e}")
        assert oracle.relative_frobenius(got, expected) < (1e-3 if case["dtype"] == "fp16" else 1e-6)


def test_golden_cases_cover_the_reference_test_shapes():
    names = {c["name"] for c in CASES}
    for required in ("grouped_generic_fp32", "grouped_generic_fp16", "grouped_homog_fp32", "grouped_homog_fp16",
                     "gate_up_fp16", "tutorial_homog_fp16", "moe_narrow_fp16", "moe_tail_fp16", "moe_hetero_fp16",
                     "single_fp32_strided_tf32"):
        assert required in names
    singles = {c["name"] for c in CASES if c["kind"] == "single"}
    assert {"single_fp16_1x5x3", "single_fp32_17x13x31", "single_fp32_33x70x65"} <= singles


@pytest.mark.parametrize("shape", [(1, 1, 1), (17, 33, 65)])
def test_exact_integer_known_answer(shape):
    """tests/test_gpu.py:127-154 of the reference: A = 1, B_e = e + 1."""
    m, k, n = shape
    for dtype in ("fp16", "bf16", "fp32"):
        outs = oracle.grouped_gemm([np.ones((m, k))] * 3, [np.full((k, n), e + 1.0) for e in range(3)], dtype)
        for got, expected in zip(outs, oracle.exact_integer_outputs(shape, 3)):
            np.testing.assert_array_equal(got, expected)


def test_gate_up_is_two_halves():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((5, 7))
    b = rng.standard_normal((7, 6))
    packed = oracle.gate_up(a, b, "fp32")
    np.testing.assert_array_equal(packed, oracle.matmul(a, b, "fp32"))
    with pytest.raises(ValueError):
        oracle.gate_up(a, rng.standard_normal((7, 5)), "fp32")


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    values = np.concatenate([
        rng.standard_normal(10000).astype(np.float32) * 10,
        # exact ties between two bf16 neighbours (round half to even)
        (np.arange(1, 200, dtype=np.float32) * 2.0**-7 + 2.0**-15).astype(np.float32),
        np.array([0.0, -0.0, 1e-40, 3.4e38, -3.4e38, np.inf, -np.inf], dtype=np.float32),
    ])
    ours = oracle.bf16_round(values)
    theirs = torch.from_numpy(values).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(ours, theirs)
    assert np.isnan(oracle.bf16_round(np.array([np.nan], dtype=np.float32))).all()


def test_rounding_is_idempotent_and_rejects_unknown():
    rng = np.random.default_rng(2)
    x = rng.standard_normal(1000)
    for dtype in oracle.DTYPES:
        once = oracle.round_to_dtype(x, dtype)
        np.testing.assert_array_equal(oracle.round_to_dtype(once, dtype), once)
    with pytest.raises(ValueError):
        oracle.round_to_dtype(x, "fp8")
    with pytest.raises(ValueError):
        oracle.matmul(np.ones((2, 3)), np.ones((4, 2)), "fp32")


def test_relative_frobenius():
    a = np.array([[3.0, 4.0]])
    assert oracle.relative_frobenius(a, a) == 0.0
    assert oracle.relative_frobenius(np.zeros((1, 2)), a) == pytest.approx(1.0)
    assert oracle.relative_frobenius(np.ones((2, 2)), np.zeros((2, 2))) == pytest.approx(2.0)


def test_swiglu_is_silu_of_gate_times_up():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((5, 7))
    b = rng.standard_normal((7, 12))
    got = oracle.swiglu(a, b, "fp32")
    gate, up = a @ b[:, :6], a @ b[:, 6:]
    expected = gate / (1.0 + np.exp(-gate)) * up
    assert oracle.relative_frobenius(got, expected) < 1e-6
    with pytest.raises(ValueError):
        oracle.swiglu(a, b[:, :11], "fp32")


def test_swiglu_known_answer():
    # A = 1, gate = 1, up = 2: every output is silu(K) * 2K.
    k = 4
    a = np.ones((3, k))
    b = np.concatenate((np.ones((k, 5)), 2 * np.ones((k, 5))), axis=1)
    expected = k / (1.0 + np.exp(-k)) * 2 * k
    np.testing.assert_allclose(oracle.swiglu(a, b, "fp32"), np.full((3, 5), expected), rtol=1e-6)
    # silu(0) = 0 whatever up is; large negative gates vanish
    assert np.all(oracle.swiglu(np.zeros((2, 3)), np.ones((3, 4)), "bf16") == 0)
    assert abs(oracle.swiglu(np.full((1, 1), -50.0), np.ones((1, 2)), "fp32")[0, 0]) < 1e-15


def test_fp8_block_scaled_oracle_is_dequantized_product():
    rng = np.random.default_rng(5)
    m, k, n = 3, 200, 130  # partial K and N blocks
    a_q = rng.integers(-8, 8, (m, k)).astype(float)
    b_q = rng.integers(-8, 8, (n, k)).astype(float)
    sa = rng.uniform(0.5, 2.0, (m, 2))
    sb = rng.uniform(0.5, 2.0, (2, 2))
    got = oracle.fp8_block_scaled(a_q, sa, b_q, sb)
    a = a_q * np.concatenate([np.repeat(sa[:, :1], 128, 1), np.repeat(sa[:, 1:], k - 128, 1)], axis=1)
    b = b_q.copy()
    for i in range(2):
        for j in range(2):
            b[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128] *= sb[i, j]
    expected = oracle.round_to_dtype(a @ b.T, "bf16")
    np.testing.assert_array_equal(got, expected)


BF16_CASES = __import__("tests.golden_data", fromlist=["load_bf16_checker_cases"]).load_bf16_checker_cases()


@pytest.mark.parametrize("case", BF16_CASES, ids=[c["name"] for c in BF16_CASES])
def test_oracle_reproduces_reference_checker_in_bf16(case):
    """bf16 pin: the reference's own checker (per-expert torch.matmul,
    benchmark_moe.py:259-266) on DeepSeek-V3 miniature groups, stored by
    tests/golden/make_bf16_golden.py.  torch accumulates in fp32 and the
    oracle in float64, each rounding once to bf16, so they differ by at most
    an output ulp on a few elements: measured relative Frobenius <= 9e-5."""
    from tests.golden_data import bf16_checker_inputs

    a, b = bf16_checker_inputs(case)
    assert len(a) == len(case["c"]) == case["experts"]
    for e in range(case["experts"]):
        a64 = a[e].float().numpy().astype(np.float64)
        b64 = b[e].float().numpy().astype(np.float64)
        if case["projection"] == "W1":
            expected = oracle.gate_up(a64, b64, "bf16")
        else:
            expected = oracle.matmul(a64, b64, "bf16")
        got = case["c"][e].astype(np.float64)
        assert got.shape == (case["m"], case["n"])
        assert oracle.relative_frobenius(got, expected) <= 5e-4
        # Elementwise: one bf16 ulp of the larger magnitude apart at most, plus
        # torch's fp32 accumulation error on results that nearly cancel
        # (measured <= 3.6e-7 absolute with |C| ~ 1 and K <= 7168).
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(expected), np.abs(got)) + 1e-300)) - 7)
        assert np.all(np.abs(got - expected) <= ulp * 1.0001 + 1e-6)
