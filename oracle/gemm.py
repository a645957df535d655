"""Float64 restatement of the reference's per-expert GEMM -- test infrastructure only.

The reference checks every grouped launch against per-expert ``torch.matmul``
on the same inputs (benchmark_moe.py:259-266): W2 / plain groups are
``A_e @ B_e``; packed W13 is ``cat(A_e @ B_e[:, :F], A_e @ B_e[:, F:])``.  Its
kernels accumulate in fp32 and cast on store (kernels/grouped_gemm.py:377,
392-396; kernels/matmul.py:256-273).  Here the products are summed in float64
(tighter than any device accumulation) and rounded once to the output type.

numpy has no bfloat16: bf16 data travels as float32 arrays whose values are
bf16-representable, and ``round_to_dtype`` rounds to nearest-even on the bit
pattern.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np

DTYPES = ("fp16", "bf16", "fp32")


def bf16_round(values: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16, returned as float32 (NaN stays NaN)."""
    x = np.ascontiguousarray(values, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = np.nan
    return out


def round_to_dtype(values: np.ndarray, dtype: str) -> np.ndarray:
    """Round float64 results once to the output type; returned as float64."""
    if dtype == "fp32":
        return values.astype(np.float32).astype(np.float64)
    if dtype == "fp16":
        return values.astype(np.float16).astype(np.float64)
    if dtype == "bf16":
        return bf16_round(values.astype(np.float32)).astype(np.float64)
    raise ValueError(f"unknown dtype {dtype}")


def quantize_input(values: np.ndarray, dtype: str) -> np.ndarray:
    """Input values as the device stores them (float64 view of the rounded data)."""
    return round_to_dtype(np.asarray(values, dtype=np.float64), dtype)


def matmul(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """C = A @ B, float64 sums, one rounding to `dtype` (kernels/matmul.py:256-273)."""
    a64 = np.asarray(a, dtype=np.float64)
    b64 = np.asarray(b, dtype=np.float64)
    if a64.ndim != 2 or b64.ndim != 2 or a64.shape[1] != b64.shape[0]:
        raise ValueError(f"shape mismatch: A={a64.shape}, B={b64.shape}")
    return round_to_dtype(a64 @ b64, dtype)


def grouped_gemm(a_list: Sequence[np.ndarray], b_list: Sequence[np.ndarray], dtype: str) -> list[np.ndarray]:
    """Per-expert C_e = A_e @ B_e (benchmark_moe.py:265-266)."""
    if len(a_list) != len(b_list) or not a_list:
        raise ValueError("grouped GEMM requires equally many A and B matrices")
    return [matmul(a, b, dtype) for a, b in zip(a_list, b_list)]


def gate_up(a: np.ndarray, packed_b: np.ndarray, dtype: str) -> np.ndarray:
    """Packed W13 output [A @ gate | A @ up] (benchmark_moe.py:260-264)."""
    if packed_b.shape[1] % 2:
        raise ValueError("packed gate+up weight needs an even output dimension")
    half = packed_b.shape[1] // 2
    return np.concatenate((matmul(a, packed_b[:, :half], dtype), matmul(a, packed_b[:, half:], dtype)), axis=1)


def swiglu(a: np.ndarray, packed_b: np.ndarray, dtype: str) -> np.ndarray:
    """SiLU(A @ gate) * (A @ up) from the packed W13 weight, float64 throughout and
    one rounding to `dtype`.  The reference applies this activation after its
    packed Gate+Up GEMM, outside the timed region (README.md:55-57,
    kernels/grouped_gemm.py:585); the fused epilogue computes it in fp32 from the
    fp32 accumulators."""
    if packed_b.shape[1] % 2:
        raise ValueError("packed gate+up weight needs an even output dimension")
    a64 = np.asarray(a, dtype=np.float64)
    b64 = np.asarray(packed_b, dtype=np.float64)
    half = b64.shape[1] // 2
    gate = a64 @ b64[:, :half]
    up = a64 @ b64[:, half:]
    return round_to_dtype(gate / (1.0 + np.exp(-gate)) * up, dtype)


def fp8_block_scaled(a_q: np.ndarray, sa: np.ndarray, b_q: np.ndarray, sb: np.ndarray, block: int = 128) -> np.ndarray:
    """FP8 block-scaled product, bf16 output: dequantize A (per row and
    `block`-deep K block) and B [N, K] (per block x block tile), float64
    C = A B^T, one rounding.  The quantization is DeepSeek-V3's
    (model_configs/deepseek-v3.json:37-44), which the reference does not
    emulate (README.md:298); a_q / b_q hold the e4m3 values as floats."""
    a_q = np.asarray(a_q, np.float64)
    b_q = np.asarray(b_q, np.float64)
    m, k = a_q.shape
    n = b_q.shape[0]
    sa_full = np.repeat(np.asarray(sa, np.float64), block, axis=1)[:, :k]
    sb_full = np.repeat(np.repeat(np.asarray(sb, np.float64), block, axis=0)[:n], block, axis=1)[:, :k]
    return round_to_dtype((a_q * sa_full) @ (b_q * sb_full).T, "bf16")


def exact_integer_outputs(shape: tuple[int, int, int], problems: int) -> list[np.ndarray]:
    """Known answer of tests/test_gpu.py:127-154: A = 1, B_e = e + 1 gives C_e = K * (e + 1)."""
    m, k, n = shape
    return [np.full((m, n), float(k * (e + 1))) for e in range(problems)]


def relative_frobenius(actual: np.ndarray, expected: np.ndarray) -> float:
    """||actual - expected||_F / ||expected||_F (0 when both are zero)."""
    diff = np.linalg.norm(np.asarray(actual, np.float64) - np.asarray(expected, np.float64))
    scale = np.linalg.norm(np.asarray(expected, np.float64))
    if scale == 0.0:
        return float(diff)
    return float(diff / scale)
