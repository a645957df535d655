"""GPU parity on the BASELINE.json configurations as stated, through the C ABI.

* bf16 against the reference's own checker: per-expert torch.matmul on the
  same bf16 tensors (benchmark_moe.py:259-266 of the reference), stored by
  tests/golden/make_bf16_golden.py for DeepSeek-V3 miniature W13/W2 EP/TP
  groups at M_e in {16, 17, 129, 256}; every native tile runs them.
* configs[0] exactly: fp32 "ieee", E = 8, W13 8 x [64, 1024] @ [1024, 1024]
  and W2 8 x [64, 512] @ [512, 1024], A ~ N(0, 1), B ~ N(0, 1/sqrt(K)),
  seed 0; against float64 and the per-expert host torch.mm (<= 1e-5).
* configs[1] and [2] at full rank size (32 or 256 experts, every expert):
  Freivalds checks with random vectors v, u in float64, C v = A (B v) per
  row and u^T C = (u^T A) B per column.  Unlike 1^T C = (1^T A) B they see
  a row or column written to the wrong place.
* configs[4]'s masked single-GEMM sweep over every {127, 1000, 4095, 8191}^3
  shape in fp32, with TF32 inputs and with full fp32 products ("ieee", the
  3xTF32 split on the tensor cores): sampled rows against the float64 oracle
  and Freivalds checks of the whole output.

Tolerances: relative Frobenius error bf16 <= 1e-2 (the target's bound) and
against the stored checker outputs also <= 1e-2; fp32 "ieee" <= 1e-5; fp32
"tf32" <= 5e-3; Freivalds relative error <= 1e-2 (bf16) / 5e-3 (tf32) /
1e-5 (fp32 "ieee").
"""

from __future__ import annotations

import itertools
import math

import numpy as np
import pytest

from tests.conftest import cuda_ready

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")]

REL_FRO_BF16 = 1e-2
REL_FRO_FP32_IEEE = 1e-5
REL_FRO_TF32 = 5e-3


def _torch():
    import torch

    return torch


def _rel_fro(got: np.ndarray, expected: np.ndarray) -> float:
    return float(np.linalg.norm(got - expected) / max(np.linalg.norm(expected), 1e-300))


def _freivalds(a, b, c, gen) -> tuple[float, float]:
    """Relative errors of C v against A (B v) and of u^T C against (u^T A) B,
    random Gaussian v and u, all in float64 on the device."""
    torch = _torch()
    m, n = c.shape
    v = torch.randn((n, 1), device=c.device, dtype=torch.float64, generator=gen)
    u = torch.randn((1, m), device=c.device, dtype=torch.float64, generator=gen)
    a64, b64, c64 = a.double(), b.double(), c.double()
    row_expected, row_got = a64 @ (b64 @ v), c64 @ v
    col_expected, col_got = (u @ a64) @ b64, u @ c64
    row = float((row_got - row_expected).norm() / row_expected.norm())
    col = float((col_got - col_expected).norm() / col_expected.norm())
    return row, col


# ------------------------------------------------ bf16 vs the reference's checker
NATIVE_TILES = {
    "policy": None, "swap16x256": (16, 256), "swap32x256": (32, 256), "swap64x256": (64, 256),
    "tok128x256": (128, 256), "pair256x256": (256, 128), "pair256x512": (256, 256),
}


@pytest.mark.parametrize("tile", list(NATIVE_TILES))
def test_bf16_matches_reference_checker_outputs(tile):
    """Every miniature group, launched with one native tile (or the autotuned
    policy), against the stored bf16 outputs of the reference's torch.matmul
    checker on the same inputs."""
    torch = _torch()
    from kernels import KernelConfig, check_device_errors, launch_grouped, workspace_from_tensors
    from tests.golden_data import bf16_checker_inputs, load_bf16_checker_cases

    worst = 0.0
    for case in load_bf16_checker_cases():
        a_host, b_host = bf16_checker_inputs(case)
        a = [t.cuda() for t in a_host]
        b = [t.cuda() for t in b_host]
        c = [torch.full((case["m"], case["n"]), float("nan"), device="cuda", dtype=torch.bfloat16) for _ in a]
        ws = workspace_from_tensors(a, b, c)
        ws.operation = "gate_up" if case["projection"] == "W1" else "down"
        if NATIVE_TILES[tile] is None:
            launch_grouped(ws)
        else:
            bm, bn = NATIVE_TILES[tile]
            launch_grouped(ws, config=KernelConfig(bm, bn, 64, 8, 4, 4), autotune=False)
        torch.cuda.synchronize()
        check_device_errors()
        assert ws.launch_info["path"].startswith("tcgen05_tma"), ws.launch_info
        for got, expected in zip(c, case["c"]):
            got_np = got.float().cpu().numpy().astype(np.float64)
            assert np.isfinite(got_np).all(), f"{case['name']}: unwritten outputs"
            err = _rel_fro(got_np, expected.astype(np.float64))
            assert err <= REL_FRO_BF16, f"{case['name']} ({tile}): {err:.3e}"
            worst = max(worst, err)
    assert worst < 2e-3, f"worst relative Frobenius {worst:.3e}: larger than one bf16 rounding apart"


# ------------------------------------------------ configs[0] exactly as stated
def _configs0_inputs(k: int, n: int):
    torch = _torch()
    gen = torch.Generator().manual_seed(0)
    a = [torch.randn((64, k), generator=gen, dtype=torch.float32) for _ in range(8)]
    b = [torch.randn((k, n), generator=gen, dtype=torch.float32) / math.sqrt(k) for _ in range(8)]
    return a, b


@pytest.mark.parametrize("projection,k,n", [("W13", 1024, 1024), ("W2", 512, 1024)])
def test_configs0_cpu_plumbing_fp32_ieee(projection, k, n):
    """E = 8, topk = 2, P = 1 (64 rows per expert), fp32
    with input_precision="ieee", seed 0; the reference there is per-expert
    torch.mm on the host."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped, workspace_from_tensors
    from oracle import gemm as oracle

    a_host, b_host = _configs0_inputs(k, n)
    a = [t.cuda() for t in a_host]
    b = [t.cuda() for t in b_host]
    c = [torch.full((64, n), float("nan"), device="cuda", dtype=torch.float32) for _ in a]
    ws = workspace_from_tensors(a, b, c)
    ws.operation = "gate_up" if projection == "W13" else "down"
    launch_grouped(ws, input_precision="ieee")
    torch.cuda.synchronize()
    check_device_errors()
    for e in range(8):
        got = c[e].cpu().double().numpy()
        a64, b64 = a_host[e].double().numpy(), b_host[e].double().numpy()
        expected = oracle.gate_up(a64, b64, "fp32") if projection == "W13" else oracle.matmul(a64, b64, "fp32")
        assert _rel_fro(got, expected) <= REL_FRO_FP32_IEEE
        host_mm = torch.mm(a_host[e], b_host[e]).double().numpy()
        assert _rel_fro(got, host_mm) <= REL_FRO_FP32_IEEE


# ------------------------------------------------ configs[1]/[2] at full size
FULL_RANKS = {"W13_EP": (32, 7168, 4096), "W13_TP": (256, 7168, 512), "W2_EP": (32, 2048, 7168),
              "W2_TP": (256, 256, 7168)}


@pytest.mark.parametrize("m_e", [16, 256, 1024])
@pytest.mark.parametrize("rank_kind", list(FULL_RANKS))
def test_full_size_rank_freivalds(rank_kind, m_e):
    """A whole DeepSeek-V3 P = 8 rank launch (every expert), autotuned, with
    row and column Freivalds checks per expert and a float64 oracle check of
    three rows of the first and last experts."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped, workspace_from_tensors
    from oracle import gemm as oracle

    experts, k, n = FULL_RANKS[rank_kind]
    gen = torch.Generator(device="cuda").manual_seed(m_e * 31 + k)
    a_all = torch.randn((experts, m_e, k), device="cuda", generator=gen).to(torch.bfloat16)
    b_all = (torch.randn((experts, k, n), device="cuda", generator=gen) / math.sqrt(k)).to(torch.bfloat16)
    c_all = torch.full((experts, m_e, n), float("nan"), device="cuda", dtype=torch.bfloat16)
    ws = workspace_from_tensors(list(a_all), list(b_all), list(c_all))
    ws.operation = "gate_up" if rank_kind.startswith("W13") else "down"
    launch_grouped(ws)
    torch.cuda.synchronize()
    check_device_errors()
    assert ws.launch_info["path"].startswith("tcgen05_tma"), ws.launch_info
    assert not torch.isnan(c_all).any(), "unwritten outputs"
    vgen = torch.Generator(device="cuda").manual_seed(5)
    worst = 0.0
    for e in range(experts):
        row, col = _freivalds(a_all[e], b_all[e], c_all[e], vgen)
        worst = max(worst, row, col)
        assert row <= REL_FRO_BF16 and col <= REL_FRO_BF16, f"expert {e}: row {row:.3e}, column {col:.3e}"
    for e in (0, experts - 1):
        rows = torch.tensor(sorted({0, m_e // 2, m_e - 1}), device="cuda")
        got = c_all[e].index_select(0, rows).double().cpu().numpy()
        expected = oracle.matmul(a_all[e].index_select(0, rows).double().cpu().numpy(),
                                 b_all[e].double().cpu().numpy(), "bf16")
        assert _rel_fro(got, expected) <= REL_FRO_BF16


# ------------------------------------------------ configs[4] masked sweep
SWEEP = (127, 1000, 4095, 8191)


@pytest.mark.parametrize("precision", ["tf32", "ieee"])
@pytest.mark.parametrize("m,k,n", list(itertools.product(SWEEP, SWEEP, SWEEP)),
                         ids=lambda v: str(v))
def test_masked_sweep_fp32(m, k, n, precision):
    """One shape of the Qwen3 masked single-GEMM sweep (fp32, non-tile-multiple
    M, N, K) with TF32 inputs, and with full fp32 products ("ieee": the
    3xTF32 split on the tensor cores for large shapes): launch_matmul,
    Freivalds checks of the whole output and the float64 oracle on sampled
    rows."""
    torch = _torch()
    from kernels import check_device_errors, launch_matmul
    from kernels.matmul import REPACK_MIN_FLOPS, last_launch_info
    from oracle import gemm as oracle

    tol = REL_FRO_TF32 if precision == "tf32" else REL_FRO_FP32_IEEE
    gen = torch.Generator(device="cuda").manual_seed(m * 7 + k * 3 + n)
    a = torch.randn((m, k), device="cuda", generator=gen)
    b = torch.randn((k, n), device="cuda", generator=gen) / math.sqrt(k)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    launch_matmul(a, b, c, input_precision=precision)
    torch.cuda.synchronize()
    check_device_errors()
    info = last_launch_info()
    if 2 * m * n * k >= REPACK_MIN_FLOPS:
        assert info["path"].startswith("tcgen05_tma"), info
        assert info["split_3xtf32"] == (precision == "ieee"), info
    assert not torch.isnan(c).any(), "unwritten outputs"
    row, col = _freivalds(a, b, c, torch.Generator(device="cuda").manual_seed(9))
    assert row <= tol and col <= tol, (row, col)
    rows = torch.tensor(sorted({0, 1, m // 3, m // 2, m - 2, m - 1}), device="cuda")
    got = c.index_select(0, rows).double().cpu().numpy()
    expected = oracle.matmul(a.index_select(0, rows).double().cpu().numpy(), b.double().cpu().numpy(), "fp32")
    assert _rel_fro(got, expected) <= tol


def test_split_tf32x3_layout_and_rounding():
    """matrix_split_tf32x3: hi has its low 13 mantissa bits clear, hi + lo
    recovers x to within 2^-21 of |x|, and the halves land where the 3K-deep
    GEMM expects them (A: [hi | lo | hi] along columns, B: [hi; hi; lo] along
    rows), from a strided source."""
    torch = _torch()
    from kernels.matmul import split_operands_3xtf32

    gen = torch.Generator(device="cuda").manual_seed(3)
    base = torch.randn((37, 2 * 19), device="cuda", generator=gen) * 1e3
    a = base[:, ::2]  # [37, 19], column stride 2
    b = torch.randn((19, 23), device="cuda", generator=gen)
    a3, b3 = split_operands_3xtf32(a, b, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert a3.shape == (37, 57) and b3.shape == (57, 23)
    assert (a3.stride(0) * 4) % 16 == 0 and (b3.stride(0) * 4) % 16 == 0
    hi_a, lo_a = a3[:, :19], a3[:, 19:38]
    assert torch.equal(a3[:, 38:], hi_a)
    assert torch.equal(b3[:19], b3[19:38])
    for hi, lo, x in ((hi_a, lo_a, a), (b3[:19], b3[38:], b)):
        assert (hi.contiguous().view(torch.int32) & 0x1FFF).eq(0).all()
        assert (lo.contiguous().view(torch.int32) & 0x1FFF).eq(0).all()
        err = ((hi.double() + lo.double()) - x.double()).abs()
        assert (err <= x.double().abs() * 2.0 ** -21).all()
        assert ((hi.double() - x.double()).abs() <= x.double().abs() * 2.0 ** -11).all()
