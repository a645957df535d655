"""Host-side logic of the kernels package that needs no GPU.

Argument validation mirrors the reference's errors (ValueError for shapes,
devices and dtypes, kernels/matmul.py:318-329; RuntimeError when no CUDA
runtime is present, kernels/grouped_gemm.py:626-627), the TMA alignment
verdict, and the EP/TP shard plans with their reassembly.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from kernels import KernelConfig, launch_grouped, launch_matmul  # noqa: E402
from kernels.grouped_gemm import GroupedWorkspace, _shape_signature, operands_tma_aligned  # noqa: E402
from kernels.matmul import _validate_matrices, dtype_name  # noqa: E402
from moe_parallel import (  # noqa: E402
    assemble_w2_tp,
    assemble_w13_tp,
    ep_owner,
    moe_shapes,
    rank_plan,
    shard_weight,
)

NO_CUDA = not torch.cuda.is_available()


def test_validate_matrices_errors():
    a, b, c = torch.zeros(2, 3), torch.zeros(3, 4), torch.zeros(2, 4)
    with pytest.raises(ValueError, match="matrices"):
        _validate_matrices(a[0], b, c)
    with pytest.raises(ValueError, match="shape mismatch"):
        _validate_matrices(a, torch.zeros(4, 4), c)
    with pytest.raises(ValueError, match="CUDA"):
        _validate_matrices(a, b, c)
    with pytest.raises(ValueError):
        dtype_name(torch.int8)


@pytest.mark.skipif(not NO_CUDA, reason="checks the CPU-only error path")
def test_launches_need_cuda():
    a, b, c = torch.zeros(2, 3), torch.zeros(3, 4), torch.zeros(2, 4)
    with pytest.raises(RuntimeError):
        launch_matmul(a, b, c)
    ws = _cpu_workspace([(2, 8, 8), (2, 8, 8)])
    with pytest.raises(RuntimeError):
        launch_grouped(ws)


def _cpu_workspace(shapes, a=None, b=None):
    a = a or [torch.zeros(m, k, dtype=torch.bfloat16) for m, k, _ in shapes]
    b = b or [torch.zeros(k, n, dtype=torch.bfloat16) for _, k, n in shapes]
    c = [torch.zeros(m, n, dtype=torch.bfloat16) for m, _, n in shapes]
    return GroupedWorkspace(a, b, c, None, None, None, None, None, tuple(shapes), KernelConfig(16, 64, 32, 4, 2, 2),
                            _shape_signature(shapes), 0, 148, 0, True)


def test_tma_alignment_verdict():
    ok = _cpu_workspace([(16, 64, 128)] * 2)
    assert operands_tma_aligned(ok)
    odd_pitch = _cpu_workspace([(17, 13, 31)])  # 26-byte rows
    assert not operands_tma_aligned(odd_pitch)
    base = torch.zeros(16, 129, dtype=torch.bfloat16)
    shifted = _cpu_workspace([(16, 64, 128)], a=[base[:, 1:65]])  # base + 2 bytes
    assert not operands_tma_aligned(shifted)
    strided = _cpu_workspace([(16, 64, 64)], b=[torch.zeros(64, 128, dtype=torch.bfloat16)[:, ::2]])
    assert not operands_tma_aligned(strided)


def test_shape_signature_is_stable_and_discriminates():
    assert _shape_signature([(1, 2, 3)]) == _shape_signature([(1, 2, 3)])
    assert _shape_signature([(1, 2, 3)]) != _shape_signature([(1, 3, 2)])
    assert 0 <= _shape_signature([(7, 7, 7)] * 100) < 2**31


def test_rank_plans_cover_the_layer():
    e, f, h, p = 8, 12, 5, 4
    ep_experts = [x for r in range(p) for x in rank_plan("W1", "EP", r, p, e, f, h).experts]
    assert ep_experts == list(range(e))
    assert all(ep_owner(x, p, e) == x // 2 for x in range(e))
    tp_slices = [rank_plan("W2", "TP", r, p, e, f, h).ffn_slice for r in range(p)]
    assert tp_slices == [(0, 3), (3, 6), (6, 9), (9, 12)]
    with pytest.raises(ValueError):
        rank_plan("W1", "EP", 4, p, e, f, h)


@pytest.mark.parametrize("p", [1, 2, 4])
def test_tp_shards_reassemble_the_global_product(p):
    """[gate_r | up_r] slices and W2 partial sums rebuild the full-layer product
    exactly (integer-valued inputs keep float64 sums exact)."""
    rng = np.random.default_rng(p)
    e, f, h, m = 4, 8, 6, 5
    a = rng.integers(-3, 4, size=(m, h)).astype(np.float64)
    w13 = rng.integers(-3, 4, size=(h, 2 * f)).astype(np.float64)
    act = rng.integers(-3, 4, size=(m, f)).astype(np.float64)
    w2 = rng.integers(-3, 4, size=(f, h)).astype(np.float64)
    w13_outs, w2_parts = [], []
    for r in range(p):
        plan13 = rank_plan("W1", "TP", r, p, e, f, h)
        plan2 = rank_plan("W2", "TP", r, p, e, f, h)
        local13 = shard_weight(w13, plan13)
        local2 = shard_weight(w2, plan2)
        assert local13.shape == (h, 2 * f // p) and local2.shape == (f // p, h)
        assert [(m,) + local13.shape] == [moe_shapes("W1", "TP", m, h, f, e, p)[0]]
        w13_outs.append(a @ local13)
        start, stop = plan2.ffn_slice
        w2_parts.append(act[:, start:stop] @ local2)
    np.testing.assert_array_equal(assemble_w13_tp(w13_outs, p), a @ w13)
    np.testing.assert_array_equal(assemble_w2_tp(w2_parts), act @ w2)
    ep = rank_plan("W1", "EP", 0, p, e, f, h)
    assert shard_weight(w13, ep) is w13


def test_torch_tensors_shard_too():
    w = torch.arange(24.0).reshape(3, 8)
    plan = rank_plan("W1", "TP", 1, 2, 2, 4, 3)
    local = shard_weight(w, plan)
    assert torch.equal(local, torch.cat((w[:, 2:4], w[:, 6:8]), 1))
    assert local.is_contiguous()


def test_native_tile_policy():
    """The fixed tile policy of autotune=True launches: exact-fit swap-AB tiles
    up to 64 tokens, 128-token tiles at 128, CTA-pair tiles beyond (256 x 512
    from M = 512, and at M = 256 when K >= 4096); short K (<= 1024) takes the
    128-token tile from M = 32 to 128 and the 256 x 512 pair above."""
    from kernels import native_candidates
    from kernels import matmul as mm

    assert native_candidates(1) == (mm.TILE_SWAP_16x256,)
    assert native_candidates(16, 7168) == (mm.TILE_SWAP_16x256,)
    assert native_candidates(32) == (mm.TILE_SWAP_32x256,)
    assert native_candidates(64, 7168) == (mm.TILE_SWAP_64x256,)
    assert native_candidates(128, 7168) == (mm.TILE_TOKENS_128x256,)
    assert native_candidates(256, 7168) == (mm.TILE_PAIR_256x512,)
    # Without a splittable tail (ragged groups, SwiGLU, aggregate layout) M = 256 keeps 256 x 256.
    assert native_candidates(256, 7168, split_tail=False) == (mm.TILE_PAIR_256x256,)
    assert native_candidates(256) == (mm.TILE_PAIR_256x256,)
    assert native_candidates(256, 2048) == (mm.TILE_PAIR_256x256,)
    assert native_candidates(1024, 2048) == (mm.TILE_PAIR_256x512,)
    assert native_candidates(256, 256) == (mm.TILE_PAIR_256x512,)
    assert native_candidates(128, 256) == (mm.TILE_TOKENS_128x256,)
    assert native_candidates(16, 256) == (mm.TILE_SWAP_16x256,)
    assert native_candidates(32, 256) == (mm.TILE_TOKENS_128x256,)
    assert native_candidates(64, 256) == (mm.TILE_TOKENS_128x256,)
    assert native_candidates(64, 2048) == (mm.TILE_SWAP_64x256,)
    assert native_candidates(1024, 256) == (mm.TILE_PAIR_256x512,)
    assert native_candidates(512, 7168) == (mm.TILE_PAIR_256x512,)
    assert native_candidates(1024) == (mm.TILE_PAIR_256x512,)


def test_fp8_quantization_round_trip_and_tiles():
    """Block quantization helpers (CPU tensors): scales per token x 128-deep K
    block and per 128 x 128 weight block; dequantized values within e4m3
    precision; the tile policy by tokens per expert."""
    torch = pytest.importorskip("torch")
    from kernels import fp8

    gen = torch.Generator().manual_seed(0)
    x = torch.randn((5, 300), generator=gen)
    q, s = fp8.quantize_activations(x)
    assert q.dtype == torch.float8_e4m3fn and tuple(s.shape) == (5, 3)
    back = fp8.dequantize_activations(q, s)
    assert float((back - x).norm() / x.norm()) < 0.05
    w = torch.randn((200, 300), generator=gen)
    qw, sw = fp8.quantize_weight(w)
    assert tuple(sw.shape) == (2, 3)
    assert float((fp8.dequantize_weight(qw, sw) - w).norm() / w.norm()) < 0.05
    assert fp8.fp8_tile_for(16).block_m == 16 and fp8.fp8_tile_for(40).block_m == 64
    assert fp8.fp8_tile_for(128).block_m == 128 and fp8.fp8_tile_for(129).block_m == 256
    assert (fp8.fp8_tile_for(256).block_m, fp8.fp8_tile_for(1024).block_n) == (256, 256)


def test_split_k_slices_for_skinny_fp32_gemms():
    """fp32 tensor-core GEMMs split K only when the output leaves most SMs idle
    and K is long; at most 32 slices of at least 1024 (256 for outputs of up
    to 8 tiles), and two only from K = 6144."""
    from kernels import matmul as mm

    assert mm.splitk_splits(127, 8191, 8191, 148) == 2   # m, n, k: 64 output tiles
    assert mm.splitk_splits(127, 127, 8191, 148) == 31   # one tile: 8191 // 256 slices
    assert mm.splitk_splits(127, 127, 3000, 148) == 11   # the 3xTF32 depth of K = 1000, one tile
    assert mm.splitk_splits(127, 4095, 4096, 148) == 4   # 32 tiles
    assert mm.splitk_splits(127, 8191, 1000, 148) == 1   # K below SPLITK_MIN_K
    assert mm.splitk_splits(1000, 1000, 8191, 148) == 2  # 64 tiles
    assert mm.splitk_splits(1000, 1000, 4095, 148) == 1  # two slices only from K = 6144
    assert mm.splitk_splits(127, 8191, 3000, 148) == 1   # the 3xTF32 depth of K = 1000
    assert mm.splitk_splits(8191, 8191, 8191, 148) == 1  # the output fills the GPU
    assert mm.splitk_splits(127, 4095, 3000, 148) == 1   # 32 tiles: 1024-deep slices, so only two
    assert mm.splitk_splits(127, 1000, 4095, 148) == 15  # 8 tiles: 256-deep slices
