"""FP8 block-scaled grouped GEMM -- the DeepSeek-V3 expert quantization.

DeepSeek-V3 declares e4m3 weights with 128 x 128 blocks and dynamic
activation scales (``quantization_config`` of model_configs/deepseek-v3.json:
``fmt: e4m3``, ``weight_block_size: [128, 128]``, ``activation_scheme:
dynamic``); the reference runs every expert in fp16 / bf16 / fp32 and does
not emulate it (README.md:298).  Here one native launch computes, per expert,

    C_e[M, N] (bf16) = sum_kb (A_e[:, kb] @ B_e[:, kb]^T) * SA_e[:, kb] * SB_e[n // 128, kb]

with A_e e4m3 ``[M, K]`` (tokens), B_e e4m3 ``[N, K]`` (the weight as
checkpoints store it: output x input features), SA_e fp32 ``[M, ceil(K/128)]``
(per token and 128-deep K block), SB_e fp32 ``[ceil(N/128), ceil(K/128)]``
(per 128 x 128 weight block), fp32 accumulation (``grouped_gemm_fp8_launch``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

try:
    import torch
except ImportError:  # pragma: no cover - the CPU tests import the host helpers only
    torch = None

from . import _native
from .matmul import KernelConfig

FP8_BLOCK = 128
E4M3_MAX = 448.0

# Native tiles of the FP8 path, by the tokens per expert they fit.
FP8_TILE_SWAP_16 = KernelConfig(16, 256, 128, 4, 8, 4)
FP8_TILE_SWAP_32 = KernelConfig(32, 256, 128, 4, 8, 4)
FP8_TILE_SWAP_64 = KernelConfig(64, 256, 128, 8, 8, 4)
FP8_TILE_ROWS_128 = KernelConfig(128, 128, 128, 8, 8, 4)
FP8_TILE_PAIR_256 = KernelConfig(256, 128, 128, 8, 8, 4)  # CTA pair: 256 tokens x 128 weight rows
FP8_TILE_PAIR_256x256 = KernelConfig(256, 256, 128, 8, 8, 4)  # CTA pair: 256 tokens x 256 weight rows


def fp8_tile_for(max_m: int) -> KernelConfig:
    """Swap-AB tiles (weight rows as MMA M, exact-fit token count) while the
    launch streams weights from HBM, 128 x 128 token tiles up to 128 tokens,
    and above that the CTA-pair 256 x 256 tile, whose M = 256, N = 256 MMAs
    do four times the work of a 128 x 128 tile's per instruction (from 129
    tokens the 128-row tile needs two row blocks anyway: 1.17-1.27x at
    M = 160-224 on DeepSeek-V3 W13 / W2 rank shapes)."""
    if max_m <= 16:
        return FP8_TILE_SWAP_16
    if max_m <= 32:
        return FP8_TILE_SWAP_32
    if max_m <= 64:
        return FP8_TILE_SWAP_64
    if max_m <= 128:
        return FP8_TILE_ROWS_128
    return FP8_TILE_PAIR_256x256


def _blocks(n: int) -> int:
    return (n + FP8_BLOCK - 1) // FP8_BLOCK


def quantize_activations(x):
    """Per token and 128-deep K block: scale = amax / 448, q = x / scale in
    e4m3.  Returns (q [M, K] float8_e4m3fn, scales [M, ceil(K/128)] fp32)."""
    m, k = x.shape
    kb = _blocks(k)
    padded = torch.zeros((m, kb * FP8_BLOCK), dtype=torch.float32, device=x.device)
    padded[:, :k] = x.float()
    blocks = padded.view(m, kb, FP8_BLOCK)
    scale = blocks.abs().amax(dim=2).clamp_min(1e-12) / E4M3_MAX
    q = (blocks / scale[:, :, None]).view(m, kb * FP8_BLOCK)[:, :k]
    return q.to(torch.float8_e4m3fn).contiguous(), scale.contiguous()


def quantize_weight(w):
    """Per 128 x 128 block of a [N, K] weight: scale = amax / 448.  Returns
    (q [N, K] float8_e4m3fn, scales [ceil(N/128), ceil(K/128)] fp32)."""
    n, k = w.shape
    nb, kb = _blocks(n), _blocks(k)
    padded = torch.zeros((nb * FP8_BLOCK, kb * FP8_BLOCK), dtype=torch.float32, device=w.device)
    padded[:n, :k] = w.float()
    blocks = padded.view(nb, FP8_BLOCK, kb, FP8_BLOCK)
    scale = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12) / E4M3_MAX
    q = (blocks / scale[:, None, :, None]).view(nb * FP8_BLOCK, kb * FP8_BLOCK)[:n, :k]
    return q.to(torch.float8_e4m3fn).contiguous(), scale.contiguous()


def dequantize_activations(q, scale):
    m, k = q.shape
    expand = scale.repeat_interleave(FP8_BLOCK, dim=1)[:, :k]
    return q.float() * expand


def dequantize_weight(q, scale):
    n, k = q.shape
    expand = scale.repeat_interleave(FP8_BLOCK, dim=0)[:n].repeat_interleave(FP8_BLOCK, dim=1)[:, :k]
    return q.float() * expand


@dataclass
class Fp8GroupedWorkspace:
    """Per-expert FP8 operands, their scales, bf16 outputs and the device
    tables one launch reads (a_ptrs / b_ptrs / c_ptrs / sa_ptrs / sb_ptrs
    int64 [E], dims int32 [E, 3] in the M N K order of the grouped tables)."""

    a: list
    b: list
    sa: list
    sb: list
    c: list
    a_ptrs: object
    b_ptrs: object
    c_ptrs: object
    sa_ptrs: object
    sb_ptrs: object
    dims: object
    shapes: tuple[tuple[int, int, int], ...]  # (M, K, N) per expert
    homogeneous: bool
    scratch: object = None
    config: KernelConfig | None = None
    launch_info: dict | None = field(default=None)
    operation: str = "fp8_block_scaled"

    @property
    def problem_count(self) -> int:
        return len(self.a)

    @property
    def max_m(self) -> int:
        return max(m for m, _, _ in self.shapes)

    def problem_tensors(self):
        return zip(self.a, self.sa, self.b, self.sb, self.c)


def fp8_workspace_from_tensors(a_list, b_list, sa_list, sb_list, c_list) -> Fp8GroupedWorkspace:
    """Tables for caller-owned FP8 expert tensors (see the module docstring
    for the layout).  Raises ValueError on shape / dtype / layout mismatches."""
    if not a_list or not (len(a_list) == len(b_list) == len(sa_list) == len(sb_list) == len(c_list)):
        raise ValueError("FP8 grouped GEMM needs equally many A, B, SA, SB and C tensors (at least one)")
    shapes = []
    for a, b, sa, sb, c in zip(a_list, b_list, sa_list, sb_list, c_list):
        if a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn:
            raise ValueError("A and B must be float8_e4m3fn")
        if sa.dtype != torch.float32 or sb.dtype != torch.float32 or c.dtype != torch.bfloat16:
            raise ValueError("scales must be float32 and C bfloat16")
        if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[1]:
            raise ValueError(f"expected A [M, K] and B [N, K], got {tuple(a.shape)} and {tuple(b.shape)}")
        m, k = a.shape
        n = b.shape[0]
        if tuple(sa.shape) != (m, _blocks(k)) or tuple(sb.shape) != (_blocks(n), _blocks(k)):
            raise ValueError(f"scale shapes {tuple(sa.shape)} / {tuple(sb.shape)} do not match M={m} N={n} K={k}")
        if tuple(c.shape) != (m, n):
            raise ValueError(f"C must be [{m}, {n}]")
        if not all(x.is_contiguous() for x in (a, b, sa, sb, c)):
            raise ValueError("FP8 operands, scales and outputs must be contiguous")
        if len({a.device, b.device, sa.device, sb.device, c.device}) != 1 or not a.is_cuda:
            raise ValueError("all FP8 tensors must be on one CUDA device")
        shapes.append((int(m), int(k), int(n)))
    device = a_list[0].device

    def pointers(items):
        return torch.tensor([item.data_ptr() for item in items], device=device, dtype=torch.int64)

    dims = torch.tensor([[m, n, k] for m, k, n in shapes], device=device, dtype=torch.int32)
    homogeneous = all(shape == shapes[0] for shape in shapes)
    return Fp8GroupedWorkspace(
        list(a_list), list(b_list), list(sa_list), list(sb_list), list(c_list),
        pointers(a_list), pointers(b_list), pointers(c_list), pointers(sa_list), pointers(sb_list), dims,
        tuple(shapes), homogeneous,
    )


def build_fp8_workspace(shapes: Sequence[tuple[int, int, int]], seed: int = 0,
                        weight_std: float | None = None) -> Fp8GroupedWorkspace:
    """Seeded experts quantized from A ~ N(0, 1) and B ~ N(0, 1/sqrt(K))
    (or ``weight_std``): shapes are (M, K, N) with B stored [N, K]."""
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch is required")
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a_list, b_list, sa_list, sb_list, c_list = [], [], [], [], []
    for m, k, n in shapes:
        a = torch.randn((m, k), device="cuda", generator=gen)
        w = torch.randn((n, k), device="cuda", generator=gen) * (weight_std or 1.0 / math.sqrt(k))
        qa, sa = quantize_activations(a)
        qb, sb = quantize_weight(w)
        a_list.append(qa)
        sa_list.append(sa)
        b_list.append(qb)
        sb_list.append(sb)
        c_list.append(torch.empty((m, n), device="cuda", dtype=torch.bfloat16))
    return fp8_workspace_from_tensors(a_list, b_list, sa_list, sb_list, c_list)


def launch_grouped_fp8(workspace: Fp8GroupedWorkspace, config: KernelConfig | None = None) -> None:
    """One native launch (map builder + GEMM kernel) of the FP8 block-scaled
    grouped GEMM; ``config`` defaults to ``fp8_tile_for(max M)``."""
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
    _native.load()
    need = _native.scratch_bytes(workspace.problem_count, 0)
    if workspace.scratch is None or workspace.scratch.numel() < need:
        workspace.scratch = torch.empty(need, dtype=torch.uint8, device=workspace.a[0].device)
    cfg = config or fp8_tile_for(workspace.max_m)
    m, k, n = (workspace.shapes[0] if workspace.homogeneous else
               (workspace.max_m, max(s[1] for s in workspace.shapes), max(s[2] for s in workspace.shapes)))
    device = workspace.a[0].device
    with torch.cuda.device(device):
        info = _native.fp8_launch(
            workspace.a_ptrs.data_ptr(), workspace.b_ptrs.data_ptr(), workspace.c_ptrs.data_ptr(),
            workspace.sa_ptrs.data_ptr(), workspace.sb_ptrs.data_ptr(), workspace.dims.data_ptr(),
            workspace.problem_count, workspace.homogeneous, m, n, k, cfg, workspace.scratch.data_ptr(),
            workspace.scratch.numel(), torch.cuda.current_stream(device).cuda_stream,
        )
    workspace.config = cfg
    workspace.launch_info = info.as_dict()
