"""Persistent grouped GEMM over distinct expert A/B/C pointers, on B200.

Drop-in for the reference's kernels/grouped_gemm.py: same names, arguments,
workspace fields, scheduler strings and errors, so benchmark_moe.py and
compare_grouped_gemm.py drive these kernels unchanged.

* ``GroupedWorkspace``              kernels/grouped_gemm.py:67-111
* ``grouped_candidate_configs``     kernels/grouped_gemm.py:114-224
* ``build_grouped_workspace``       kernels/grouped_gemm.py:507-572
* ``build_fused_gate_up_workspace`` kernels/grouped_gemm.py:575-594
* ``launch_grouped``                kernels/grouped_gemm.py:618-760

One ``launch_grouped`` call is one native launch that walks the device-side
pointer / dims / stride tables.  W13 gate+up is the same launch with a packed
``[gate | up]`` output dimension N = 2 * F_local (vLLM W13 order).
"""

from __future__ import annotations

import math
import zlib
from collections.abc import Sequence
from dataclasses import dataclass, field

try:
    import torch
except ImportError:
    torch = None

from . import _native
from .matmul import (
    _MATMUL_CONFIG_POOL,
    KernelConfig,
    autotune_over,
    diverse_configs,
    dtype_name,
    last_matmul_config,
    launch_matmul,
    matmul_candidate_configs,
    native_candidates,
    select_config,
)

# Skinny-M tiles added to the single-GEMM pool for grouped MoE problems, in the
# reference's order (kernels/grouped_gemm.py:41-63); the merged, de-duplicated
# pool is the reference's _GROUPED_BASE_CONFIG_POOL (:64).
_GROUPED_EXTRA_ROWS = (
    (16, 64, 64, 4, 4, 3), (16, 128, 128, 4, 4, 4), (16, 256, 32, 4, 8, 3), (16, 256, 64, 4, 8, 4),
    (32, 64, 128, 4, 4, 4), (32, 128, 128, 4, 8, 4), (32, 256, 64, 4, 8, 4), (64, 32, 64, 4, 4, 3),
    (64, 256, 128, 4, 8, 4), (128, 128, 128, 8, 8, 4), (16, 64, 128, 1, 4, 2), (16, 128, 64, 1, 4, 5),
    (32, 128, 128, 1, 4, 2), (32, 256, 64, 4, 8, 5), (64, 128, 128, 1, 4, 3), (128, 128, 128, 4, 8, 3),
    (64, 64, 32, 1, 4, 3), (128, 128, 32, 1, 4, 3), (128, 128, 64, 1, 4, 3), (64, 128, 64, 1, 4, 3),
)
_GROUPED_EXTRA_CONFIG_POOL: tuple[KernelConfig, ...] = tuple(KernelConfig(*row) for row in _GROUPED_EXTRA_ROWS)
_GROUPED_BASE_CONFIG_POOL = tuple(dict.fromkeys((*_MATMUL_CONFIG_POOL, *_GROUPED_EXTRA_CONFIG_POOL)))

SCHEDULER_SINGLE = "single_problem_matmul"
SCHEDULER_HOMOGENEOUS = "homogeneous_persistent"
SCHEDULER_GENERIC = "generic_persistent"


@dataclass
class GroupedWorkspace:
    """Per-expert tensors plus the device tables one launch reads.

    Fields a_ptrs / b_ptrs / c_ptrs (int64 [E]), dims (int32 [E, 3], M N K
    order), strides (int64 [E, 6]: am ak bk bn cm cn) are the reference's
    (kernels/grouped_gemm.py:67-111).  ``scratch`` holds the per-problem
    tensor maps of the TMA path; ``launch_info`` records the native kernel of
    the most recent launch.  ``operation == "swiglu"`` marks a workspace whose
    C_e is [M_e, N/2] and whose launches apply the fused SwiGLU epilogue.
    """

    a: list
    b: list
    c: list
    a_ptrs: object
    b_ptrs: object
    c_ptrs: object
    dims: object
    strides: object
    shapes: tuple[tuple[int, int, int], ...]
    config: KernelConfig
    shape_signature: int
    device_signature: int
    sm_count: int
    storage_bytes: int
    homogeneous: bool
    operation: str = "gemm"
    scheduler: str = "not_launched"
    scratch: object = None
    launch_info: dict | None = field(default=None)
    # Host-side TMA verdict for the A / B lists, computed once (see
    # operands_tma_aligned).  The device re-checks every table entry, so an
    # entry swapped later for a misaligned one is skipped, never dereferenced.
    tma_aligned: bool | None = None

    @property
    def problem_count(self) -> int:
        return len(self.a)

    @property
    def max_m(self) -> int:
        return max(m for m, _, _ in self.shapes)

    @property
    def max_n(self) -> int:
        return max(n for _, _, n in self.shapes)

    @property
    def max_k(self) -> int:
        return max(k for _, k, _ in self.shapes)

    def tile_count_for(self, config: KernelConfig) -> int:
        return sum(math.ceil(m / config.block_m) * math.ceil(n / config.block_n) for m, _, n in self.shapes)

    @property
    def tile_count(self) -> int:
        return self.tile_count_for(self.config)

    def problem_tensors(self):
        return zip(self.a, self.b, self.c)


def _grouped_row_sizes(max_m: int) -> set[int]:
    if max_m <= 32:
        return {16, 32, 64}
    if max_m <= 64:
        return {32, 64, 128}
    if max_m <= 128:
        return {64, 128}
    return {64, 128, 256}


def _grouped_col_sizes(max_m: int, max_n: int) -> set[int]:
    if max_n <= 32:
        return {32, 64}
    if max_n <= 64:
        return {32, 64, 128}
    if max_n <= 128 or max_m <= 64:
        # Wide outputs with few tokens keep 64-column tiles: more independent
        # expert tiles can beat padding efficiency.
        return {64, 128, 256}
    return {128, 256}


def grouped_candidate_configs(
    max_m: int,
    max_n: int,
    max_k: int,
    base_limit: int = 12,
    *,
    problem_count: int = 1,
    sm_count: int = 0,
) -> tuple[KernelConfig, ...]:
    """Bounded tile x persistence candidates (kernels/grouped_gemm.py:114-224)."""
    if min(max_m, max_n, max_k, problem_count) <= 0:
        raise ValueError("grouped candidate dimensions and problem_count must be positive")
    if sm_count < 0:
        raise ValueError("sm_count must be non-negative")
    if problem_count == 1:
        return tuple(
            KernelConfig(c.block_m, c.block_n, c.block_k, c.group_size_m, c.num_warps, c.num_stages, 1)
            for c in matmul_candidate_configs(max_m, max_n, max_k, limit=base_limit)
        )
    rows_ok = _grouped_row_sizes(max_m)
    cols_ok = _grouped_col_sizes(max_m, max_n)
    pool = [
        cfg for cfg in _GROUPED_BASE_CONFIG_POOL
        if cfg.block_m in rows_ok and cfg.block_n in cols_ok and (cfg.block_k == 32 or cfg.block_k <= max_k)
    ]
    heuristic = select_config(max_m, max_n, max_k)
    if heuristic not in pool:
        pool.append(heuristic)

    def score(cfg: KernelConfig) -> tuple[float, float, int, int, int]:
        m_tiles = math.ceil(max_m / cfg.block_m)
        n_tiles = math.ceil(max_n / cfg.block_n)
        k_tiles = math.ceil(max_k / cfg.block_k)
        efficiency = (max_m * max_n * max_k) / (
            m_tiles * cfg.block_m * n_tiles * cfg.block_n * k_tiles * cfg.block_k
        )
        fill = min(1.0, problem_count * m_tiles * n_tiles / sm_count) if sm_count else 1.0
        weighted = efficiency * (0.85 + 0.15 * fill)
        return (-weighted, -fill, cfg.block_m * cfg.block_n, cfg.block_k, cfg.num_warps)

    chosen = diverse_configs(sorted(dict.fromkeys(pool), key=score), base_limit)
    expanded: list[KernelConfig] = []
    for cfg in chosen:
        tiles = problem_count * math.ceil(max_m / cfg.block_m) * math.ceil(max_n / cfg.block_n)
        multipliers = [1]
        if not sm_count or tiles > sm_count:
            multipliers.append(2)
        if cfg.block_m <= 32 and (not sm_count or tiles > 2 * sm_count):
            multipliers.append(4)
        for multiplier in multipliers:
            expanded.append(
                KernelConfig(
                    cfg.block_m, cfg.block_n, cfg.block_k, cfg.group_size_m, cfg.num_warps, cfg.num_stages, multiplier
                )
            )
    return tuple(dict.fromkeys(expanded))


def _shape_signature(shapes: Sequence[tuple[int, int, int]]) -> int:
    """Cache discriminator for a problem list (CRC-32 of the dims, 31 bits)."""
    flat = ",".join(f"{m}x{k}x{n}" for m, k, n in shapes).encode()
    return zlib.crc32(flat) & 0x7FFFFFFF


def _normalize(shapes: Sequence[tuple[int, int, int]], what: str) -> tuple[tuple[int, int, int], ...]:
    normalized = tuple(tuple(int(value) for value in shape) for shape in shapes)
    if any(len(shape) != 3 or any(value <= 0 for value in shape) for shape in normalized):
        raise ValueError(f"every {what} shape must be a positive (M, K, N) triple")
    return normalized


def workspace_from_tensors(a_list, b_list, c_list, config: KernelConfig | None = None, *,
                           swiglu: bool = False) -> GroupedWorkspace:
    """Builds the device tables for caller-owned per-expert tensors.

    The reference builds its tables inside build_grouped_workspace
    (kernels/grouped_gemm.py:528-572); this is the same step for tensors the
    caller already holds (the bench, the multi-rank shards).  With ``swiglu``
    each B_e is a packed [gate | up] weight [K, N] and C_e is [M, N/2]; the
    workspace's operation is "swiglu".
    """
    if not a_list or not (len(a_list) == len(b_list) == len(c_list)):
        raise ValueError("grouped GEMM requires equally many A, B and C matrices (at least one)")
    shapes = []
    for a, b, c in zip(a_list, b_list, c_list):
        out_n = b.shape[1] // 2 if swiglu else b.shape[1]
        if a.ndim != 2 or b.ndim != 2 or c.ndim != 2 or a.shape[1] != b.shape[0] or c.shape != (a.shape[0], out_n):
            raise ValueError(f"shape mismatch: A={tuple(a.shape)}, B={tuple(b.shape)}, C={tuple(c.shape)}")
        if swiglu and b.shape[1] % 2:
            raise ValueError("SwiGLU requires an even packed [gate | up] width")
        if a.dtype != b.dtype or a.dtype != c.dtype or a.dtype != a_list[0].dtype:
            raise ValueError("A, B, and C must share one dtype")
        if not (a.is_cuda and b.is_cuda and c.is_cuda) or len({a.device, b.device, c.device, a_list[0].device}) != 1:
            raise ValueError("A, B, and C must be on the same CUDA device")
        shapes.append((int(a.shape[0]), int(a.shape[1]), int(b.shape[1])))
    normalized = _normalize(shapes, "grouped")
    dtype_name(a_list[0].dtype)
    first_m, first_k, first_n = normalized[0]
    config = config or select_config(first_m, first_n, first_k)
    device = a_list[0].device

    def pointer_tensor(arrays):
        return torch.tensor([item.data_ptr() for item in arrays], device=device, dtype=torch.int64)

    a_ptrs, b_ptrs, c_ptrs = pointer_tensor(a_list), pointer_tensor(b_list), pointer_tensor(c_list)
    dims = torch.tensor([[m, n, k] for m, k, n in normalized], device=device, dtype=torch.int32)
    strides = torch.tensor(
        [[a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1)]
         for a, b, c in zip(a_list, b_list, c_list)],
        device=device, dtype=torch.int64,
    )
    metadata = [a_ptrs, b_ptrs, c_ptrs, dims, strides]
    storage_bytes = sum(x.numel() * x.element_size() for x in [*a_list, *b_list, *c_list, *metadata])
    properties = torch.cuda.get_device_properties(device)
    sm_count = int(properties.multi_processor_count)
    device_signature = (int(properties.major) * 10 + int(properties.minor)) * 1000 + sm_count
    homogeneous = all(shape == normalized[0] for shape in normalized) and all(
        x.is_contiguous() for x in [*a_list, *b_list, *c_list]
    )
    workspace = GroupedWorkspace(
        list(a_list), list(b_list), list(c_list), a_ptrs, b_ptrs, c_ptrs, dims, strides, normalized, config,
        _shape_signature(normalized), device_signature, sm_count, storage_bytes, homogeneous,
    )
    if swiglu:
        workspace.operation = "swiglu"
    return workspace


def build_grouped_workspace(
    shapes: Sequence[tuple[int, int, int]],
    dtype,
    seed: int = 0,
    config: KernelConfig | None = None,
) -> GroupedWorkspace:
    """Seeded per-expert A ~ N(0,1)*0.1, B ~ N(0,1)*0.1, empty C, plus tables
    (kernels/grouped_gemm.py:507-572).  Same generator and draw order as the
    reference, so a seed gives the reference's inputs."""
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch is required")
    if not shapes:
        raise ValueError("grouped GEMM requires at least one problem")
    normalized = _normalize(shapes, "grouped")
    generator = torch.Generator(device="cuda").manual_seed(seed)
    a_list, b_list, c_list = [], [], []
    for m, k, n in normalized:
        a_list.append(torch.empty((m, k), device="cuda", dtype=dtype).normal_(generator=generator).mul_(0.1))
        b_list.append(torch.empty((k, n), device="cuda", dtype=dtype).normal_(generator=generator).mul_(0.1))
        c_list.append(torch.empty((m, n), device="cuda", dtype=dtype))
    return workspace_from_tensors(a_list, b_list, c_list, config)


def build_fused_gate_up_workspace(
    shapes: Sequence[tuple[int, int, int]],
    dtype,
    seed: int = 0,
    config: KernelConfig | None = None,
) -> GroupedWorkspace:
    """Packed W13 problems: N = 2 * local_ffn, output laid out [gate, up]
    (kernels/grouped_gemm.py:575-594).  SiLU(gate) * up stays outside."""
    normalized = tuple(tuple(int(value) for value in shape) for shape in shapes)
    if any(len(shape) != 3 or shape[2] % 2 for shape in normalized):
        raise ValueError("fused Gate+Up shapes require an even packed output dimension")
    workspace = build_grouped_workspace(normalized, dtype, seed, config)
    workspace.operation = "gate_up"
    return workspace


def build_fused_swiglu_workspace(
    shapes: Sequence[tuple[int, int, int]],
    dtype,
    seed: int = 0,
    config: KernelConfig | None = None,
) -> GroupedWorkspace:
    """Packed W13 problems with the SwiGLU epilogue fused: (M, K, N) with
    N = 2 * local_ffn, B_e = [gate | up] drawn exactly as
    build_fused_gate_up_workspace draws it, C_e = silu(A B_gate) * (A B_up)
    of shape [M, N/2].  The reference computes SiLU(gate) * up outside its
    timed GEMM (README.md:55-60); here one launch writes the activation."""
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch is required")
    normalized = tuple(tuple(int(value) for value in shape) for shape in shapes)
    if not normalized:
        raise ValueError("grouped GEMM requires at least one problem")
    if any(len(shape) != 3 or shape[2] % 2 for shape in normalized):
        raise ValueError("fused SwiGLU shapes require an even packed output dimension")
    normalized = _normalize(normalized, "grouped")
    generator = torch.Generator(device="cuda").manual_seed(seed)
    a_list, b_list, c_list = [], [], []
    for m, k, n in normalized:
        a_list.append(torch.empty((m, k), device="cuda", dtype=dtype).normal_(generator=generator).mul_(0.1))
        b_list.append(torch.empty((k, n), device="cuda", dtype=dtype).normal_(generator=generator).mul_(0.1))
        c_list.append(torch.empty((m, n // 2), device="cuda", dtype=dtype))
    return workspace_from_tensors(a_list, b_list, c_list, config, swiglu=True)


def _grid_size(workspace: GroupedWorkspace, config: KernelConfig) -> int:
    """Persistent grid of the reference's kernels (kernels/grouped_gemm.py:597-599).

    The native launch sizes its own grid (one CTA per SM at most, reported in
    ``workspace.launch_info['grid']``); this stays for callers that read it.
    """
    tiles = workspace.tile_count_for(config)
    return max(1, min(tiles, workspace.sm_count * config.cta_multiplier))


def operands_tma_aligned(workspace: GroupedWorkspace) -> bool:
    """True when every A_e and B_e has a 16-byte aligned base, unit inner
    stride and a 16-byte multiple row pitch (the TMA rules)."""
    for a, b in zip(workspace.a, workspace.b):
        for x in (a, b):
            if x.data_ptr() % 16 or x.stride(1) != 1 or x.stride(0) <= 0 or (x.stride(0) * x.element_size()) % 16:
                return False
    return True


_GROUPED_TUNED: dict[tuple, KernelConfig] = {}


def _ensure_scratch(workspace: GroupedWorkspace):
    need = _native.scratch_bytes(workspace.problem_count, workspace.sm_count)
    if workspace.scratch is None or workspace.scratch.numel() < need:
        workspace.scratch = torch.empty(need, dtype=torch.uint8, device=workspace.a[0].device)
    return workspace.scratch


def _launch_native(workspace: GroupedWorkspace, config: KernelConfig, precision: str, aligned: bool) -> dict:
    swiglu = workspace.operation == "swiglu"
    scratch = _ensure_scratch(workspace)
    device = workspace.a[0].device
    if workspace.homogeneous:
        m, k, n = workspace.shapes[0]
    else:
        m, k, n = workspace.max_m, workspace.max_k, workspace.max_n
    with torch.cuda.device(device):
        info = _native.grouped_launch(
            workspace.a_ptrs.data_ptr(), workspace.b_ptrs.data_ptr(), workspace.c_ptrs.data_ptr(),
            workspace.dims.data_ptr(), workspace.strides.data_ptr(), workspace.problem_count,
            workspace.homogeneous, m, n, k, dtype_name(workspace.a[0].dtype), precision, aligned, config,
            scratch.data_ptr(), scratch.numel(), torch.cuda.current_stream(device).cuda_stream, swiglu=swiglu,
        )
    workspace.launch_info = info.as_dict()
    return workspace.launch_info


def launch_grouped(
    workspace: GroupedWorkspace,
    input_precision: str = "ieee",
    config: KernelConfig | None = None,
    *,
    autotune: bool = True,
) -> None:
    """One native launch of the persistent grouped GEMM (kernels/grouped_gemm.py:618-760).

    One problem dispatches to ``launch_matmul`` (scheduler
    ``single_problem_matmul``).  Otherwise the scheduler is
    ``homogeneous_persistent`` for equal contiguous problems and
    ``generic_persistent`` for the rest; ``workspace.config`` records the
    config that ran.  ``autotune=True`` launches the native tile
    ``native_candidates`` picks for the group's largest M (measured policy,
    cached per shape / dtype / precision); ``autotune=False`` launches
    ``config`` mapped to a native tile, so every ``grouped_candidate_configs``
    entry launches.
    """
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
    _native.load()
    if input_precision not in _native.PUBLIC_PRECISIONS:
        raise ValueError(f"input_precision must be 'ieee' or 'tf32', got {input_precision!r}")
    cfg = config or workspace.config
    if workspace.problem_count == 1 and workspace.operation != "swiglu":
        launch_matmul(workspace.a[0], workspace.b[0], workspace.c[0], cfg, input_precision, autotune=autotune)
        from .matmul import last_launch_info

        workspace.config = last_matmul_config(cfg) if autotune else cfg
        workspace.launch_info = last_launch_info()
        workspace.scheduler = SCHEDULER_SINGLE
        return
    if workspace.tma_aligned is None:
        workspace.tma_aligned = operands_tma_aligned(workspace)
    aligned = workspace.tma_aligned
    scheduler = SCHEDULER_HOMOGENEOUS if workspace.homogeneous else SCHEDULER_GENERIC
    if not autotune:
        _launch_native(workspace, cfg, input_precision, aligned)
        workspace.config = cfg
        workspace.scheduler = scheduler
        return
    key = (
        workspace.shape_signature, workspace.problem_count, workspace.device_signature, workspace.homogeneous,
        aligned, input_precision, workspace.a[0].dtype,
    )
    candidates = native_candidates(workspace.max_m, workspace.max_k,
                                   split_tail=workspace.homogeneous and workspace.operation != "swiglu")
    best, _ = autotune_over(
        candidates, lambda c: _launch_native(workspace, c, input_precision, aligned), key, _GROUPED_TUNED
    )
    workspace.config = best
    workspace.scheduler = scheduler


_AGGREGATE_SCRATCH: dict[tuple[int, int], object] = {}
_last_aggregate_info: dict | None = None


def last_aggregate_launch_info() -> dict | None:
    """Native kernel of the most recent launch_grouped_mm call (path, tile, grid)."""
    return _last_aggregate_info


def launch_grouped_mm(mat_a, mat_b, offs, out=None, *, config: KernelConfig | None = None,
                      input_precision: str = "ieee", swiglu: bool = False):
    """Grouped GEMM over the expert-sorted aggregate layout, in one native launch:
    ``out[offs[e-1]:offs[e]] = mat_a[offs[e-1]:offs[e]] @ mat_b[e]``.

    The layout of ``torch.nn.functional.grouped_mm(mat_a, mat_b, offs=offs)``
    that the reference's torch provider builds (kernels/torch_grouped_gemm.py:
    142-158): ``mat_a`` [T, K] with tokens sorted by expert, ``mat_b`` [E, K, N],
    ``offs`` int32 [E] cumulative row ends on the same device (read by the
    kernel, so no host synchronisation and CUDA-graph capturable once the
    scratch exists: make the first call for a group size eagerly).  ``offs``
    may also hold S = P * E segments (P senders' blocks, each sorted by the E
    experts, as an expert-parallel rank receives them): segment s multiplies
    ``mat_b[s % E]``.  Rows of
    ``mat_a`` / ``mat_b`` / ``out`` may be padded (row strides ≥ the logical
    width); columns must be contiguous.  With ``swiglu`` each ``mat_b[e]`` is a
    packed [gate | up] weight and ``out`` is [T, N/2] =
    silu(A B_gate) * (A B_up).  ``config`` defaults to the native tile policy
    for the average rows per expert.  Returns ``out``.
    """
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
    _native.load()
    if mat_a.ndim != 2 or mat_b.ndim != 3 or offs.ndim != 1:
        raise ValueError("expected mat_a [T, K], mat_b [E, K, N] and offs [E]")
    total, k = mat_a.shape
    experts, kb, n = mat_b.shape
    segments = offs.shape[0]
    if kb != k or experts == 0 or segments == 0 or segments % experts:
        raise ValueError(f"shape mismatch: mat_a={tuple(mat_a.shape)}, mat_b={tuple(mat_b.shape)}, offs={tuple(offs.shape)}")
    if offs.dtype != torch.int32:
        raise ValueError("offs must be int32 cumulative row ends")
    if mat_a.dtype != mat_b.dtype:
        raise ValueError("mat_a and mat_b must share one dtype")
    if len({mat_a.device, mat_b.device, offs.device}) != 1 or not mat_a.is_cuda:
        raise ValueError("mat_a, mat_b and offs must be on the same CUDA device")
    if swiglu and n % 2:
        raise ValueError("SwiGLU requires an even packed [gate | up] width")
    out_n = n // 2 if swiglu else n
    if out is None:
        out = torch.empty((total, out_n), device=mat_a.device, dtype=mat_a.dtype)
    if out.shape != (total, out_n) or out.dtype != mat_a.dtype or out.device != mat_a.device:
        raise ValueError(f"out must be [{total}, {out_n}] {mat_a.dtype} on {mat_a.device}")
    if mat_a.stride(1) != 1 or mat_b.stride(2) != 1 or out.stride(1) != 1 or mat_b.stride(0) < k * mat_b.stride(1):
        raise ValueError("columns of mat_a, mat_b and out must be contiguous (row padding is allowed)")
    if input_precision not in _native.PUBLIC_PRECISIONS:
        raise ValueError(f"input_precision must be 'ieee' or 'tf32', got {input_precision!r}")
    key = (mat_a.device.index or 0, segments)
    scratch = _AGGREGATE_SCRATCH.get(key)
    if scratch is None:
        scratch = torch.empty(_native.scratch_bytes(segments, 0), dtype=torch.uint8, device=mat_a.device)
        _AGGREGATE_SCRATCH[key] = scratch
    global _last_aggregate_info
    cfg = config or native_candidates(max(1, -(-total // segments)), k, split_tail=False)[0]
    with torch.cuda.device(mat_a.device):
        info = _native.offsets_launch(
            mat_a.data_ptr(), mat_b.data_ptr(), out.data_ptr(), offs.data_ptr(), segments, total, n, k,
            mat_a.stride(0), mat_b.stride(0), mat_b.stride(1), out.stride(0), dtype_name(mat_a.dtype),
            input_precision, swiglu, cfg, scratch.data_ptr(), scratch.numel(),
            torch.cuda.current_stream(mat_a.device).cuda_stream, b_count=experts if segments != experts else 0,
        )
    _last_aggregate_info = info.as_dict()
    return out


def launch_grouped_mm_scatter(mat_a, mat_b, offs, row_origin, peer_regions, dst_offset: int, dst_pitch_bytes: int,
                              *, config: KernelConfig | None = None, input_precision: str = "ieee") -> None:
    """``launch_grouped_mm`` whose output rows are not written to an ``out``
    matrix but each to its own destination: row R goes to byte ``dst_offset +
    (row_origin[R] & (2**40 - 1)) * dst_pitch_bytes`` of the region whose base
    is ``peer_regions[row_origin[R] >> 40]`` (int64 device tables; a negative
    origin drops the row).  The expert-parallel layer returns W2 rows to the
    ranks that sent the tokens this way, from the GEMM epilogue."""
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
    _native.load()
    total, k = mat_a.shape
    experts, kb, n = mat_b.shape
    segments = offs.shape[0]
    if kb != k or experts == 0 or segments == 0 or segments % experts or offs.dtype != torch.int32:
        raise ValueError(f"shape mismatch: mat_a={tuple(mat_a.shape)}, mat_b={tuple(mat_b.shape)}, offs={tuple(offs.shape)}")
    if row_origin.dtype != torch.int64 or row_origin.numel() < total or peer_regions.dtype != torch.int64:
        raise ValueError("row_origin must be int64 with a row per row of mat_a; peer_regions int64")
    if mat_a.stride(1) != 1 or mat_b.stride(2) != 1 or mat_b.stride(0) < k * mat_b.stride(1):
        raise ValueError("columns of mat_a and mat_b must be contiguous")
    key = (mat_a.device.index or 0, segments)
    scratch = _AGGREGATE_SCRATCH.get(key)
    if scratch is None:
        scratch = torch.empty(_native.scratch_bytes(segments, 0), dtype=torch.uint8, device=mat_a.device)
        _AGGREGATE_SCRATCH[key] = scratch
    cfg = config or native_candidates(max(1, -(-total // segments)), k, split_tail=False)[0]
    with torch.cuda.device(mat_a.device):
        _native.offsets_scatter_launch(
            mat_a.data_ptr(), mat_b.data_ptr(), offs.data_ptr(), segments,
            experts if segments != experts else 0, total, n, k, mat_a.stride(0), mat_b.stride(0), mat_b.stride(1),
            row_origin.data_ptr(), peer_regions.data_ptr(), peer_regions.numel(), dst_offset, dst_pitch_bytes,
            dtype_name(mat_a.dtype),
            input_precision, cfg, scratch.data_ptr(), scratch.numel(), torch.cuda.current_stream(mat_a.device).cuda_stream,
        )


def check_device_errors(device=None) -> None:
    """Synchronises ``device`` and raises RuntimeError if a native kernel
    reported a device-side failure (bounded wait expiry, skipped problem)."""
    index = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    torch.cuda.synchronize(index)
    word = _native.read_and_clear_error_word(index)
    if word:
        raise RuntimeError("native kernel reported: " + "; ".join(_native.describe_error_word(word)))
