"""Masked single GEMM on B200: the drop-in for the reference's kernels/matmul.py.

Public surface (names, arguments, errors and return values) follows the
reference module so its drivers (benchmark_shapes.py, benchmark_moe.py via
select_config) run unchanged:

* ``KernelConfig``            kernels/matmul.py:19-32
* ``select_config``           kernels/matmul.py:35-45
* ``_MATMUL_CONFIG_POOL``     kernels/matmul.py:54-98
* ``diverse_configs``         kernels/matmul.py:101-120
* ``matmul_candidate_configs`` kernels/matmul.py:146-170
* ``last_matmul_config``      kernels/matmul.py:300-315
* ``launch_matmul``           kernels/matmul.py:332-392

The candidate heuristics are restated so that they return what the
reference returns (pinned by tests/golden/configs.json.gz, generated from the
reference).  The launch itself goes to the native sm_100a library: a TMA +
tcgen05 tensor-core kernel when the operands satisfy the TMA rules, a
generic-stride kernel otherwise.  A ``KernelConfig`` selects the native tile
(block_m / block_n); see ``native_tile_note``.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

try:
    import torch
except ImportError:  # CPU-only inspection of the config heuristics stays possible
    torch = None

from . import _native, _timing


@dataclass(frozen=True)
class KernelConfig:
    """Tile record (fields of kernels/matmul.py:19-32).

    block_m / block_n choose the native tile; block_k, group_size_m,
    num_warps, num_stages and cta_multiplier are carried for provenance and
    for the reference's candidate bookkeeping.
    """

    block_m: int
    block_n: int
    block_k: int
    group_size_m: int
    num_warps: int
    num_stages: int
    cta_multiplier: int = 1

    def as_dict(self) -> dict[str, int]:
        return asdict(self)


native_tile_note = (
    "block_m <= 64 -> swap-AB tile with block_m tokens (16/32/64) x 128 or 256 weight columns; "
    "block_m == 128 -> 128-token MMA tile x 64/128/256 columns; block_m >= 256 -> CTA-pair 256 x 256 tile "
    "(256 x 512 with block_n >= 256) for fp16/bf16, swap-AB 256 x 128 for fp32"
)


def _n_tile_for_small_m(n: int, inclusive_64: bool) -> int:
    if n <= 32:
        return 32
    if n < 128 if not inclusive_64 else n <= 64:
        return 64
    return 128


def select_config(m: int, n: int, k: int) -> KernelConfig:
    """Heuristic tile used before any autotuned launch (kernels/matmul.py:35-45)."""
    if m <= 32:
        rows = 16 if m <= 16 else 32
        return KernelConfig(rows, _n_tile_for_small_m(n, inclusive_64=False), 32, 4, 2, 2 if rows == 16 else 3)
    if m <= 64:
        return KernelConfig(64, _n_tile_for_small_m(n, inclusive_64=True), 32, 8, 4, 3)
    if n <= 64:
        return KernelConfig(128, 32 if n <= 32 else 64, 32, 8, 4, 3)
    return KernelConfig(64, 128, 64 if k >= 8192 else 32, 8, 4, 3)


# (block_m, block_n, block_k, group_size_m, num_warps, num_stages), in the
# reference's order (kernels/matmul.py:54-98).  The order is part of the
# contract: candidate ranking is a stable sort and coverage ties go to the
# earlier entry.
_MATMUL_POOL_ROWS = (
    (16, 32, 32, 1, 2, 2), (16, 64, 32, 4, 2, 2), (16, 128, 32, 4, 4, 2), (16, 128, 64, 8, 4, 3),
    (32, 32, 32, 4, 2, 2), (32, 64, 32, 8, 2, 3), (32, 64, 64, 4, 4, 3), (32, 128, 32, 8, 4, 3),
    (32, 128, 64, 4, 4, 3), (32, 256, 32, 8, 8, 3), (64, 32, 32, 8, 4, 3), (64, 64, 32, 8, 4, 3),
    (64, 64, 64, 4, 4, 4), (64, 64, 128, 4, 4, 4), (64, 128, 32, 8, 4, 3), (64, 128, 64, 8, 4, 4),
    (64, 128, 128, 4, 8, 4), (64, 256, 32, 8, 8, 3), (64, 256, 64, 8, 8, 4), (128, 32, 32, 8, 4, 3),
    (128, 64, 32, 8, 4, 3), (128, 64, 64, 8, 4, 4), (128, 128, 32, 8, 8, 3), (128, 128, 64, 8, 8, 4),
    (128, 256, 64, 8, 8, 4), (256, 32, 32, 8, 8, 3), (256, 64, 32, 8, 8, 3), (256, 64, 64, 8, 8, 4),
    (256, 128, 64, 8, 8, 4),
    (16, 32, 32, 4, 2, 2), (16, 128, 32, 4, 2, 2), (32, 32, 32, 4, 2, 3), (32, 64, 32, 4, 2, 3),
    (32, 128, 32, 4, 2, 3), (16, 128, 64, 4, 4, 2), (32, 128, 64, 4, 4, 5), (64, 128, 64, 4, 4, 2),
    (64, 128, 64, 4, 4, 5), (64, 128, 64, 8, 4, 3), (128, 128, 64, 4, 4, 3), (128, 128, 64, 8, 8, 5),
)
_MATMUL_CONFIG_POOL: tuple[KernelConfig, ...] = tuple(KernelConfig(*row) for row in _MATMUL_POOL_ROWS)

_FEATURE_FIELDS = ("block_m", "block_n", "block_k", "num_warps", "num_stages", "group_size_m")


def _features(config: KernelConfig) -> frozenset:
    return frozenset((field, getattr(config, field)) for field in _FEATURE_FIELDS)


def diverse_configs(ordered: list[KernelConfig], limit: int) -> list[KernelConfig]:
    """Greedy feature coverage (kernels/matmul.py:101-120).

    Repeatedly takes the first remaining config that adds the most uncovered
    (field, value) features, so rank order breaks ties.
    """
    pending = list(dict.fromkeys(ordered))
    chosen: list[KernelConfig] = []
    covered: set = set()
    while pending and len(chosen) < max(1, limit):
        gains = [len(_features(cfg) - covered) for cfg in pending]
        pick = pending.pop(gains.index(max(gains)))
        chosen.append(pick)
        covered |= _features(pick)
    return chosen


# Upper bounds of each shape family and the tile sizes it admits
# (kernels/matmul.py:123-143).
_M_FAMILIES = ((16, {16, 32}), (32, {16, 32, 64}), (64, {32, 64, 128}), (128, {64, 128}), (None, {64, 128, 256}))
_N_FAMILIES = ((32, {32, 64}), (64, {32, 64, 128}), (128, {64, 128, 256}), (None, {128, 256}))


def _family(value: int, families) -> set[int]:
    for bound, sizes in families:
        if bound is None or value <= bound:
            return set(sizes)
    raise AssertionError("unreachable")


def _family_limits(m: int, n: int) -> tuple[set[int], set[int]]:
    return _family(m, _M_FAMILIES), _family(n, _N_FAMILIES)


def matmul_candidate_configs(m: int, n: int, k: int, limit: int = 10) -> tuple[KernelConfig, ...]:
    """Bounded candidate set for one M/N/K shape family (kernels/matmul.py:146-170)."""
    rows_ok, cols_ok = _family_limits(m, n)
    pool = [
        cfg for cfg in _MATMUL_CONFIG_POOL
        if cfg.block_m in rows_ok and cfg.block_n in cols_ok and (cfg.block_k == 32 or cfg.block_k <= k)
    ]
    heuristic = select_config(m, n, k)
    if heuristic not in pool:
        pool.append(heuristic)

    def padded(size: int, tile: int) -> int:
        return -(-size // tile) * tile

    def score(cfg: KernelConfig) -> tuple[float, int, int]:
        useful = (m * n) / max(1, padded(m, cfg.block_m) * padded(n, cfg.block_n))
        shallow_k = 0.15 if k < 2 * cfg.block_k else 0.0
        return (shallow_k - useful, cfg.block_m * cfg.block_n, cfg.block_k)

    ordered = sorted(dict.fromkeys(pool), key=score)
    chosen = diverse_configs(ordered, limit)
    two_warp = next((cfg for cfg in ordered if cfg.num_warps == 2), None)
    if two_warp is not None and two_warp not in chosen:
        chosen[-1] = two_warp
    return tuple(chosen)


# ------------------------------------------------------------------ launches
_DTYPE_NAMES = {}
if torch is not None:
    _DTYPE_NAMES = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}

# autotune cache: key -> winning KernelConfig; and the most recent winner
_MATMUL_TUNED: dict[tuple, KernelConfig] = {}
_last_tuned: KernelConfig | None = None
_last_launch_info: dict | None = None


def dtype_name(dtype) -> str:
    try:
        return _DTYPE_NAMES[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {dtype}; expected float16, bfloat16 or float32") from exc


def _device_signature(device) -> int:
    properties = torch.cuda.get_device_properties(device)
    return (int(properties.major) * 10 + int(properties.minor)) * 1000 + int(properties.multi_processor_count)


def last_matmul_config(fallback: KernelConfig) -> KernelConfig:
    """Config chosen by the most recent autotuned launch (kernels/matmul.py:300-315)."""
    return _last_tuned if _last_tuned is not None else fallback


def last_launch_info() -> dict | None:
    """Native kernel (path, tile, stages, grid) that ran for the most recent launch."""
    return _last_launch_info


def _validate_matrices(a, b, c) -> tuple[int, int, int]:
    """Shape / device / dtype checks with the reference's errors (kernels/matmul.py:318-329)."""
    if a.ndim != 2 or b.ndim != 2 or c.ndim != 2:
        raise ValueError("A, B, and C must be matrices")
    m, k = a.shape
    kb, n = b.shape
    if k != kb or c.shape != (m, n):
        raise ValueError(f"shape mismatch: A={a.shape}, B={b.shape}, C={c.shape}")
    if a.device != b.device or a.device != c.device or not a.is_cuda:
        raise ValueError("A, B, and C must be on the same CUDA device")
    if a.dtype != b.dtype or a.dtype != c.dtype:
        raise ValueError("A, B, and C must have the same dtype")
    dtype_name(a.dtype)
    return int(m), int(n), int(k)


def _check_precision(input_precision: str) -> str:
    if input_precision not in _native.PUBLIC_PRECISIONS:
        raise ValueError(f"input_precision must be 'ieee' or 'tf32', got {input_precision!r}")
    return input_precision


# Single GEMMs at least this large repack operands the TMA cannot address
# (row pitch not a multiple of 16 bytes, unit-stride violations) so they run
# on the tensor cores, and fp32 "ieee" ones take the 3xTF32 split; smaller
# ones use the generic-stride kernel directly.  The generic kernel has one
# 64 x 64 tile per CTA and no split of K, so a small output with a long K
# leaves most SMs idle: 127 x 8191 x 127 (0.26 GFLOP) ran 1.17 ms there
# against tens of microseconds for one tensor-core CTA after the repack.
REPACK_MIN_FLOPS = 1 << 24


def _tma_addressable(x) -> bool:
    return (x.data_ptr() % 16 == 0 and x.stride(1) == 1 and x.stride(0) > 0
            and (x.stride(0) * x.element_size()) % 16 == 0)


def _repacked(x, stream: int):
    """Copy of ``x`` in a buffer whose row pitch is a multiple of 16 bytes
    (a view of its first ``cols`` columns), made by the native repack kernel
    on ``stream``."""
    rows, cols = x.shape
    step = 16 // x.element_size()
    pitch = -(-cols // step) * step
    buffer = torch.empty((rows, pitch), dtype=x.dtype, device=x.device)
    _native.repack(x.data_ptr(), rows, cols, x.stride(0), x.stride(1), buffer.data_ptr(), pitch,
                   x.element_size(), stream)
    return buffer[:, :cols]


def split_operands_3xtf32(a, b, stream: int):
    """The 3xTF32 operands of an fp32 "ieee" GEMM (matrix_split_tf32x3):
    A' = [hi(A) | lo(A) | hi(A)] of shape [M, 3K] and B' = [hi(B); hi(B);
    lo(B)] of shape [3K, N], in buffers whose row pitch is a multiple of 16
    bytes.  A' @ B' in TF32 = hi hi + lo hi + hi lo, which restores fp32
    accuracy (Ootomo & Yokota 2022) on the tensor cores."""
    m, k = a.shape
    n = b.shape[1]
    a3 = torch.empty((m, -(-3 * k // 4) * 4), dtype=torch.float32, device=a.device)[:, :3 * k]
    b3 = torch.empty((3 * k, -(-n // 4) * 4), dtype=torch.float32, device=a.device)[:, :n]
    _native.split_tf32x3(a.data_ptr(), m, k, a.stride(0), a.stride(1), a3.data_ptr(), a3.stride(0), 0, stream)
    _native.split_tf32x3(b.data_ptr(), k, n, b.stride(0), b.stride(1), b3.data_ptr(), b3.stride(0), 1, stream)
    return a3, b3


# Split-K for fp32 single GEMMs on the tensor cores: an output of few tiles
# (127 rows or columns) with a long K leaves most SMs idle, e.g.
# 127 x 8191 @ 8191 x 8191 covers 64 of 148 SMs for its whole K.  From
# SPLITK_MIN_K such a GEMM runs as one grouped launch over `splits` K slices
# (problem s multiplies A[:, s kc : (s + 1) kc] by the matching rows of B into
# fp32 partial s), and matrix_sum_partials adds the partials in a fixed order.
# fp32 only: the partials keep fp32, so the result is rounded once, as one
# tensor-core launch rounds it.
SPLITK_MIN_K = 2048
_SM_COUNT: dict = {}


def _sm_count(device) -> int:
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _SM_COUNT:
        _SM_COUNT[index] = torch.cuda.get_device_properties(index).multi_processor_count
    return _SM_COUNT[index]


def splitk_splits(m: int, n: int, k: int, sms: int) -> int:
    """K slices for an fp32 tensor-core GEMM: 1 (no split) unless the output
    has at most half as many 128 x 128 tiles as the GPU has SMs and K is at
    least SPLITK_MIN_K; then enough slices to cover the SMs, at most 32, each
    at least 1024 deep, or 256 for an output of at most 8 tiles (a single
    tile's long K is latency-bound: its ring holds only a few k-blocks in
    flight).  Two slices only from K = 6144: below it the partials' traffic
    and the sum cost more than the second half of the SMs gains.  Measured
    on the configs[4] sweep: 256-deep slices gain 1.1-1.4x on 1-8 tile
    outputs and lose 0.85x at 32 tiles (127 x 3000 x 4095); two slices lose
    0.85x at 1000 x 4095 x 1000."""
    tiles = -(-m // 128) * -(-n // 128)
    if k < SPLITK_MIN_K or 2 * tiles > sms:
        return 1
    depth = 256 if tiles <= 8 else 1024
    splits = max(1, min(32, sms // tiles, k // depth))
    return 1 if splits == 2 and k < 6144 else splits


def _launch_split_k(a, b, c, m: int, n: int, k: int, splits: int, precision: str, config, stream: int):
    """One grouped launch over `splits` K slices of the fp32 GEMM a @ b (both
    TMA-addressable: unit column stride, 16-byte row pitch) into fp32
    partials, then their sum into c.  Every table is built on the device, so
    the launch can be recorded into a CUDA graph."""
    device = a.device
    kc = -(-k // splits)
    kc = -(-kc // 64) * 64  # whole 64-element slices keep every slice base 16-byte aligned
    splits = -(-k // kc)
    partials = torch.empty((splits, m, n), dtype=torch.float32, device=device)
    index = torch.arange(splits, dtype=torch.int64, device=device)
    a_ptrs = index * (kc * 4) + a.data_ptr()
    b_ptrs = index * (kc * b.stride(0) * 4) + b.data_ptr()
    c_ptrs = index * (m * n * 4) + partials.data_ptr()
    # fill_ on views only: an element assignment would copy a host scalar,
    # which a CUDA-graph capture refuses.
    dims = torch.empty((splits, 3), dtype=torch.int32, device=device)
    for col, value in ((0, m), (1, n), (2, kc)):
        dims[:, col].fill_(value)
    dims[splits - 1:, 2].fill_(k - kc * (splits - 1))
    strides = torch.empty((splits, 6), dtype=torch.int64, device=device)
    for col, value in enumerate((a.stride(0), 1, b.stride(0), 1, n, 1)):
        strides[:, col].fill_(value)
    need = _native.scratch_bytes(splits, _sm_count(device))
    scratch = torch.empty(need, dtype=torch.uint8, device=device)
    info = _native.grouped_launch(
        a_ptrs.data_ptr(), b_ptrs.data_ptr(), c_ptrs.data_ptr(), dims.data_ptr(), strides.data_ptr(), splits,
        False, m, n, kc, "fp32", precision, True, config, scratch.data_ptr(), need, stream,
    )
    _native.sum_partials(partials.data_ptr(), splits, m, n, c.data_ptr(), c.stride(0), c.stride(1), "fp32", stream)
    return info, splits


def _launch_once(a, b, c, m: int, n: int, k: int, config: KernelConfig, precision: str) -> dict:
    global _last_launch_info
    stream = torch.cuda.current_stream(a.device).cuda_stream
    if a.dtype == torch.float32 and precision == "ieee" and 2 * m * n * k >= REPACK_MIN_FLOPS and k > 0:
        # Full fp32 accuracy on the tensor cores: one TF32 GEMM of depth 3K
        # over the split operands, its accumulator summed in fp32 registers
        # every 256 K (the tensor core's own accumulation loses accuracy in
        # proportion to K).
        with torch.cuda.device(a.device):
            a3, b3 = split_operands_3xtf32(a, b, stream)
            splits = splitk_splits(m, n, 3 * k, _sm_count(a.device))
            if splits > 1:
                info, splits = _launch_split_k(a3, b3, c, m, n, 3 * k, splits, "tf32_fp32acc", config, stream)
            else:
                info = _native.matmul_launch(
                    a3.data_ptr(), b3.data_ptr(), c.data_ptr(), m, n, 3 * k,
                    (a3.stride(0), 1, b3.stride(0), 1, c.stride(0), c.stride(1)), "fp32", "tf32_fp32acc", config,
                    stream,
                )
        _last_launch_info = {**info.as_dict(), "repacked": True, "split_3xtf32": True, "split_k": splits}
        return _last_launch_info
    tensor_core = a.dtype != torch.float32 or precision == "tf32"
    repacked = False
    splits = 1
    with torch.cuda.device(a.device):
        if tensor_core and 2 * m * n * k >= REPACK_MIN_FLOPS and k > 0:
            if not _tma_addressable(a):
                a, repacked = _repacked(a, stream), True
            if not _tma_addressable(b):
                b, repacked = _repacked(b, stream), True
            if a.dtype == torch.float32:
                splits = splitk_splits(m, n, k, _sm_count(a.device))
        if splits > 1:
            info, splits = _launch_split_k(a, b, c, m, n, k, splits, precision, config, stream)
        else:
            info = _native.matmul_launch(
                a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
                (a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1)),
                dtype_name(a.dtype), precision, config, stream,
            )
    _last_launch_info = {**info.as_dict(), "repacked": repacked, "split_3xtf32": False, "split_k": splits}
    return _last_launch_info


def _tile_key(info: dict) -> tuple:
    return (info["path"], info["swap_ab"], info["tile_m"], info["tile_n"])


# Native tiles, named by the pool KernelConfig that selects them.
TILE_SWAP_16x256 = KernelConfig(16, 256, 64, 4, 8, 4)
TILE_SWAP_32x256 = KernelConfig(32, 256, 64, 4, 8, 4)
TILE_SWAP_64x256 = KernelConfig(64, 256, 64, 8, 8, 4)
TILE_TOKENS_128x256 = KernelConfig(128, 256, 64, 8, 8, 4)
TILE_PAIR_256x256 = KernelConfig(256, 128, 64, 8, 8, 4)  # CTA pair for fp16/bf16, swap-AB 256 x 128 for fp32
TILE_PAIR_256x512 = KernelConfig(256, 256, 64, 8, 8, 4)  # CTA pair, two 256-column halves (fp16/bf16)


def native_candidates(max_m: int, max_k: int | None = None, *, split_tail: bool = True) -> tuple[KernelConfig, ...]:
    """The native tile ``autotune=True`` launches for ``max_m`` token rows
    (and reduction depth ``max_k``).  ``split_tail`` says whether the launch
    can run a short last wave of 256 x 512 tiles as half-width items (an
    exact tile count: a single GEMM or a homogeneous group, no SwiGLU).

    Measured on B200 over whole DeepSeek-V3 W13 and W2 steps (same-box A/B
    runs of tile maps), where the GPU sits at its power cap and every launch's
    energy sets the clock of the others: the token tile fits M exactly (swap-AB
    16 / 32 / 64 tokens x 256 weight columns, so no MMA work is spent on padding
    rows), 128-token x 256-column tiles at M <= 128, and CTA-pair tiles beyond.
    The 256 x 512 pair tile moves 25% fewer bytes from L2 per MMA than the
    256 x 256 one but has a single TMEM accumulator, freed by halves (only
    the first k-blocks of the next tile overlap the drain), and half as many
    tiles; a short last wave of them runs as half-width items.  It wins from
    M = 512, and at M = 256 on deep K (W13, K = 7168: 4% on the EP and TP
    launches); at M = 256 with K = 2048 (W2 EP) the 256 x 256 tile's fully
    overlapped epilogue keeps it level or ahead.  On
    short K (K <= 1024: W2 TP, K = 256) the epilogue dominates every tile:
    above M = 128 the 256 x 512 pair (its drain overlapped by the next tile's
    first k-blocks, a four-stage ring) beats the one-CTA 128 x 256 tile by
    9-17% per launch (whole W2 TP step 609 against 543 TFLOP/s), and from
    M = 32 to 128 the 128 x 256 tile beats the swap-AB tiles, whose
    column-per-lane stores suit outputs that are small next to the weights.
    Timing candidates alone at boost clocks (the reference's hot
    autotune) picks tiles that lose once the GPU is power-capped, so the
    policy is fixed rather than re-timed per shape.
    """
    if max_m <= 16:
        return (TILE_SWAP_16x256,)
    if max_k is not None and max_k <= 1024:
        # Short K (W2 TP, K = 256): output writes dominate, and the row
        # tiles' TMA-store epilogues beat the swap-AB tiles' column-per-lane
        # stores from M = 32 (tile sweep: 0.75 vs 0.63 of roofline at M = 32,
        # 0.79 vs 0.46 at M = 64).
        return (TILE_PAIR_256x512,) if max_m > 128 else (TILE_TOKENS_128x256,)
    if max_m <= 32:
        return (TILE_SWAP_32x256,)
    if max_m <= 64:
        return (TILE_SWAP_64x256,)
    if max_m <= 128:
        return (TILE_TOKENS_128x256,)
    if max_m > 256 or (split_tail and max_k is not None and max_k >= 4096):
        return (TILE_PAIR_256x512,)
    return (TILE_PAIR_256x256,)


def autotune_over(candidates, launch, key: tuple, cache: dict) -> tuple[KernelConfig, dict]:
    """Launches the cached choice for `key`, choosing it on first use.

    One candidate is launched as is.  With several, each is launched once
    eagerly; candidates that map to a native tile already seen are not timed
    again, and the distinct tiles are timed with CUDA-graph event samples
    (_timing.graph_median_ms).  Under stream capture nothing is timed.
    """
    if key in cache:
        return cache[key], launch(cache[key])
    if len(candidates) == 1 or _timing.capturing():
        cache[key] = candidates[0]
        return candidates[0], launch(candidates[0])
    seen: dict[tuple, KernelConfig] = {}
    for candidate in candidates:
        info = launch(candidate)
        seen.setdefault(_tile_key(info), candidate)
    if len(seen) == 1:  # every candidate runs the same kernel (e.g. the generic-stride path)
        cache[key] = next(iter(seen.values()))
        return cache[key], launch(cache[key])
    best, best_ms = None, float("inf")
    for candidate in seen.values():
        ms = _timing.graph_median_ms(lambda cand=candidate: launch(cand))
        if ms < best_ms:
            best, best_ms = candidate, ms
    cache[key] = best
    return best, launch(best)


def launch_matmul(
    a,
    b,
    c,
    config: KernelConfig | None = None,
    input_precision: str = "ieee",
    *,
    autotune: bool = True,
) -> None:
    """C = A @ B on the native kernels (kernels/matmul.py:332-392).

    ``autotune=True`` launches the native tile ``native_candidates`` picks
    for the shape (cached per shape/stride/dtype/precision key);
    ``autotune=False`` launches ``config`` (or the heuristic
    ``select_config``), mapped to a native tile.  Large GEMMs whose A or B the
    TMA cannot address (masked shapes such as fp32 rows of 127 or 8191
    elements) are first copied into 16-byte-pitched buffers by the native
    repack kernel; C is always written in place through its own strides.
    """
    global _last_tuned
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
    _native.load()
    m, n, k = _validate_matrices(a, b, c)
    precision = _check_precision(input_precision)
    if not autotune:
        _launch_once(a, b, c, m, n, k, config or select_config(m, n, k), precision)
        return
    key = (
        m, n, k, a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1),
        a.dtype, precision, _device_signature(a.device),
        a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0,
    )
    best, _ = autotune_over(
        native_candidates(m, k), lambda cfg: _launch_once(a, b, c, m, n, k, cfg, precision), key, _MATMUL_TUNED,
    )
    _last_tuned = best
