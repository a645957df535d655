"""ctypes binding of the native library (``include/moe_gemm_b200.h``).

The shared object ``libmoe_gemm_b200.so`` is built in-tree next to this file
(``make -C moe-gemm-parallel-bench_b200/csrc``).  There is no fallback: if the
library is missing or cannot be loaded, every launch raises ``RuntimeError`` --
the same exception the reference raises when its Triton runtime is unavailable
(kernels/grouped_gemm.py:626-627, kernels/matmul.py:342-343).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIBRARY_NAME = "libmoe_gemm_b200.so"
LIBRARY_PATH = Path(os.environ.get("MGB_LIBRARY", Path(__file__).resolve().parent / LIBRARY_NAME))

# enum values of include/moe_gemm_b200.h
DTYPE_CODES = {"fp16": 0, "bf16": 1, "fp32": 2}
PRECISION_CODES = {"ieee": 0, "tf32": 1, "tf32_fp32acc": 2}
# The precisions of the reference's API (kernels/matmul.py:268); "tf32_fp32acc" is
# internal: TF32 products with chunked fp32 accumulation, used on 3xTF32 operands.
PUBLIC_PRECISIONS = ("ieee", "tf32")
STATUS_OK = 0
STATUS_INVALID = 1
STATUS_UNSUPPORTED = 2
STATUS_CUDA = 3
STATUS_SCRATCH = 4

# Every symbol the header declares (checked by the CPU tests).
EXPORTED_SYMBOLS = (
    "grouped_gemm_scratch_bytes",
    "grouped_gemm_launch",
    "grouped_gemm_swiglu_launch",
    "grouped_gemm_offsets_launch",
    "grouped_gemm_offsets_launch_ex",
    "grouped_gemm_offsets_scatter_launch",
    "moe_route_layout",
    "moe_permute",
    "moe_combine",
    "moe_ep_region_layout",
    "moe_ep_shared_alloc",
    "moe_ep_shared_free",
    "moe_ep_peer_open",
    "moe_ep_peer_close",
    "moe_ep_exchange_counts",
    "moe_ep_dispatch",
    "moe_ep_combine",
    "grouped_gemm_fp8_launch",
    "grouped_gemm_launch_noalloc",
    "matmul_launch",
    "matrix_repack",
    "matrix_split_tf32x3",
    "matrix_sum_partials",
    "read_and_clear_error_word",
    "mgb_set_debug",
    "mgb_status_string",
    "mgb_abi_version",
)

# error bits of the device error word (mgb_ptx.cuh ErrorBits)
ERROR_BITS = {
    1 << 0: "MMA issuer timed out waiting for a loaded stage",
    1 << 1: "producer timed out waiting for a free stage",
    1 << 2: "epilogue timed out waiting for an accumulator",
    1 << 3: "MMA issuer timed out waiting for a drained accumulator",
    1 << 4: "teardown timed out waiting for in-flight copies",
    1 << 5: "a problem's operands broke the TMA alignment promise and were skipped",
    1 << 6: "a problem had invalid dimensions and was skipped",
    1 << 7: "test-only barrier wait timed out",
    1 << 8: "an output tile store fell outside C and was not issued (kernel bug)",
    1 << 9: "an expert-parallel barrier timed out waiting for a peer rank",
    1 << 10: "expert-parallel rows beyond a rank's receive capacity were dropped",
}
EP_HANDLE_BYTES = 64
EP_MAX_WORLD = 16
TEST_WAIT_BIT = 1 << 7


class TileConfig(ctypes.Structure):
    _fields_ = [
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("group_size_m", ctypes.c_int32),
        ("num_warps", ctypes.c_int32),
        ("num_stages", ctypes.c_int32),
        ("cta_multiplier", ctypes.c_int32),
    ]


class LaunchInfo(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_int32),
        ("swap_ab", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("tile_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("grid", ctypes.c_int32),
    ]

    def as_dict(self) -> dict[str, int | str]:
        return {
            "path": {0: "tcgen05_tma", 1: "simt_generic", 2: "tcgen05_tma_pair"}.get(int(self.path), "unknown"),
            "swap_ab": int(self.swap_ab),
            "tile_m": int(self.tile_m),
            "tile_n": int(self.tile_n),
            "tile_k": int(self.tile_k),
            "stages": int(self.stages),
            "grid": int(self.grid),
        }


class EpConfig(ctypes.Structure):
    """mgb_ep_config: one rank's view of an expert-parallel layer."""

    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("num_experts", ctypes.c_int32),
        ("elem_bytes", ctypes.c_int32),
        ("hidden", ctypes.c_int64),
        ("capacity", ctypes.c_int64),
        ("timeout_ns", ctypes.c_int64),
        ("max_slots", ctypes.c_int64),
    ]


class EpRegion(ctypes.Structure):
    """mgb_ep_region: byte offsets inside one rank's shared region."""

    _fields_ = [
        ("counts", ctypes.c_int64),
        ("send_base", ctypes.c_int64),
        ("recv_offs", ctypes.c_int64),
        ("recv", ctypes.c_int64),
        ("out", ctypes.c_int64),
        ("origin", ctypes.c_int64),
        ("ret", ctypes.c_int64),
        ("bytes", ctypes.c_int64),
    ]


class NativeLaunchError(RuntimeError):
    """A native launch returned a non-OK status."""


_lib = None
_load_error: str | None = None


def _declare(lib) -> None:
    c_i64p = ctypes.c_void_p
    lib.grouped_gemm_scratch_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32]
    lib.grouped_gemm_scratch_bytes.restype = ctypes.c_size_t
    lib.grouped_gemm_launch.argtypes = [
        c_i64p, c_i64p, c_i64p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.POINTER(TileConfig), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_launch.restype = ctypes.c_int
    lib.grouped_gemm_swiglu_launch.argtypes = [
        c_i64p, c_i64p, c_i64p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.POINTER(TileConfig), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_swiglu_launch.restype = ctypes.c_int
    lib.grouped_gemm_launch_noalloc.argtypes = [
        c_i64p, c_i64p, c_i64p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.POINTER(TileConfig), ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_launch_noalloc.restype = ctypes.c_int
    lib.grouped_gemm_offsets_launch.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(TileConfig), ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_offsets_launch.restype = ctypes.c_int
    lib.grouped_gemm_offsets_launch_ex.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(TileConfig),
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_offsets_launch_ex.restype = ctypes.c_int
    lib.moe_route_layout.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.moe_route_layout.restype = ctypes.c_int
    lib.moe_permute.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
                                ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p]
    lib.moe_permute.restype = ctypes.c_int
    lib.moe_combine.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.moe_combine.restype = ctypes.c_int
    lib.moe_ep_region_layout.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int32, ctypes.POINTER(EpRegion)]
    lib.moe_ep_region_layout.restype = ctypes.c_int
    lib.moe_ep_shared_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
    lib.moe_ep_shared_alloc.restype = ctypes.c_int
    lib.moe_ep_shared_free.argtypes = [ctypes.c_void_p]
    lib.moe_ep_shared_free.restype = ctypes.c_int
    lib.moe_ep_peer_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.moe_ep_peer_open.restype = ctypes.c_int
    lib.moe_ep_peer_close.argtypes = [ctypes.c_void_p]
    lib.moe_ep_peer_close.restype = ctypes.c_int
    lib.moe_ep_exchange_counts.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(EpConfig), ctypes.c_void_p]
    lib.moe_ep_exchange_counts.restype = ctypes.c_int
    lib.moe_ep_dispatch.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(EpConfig), ctypes.c_void_p]
    lib.moe_ep_dispatch.restype = ctypes.c_int
    lib.moe_ep_combine.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                                   ctypes.c_void_p, ctypes.POINTER(EpConfig), ctypes.c_int32, ctypes.c_void_p,
                                   ctypes.c_int64, ctypes.c_void_p]
    lib.grouped_gemm_offsets_scatter_launch.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
        ctypes.POINTER(TileConfig),
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_offsets_scatter_launch.restype = ctypes.c_int
    lib.moe_ep_combine.restype = ctypes.c_int
    lib.grouped_gemm_fp8_launch.argtypes = [
        c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(TileConfig), ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.grouped_gemm_fp8_launch.restype = ctypes.c_int
    lib.matmul_launch.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(TileConfig), ctypes.c_void_p, ctypes.POINTER(LaunchInfo),
    ]
    lib.matmul_launch.restype = ctypes.c_int
    lib.matrix_repack.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
    ]
    lib.matrix_repack.restype = ctypes.c_int
    lib.matrix_split_tf32x3.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
    ]
    lib.matrix_split_tf32x3.restype = ctypes.c_int
    lib.matrix_sum_partials.argtypes = [
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
    ]
    lib.matrix_sum_partials.restype = ctypes.c_int
    lib.read_and_clear_error_word.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32)]
    lib.read_and_clear_error_word.restype = ctypes.c_int
    lib.mgb_set_debug.argtypes = [ctypes.c_int64, ctypes.c_int32]
    lib.mgb_set_debug.restype = ctypes.c_int
    lib.mgb_status_string.argtypes = [ctypes.c_int32]
    lib.mgb_status_string.restype = ctypes.c_char_p
    lib.mgb_abi_version.argtypes = []
    lib.mgb_abi_version.restype = ctypes.c_int32


def load():
    """Load (once) and return the native library; raise RuntimeError when unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise RuntimeError(_load_error)
    if not LIBRARY_PATH.exists():
        _load_error = (
            f"native library {LIBRARY_PATH} is missing; build it with "
            "`make -C moe-gemm-parallel-bench_b200/csrc` (or __graft_entry__.build())"
        )
        raise RuntimeError(_load_error)
    try:
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        _declare(lib)
    except (OSError, AttributeError) as exc:
        _load_error = f"native library {LIBRARY_PATH} failed to load: {exc}"
        raise RuntimeError(_load_error) from exc
    _lib = lib
    return lib


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def status_text(status: int) -> str:
    return load().mgb_status_string(int(status)).decode()


def _check(status: int, what: str) -> None:
    if status != STATUS_OK:
        raise NativeLaunchError(f"{what} failed: {status_text(status)} (status {status})")


def tile_config(config) -> TileConfig:
    return TileConfig(
        int(config.block_m), int(config.block_n), int(config.block_k), int(config.group_size_m),
        int(config.num_warps), int(config.num_stages), int(config.cta_multiplier),
    )


def scratch_bytes(problem_count: int, sm_count: int) -> int:
    return int(load().grouped_gemm_scratch_bytes(int(problem_count), int(sm_count)))


def grouped_launch(
    a_ptrs: int, b_ptrs: int, c_ptrs: int, dims: int, strides: int, problem_count: int, homogeneous: bool,
    m: int, n: int, k: int, dtype: str, precision: str, tma_aligned: bool, config, scratch: int,
    scratch_nbytes: int, stream: int, swiglu: bool = False,
) -> LaunchInfo:
    """grouped_gemm_launch, or grouped_gemm_swiglu_launch with `swiglu`."""
    info = LaunchInfo()
    cfg = tile_config(config)
    lib = load()
    entry = lib.grouped_gemm_swiglu_launch if swiglu else lib.grouped_gemm_launch
    status = entry(
        a_ptrs, b_ptrs, c_ptrs, dims, strides, int(problem_count), int(bool(homogeneous)), int(m), int(n), int(k),
        DTYPE_CODES[dtype], PRECISION_CODES[precision], int(bool(tma_aligned)), ctypes.byref(cfg), scratch,
        int(scratch_nbytes), stream, ctypes.byref(info),
    )
    _check(status, "grouped_gemm_swiglu_launch" if swiglu else "grouped_gemm_launch")
    return info


def offsets_launch(
    a: int, b: int, c: int, offs: int, problem_count: int, total_rows: int, n: int, k: int, stride_am: int,
    stride_be: int, stride_bk: int, stride_cm: int, dtype: str, precision: str, swiglu: bool, config, scratch: int,
    scratch_nbytes: int, stream: int, b_count: int = 0,
) -> LaunchInfo:
    """grouped_gemm_offsets_launch_ex: the expert-sorted aggregate layout
    (segment e multiplies B[e % b_count] when b_count > 0)."""
    info = LaunchInfo()
    cfg = tile_config(config)
    status = load().grouped_gemm_offsets_launch_ex(
        a, b, c, offs, int(problem_count), int(b_count), int(total_rows), int(n), int(k), int(stride_am),
        int(stride_be), int(stride_bk), int(stride_cm), DTYPE_CODES[dtype], PRECISION_CODES[precision],
        int(bool(swiglu)), ctypes.byref(cfg), scratch, int(scratch_nbytes), stream, ctypes.byref(info),
    )
    _check(status, "grouped_gemm_offsets_launch_ex")
    return info


def route_layout(topk_ids: int, tokens: int, top_k: int, num_experts: int, counts: int, position: int,
                 stream: int) -> None:
    _check(load().moe_route_layout(topk_ids, int(tokens), int(top_k), int(num_experts), counts, position, stream),
           "moe_route_layout")


def permute(x: int, x_pitch: int, topk_ids: int, position: int, offsets: int, tokens: int, top_k: int,
            num_experts: int, hidden: int, sorted_rows: int, sorted_pitch: int, elem_bytes: int, stream: int) -> None:
    _check(load().moe_permute(x, int(x_pitch), topk_ids, position, offsets, int(tokens), int(top_k), int(num_experts),
                              int(hidden), sorted_rows, int(sorted_pitch), int(elem_bytes), stream), "moe_permute")


def combine(y: int, y_pitch: int, topk_ids: int, weights: int, position: int, offsets: int, tokens: int, top_k: int,
            num_experts: int, hidden: int, out: int, out_pitch: int, stream: int) -> None:
    _check(load().moe_combine(y, int(y_pitch), topk_ids, weights, position, offsets, int(tokens), int(top_k),
                              int(num_experts), int(hidden), out, int(out_pitch), stream), "moe_combine")


def ep_region_layout(world: int, num_experts: int, hidden: int, capacity: int, max_slots: int,
                     elem_bytes: int) -> EpRegion:
    region = EpRegion()
    _check(load().moe_ep_region_layout(int(world), int(num_experts), int(hidden), int(capacity), int(max_slots),
                                       int(elem_bytes), ctypes.byref(region)), "moe_ep_region_layout")
    return region


def ep_shared_alloc(nbytes: int, with_handle: bool = True) -> tuple[int, bytes]:
    """Zero-filled device region on the current device and its IPC handle
    (empty without ``with_handle``)."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(EP_HANDLE_BYTES) if with_handle else None
    _check(load().moe_ep_shared_alloc(int(nbytes), ctypes.byref(ptr), handle), "moe_ep_shared_alloc")
    return int(ptr.value), (handle.raw if with_handle else b"")


def ep_shared_free(ptr: int) -> None:
    _check(load().moe_ep_shared_free(ptr), "moe_ep_shared_free")


def ep_peer_open(handle: bytes) -> int:
    if len(handle) != EP_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {EP_HANDLE_BYTES} bytes, got {len(handle)}")
    ptr = ctypes.c_void_p()
    _check(load().moe_ep_peer_open(ctypes.create_string_buffer(handle, EP_HANDLE_BYTES), ctypes.byref(ptr)),
           "moe_ep_peer_open")
    return int(ptr.value)


def ep_peer_close(ptr: int) -> None:
    _check(load().moe_ep_peer_close(ptr), "moe_ep_peer_close")


def ep_exchange_counts(counts: int, peers: int, config: EpConfig, stream: int) -> None:
    _check(load().moe_ep_exchange_counts(counts, peers, ctypes.byref(config), stream), "moe_ep_exchange_counts")


def ep_dispatch(x: int, x_pitch: int, topk_ids: int, position: int, tokens: int, top_k: int, peers: int,
                config: EpConfig, stream: int) -> None:
    _check(load().moe_ep_dispatch(x, int(x_pitch), topk_ids, position, int(tokens), int(top_k), peers,
                                  ctypes.byref(config), stream), "moe_ep_dispatch")


def ep_combine(topk_ids: int, weights: int, position: int, tokens: int, top_k: int, peers: int, config: EpConfig,
               out: int, out_pitch: int, stream: int, returned: bool = False) -> None:
    _check(load().moe_ep_combine(topk_ids, weights, position, int(tokens), int(top_k), peers, ctypes.byref(config),
                                 int(bool(returned)), out, int(out_pitch), stream), "moe_ep_combine")


def offsets_scatter_launch(
    a: int, b: int, offs: int, problem_count: int, b_count: int, total_rows: int, n: int, k: int, stride_am: int,
    stride_be: int, stride_bk: int, row_origin: int, peers: int, peer_count: int, dst_offset: int,
    dst_pitch_bytes: int, dtype: str, precision: str, config, scratch: int, scratch_nbytes: int, stream: int,
) -> LaunchInfo:
    """grouped_gemm_offsets_scatter_launch: aggregate-layout GEMM whose rows
    are stored at per-row destinations (see the C header)."""
    info = LaunchInfo()
    cfg = tile_config(config)
    status = load().grouped_gemm_offsets_scatter_launch(
        a, b, offs, int(problem_count), int(b_count), int(total_rows), int(n), int(k), int(stride_am),
        int(stride_be), int(stride_bk), row_origin, peers, int(peer_count), int(dst_offset), int(dst_pitch_bytes),
        DTYPE_CODES[dtype], PRECISION_CODES[precision], ctypes.byref(cfg), scratch, int(scratch_nbytes), stream,
        ctypes.byref(info),
    )
    _check(status, "grouped_gemm_offsets_scatter_launch")
    return info


def fp8_launch(
    a_ptrs: int, b_ptrs: int, c_ptrs: int, sa_ptrs: int, sb_ptrs: int, dims: int, problem_count: int,
    homogeneous: bool, m: int, n: int, k: int, config, scratch: int, scratch_nbytes: int, stream: int,
) -> LaunchInfo:
    """grouped_gemm_fp8_launch: e4m3 A [M, K] / B [N, K] with fp32 block scales, bf16 C."""
    info = LaunchInfo()
    cfg = tile_config(config)
    status = load().grouped_gemm_fp8_launch(
        a_ptrs, b_ptrs, c_ptrs, sa_ptrs, sb_ptrs, dims, int(problem_count), int(bool(homogeneous)), int(m), int(n),
        int(k), ctypes.byref(cfg), scratch, int(scratch_nbytes), stream, ctypes.byref(info),
    )
    _check(status, "grouped_gemm_fp8_launch")
    return info


# Size of the library's fixed scratch array (MGB_NOALLOC_SCRATCH_BYTES in the header).
NOALLOC_SCRATCH_BYTES = 1 << 20


def grouped_launch_noalloc(
    a_ptrs: int, b_ptrs: int, c_ptrs: int, dims: int, strides: int, problem_count: int, homogeneous: bool,
    m: int, n: int, k: int, dtype: str, precision: str, tma_aligned: bool, config, stream: int,
) -> LaunchInfo:
    """grouped_gemm_launch_noalloc: the grouped launch for callers that cannot
    allocate device memory (a plugin whose host framework owns all device
    memory, a launch path that must not enter the driver's allocator): its
    tensor-map scratch is a fixed array inside the library.  The first call on
    a device looks the array up and must come before any stream capture;
    groups of more than 2674 problems are refused; calls that overlap on the
    GPU race on the shared array."""
    info = LaunchInfo()
    cfg = tile_config(config)
    status = load().grouped_gemm_launch_noalloc(
        a_ptrs, b_ptrs, c_ptrs, dims, strides, int(problem_count), int(bool(homogeneous)), int(m), int(n), int(k),
        DTYPE_CODES[dtype], PRECISION_CODES[precision], int(bool(tma_aligned)), ctypes.byref(cfg), stream,
        ctypes.byref(info),
    )
    _check(status, "grouped_gemm_launch_noalloc")
    return info


def matmul_launch(
    a: int, b: int, c: int, m: int, n: int, k: int, strides: tuple[int, ...], dtype: str, precision: str, config,
    stream: int,
) -> LaunchInfo:
    info = LaunchInfo()
    cfg = tile_config(config)
    status = load().matmul_launch(
        a, b, c, int(m), int(n), int(k), *(int(s) for s in strides), DTYPE_CODES[dtype], PRECISION_CODES[precision],
        ctypes.byref(cfg), stream, ctypes.byref(info),
    )
    _check(status, "matmul_launch")
    return info


def repack(src: int, rows: int, cols: int, stride_r: int, stride_c: int, dst: int, dst_pitch: int,
           elem_bytes: int, stream: int) -> None:
    """matrix_repack: copy a strided matrix into a row-pitched buffer."""
    _check(load().matrix_repack(src, int(rows), int(cols), int(stride_r), int(stride_c), dst, int(dst_pitch),
                                int(elem_bytes), stream), "matrix_repack")


def split_tf32x3(src: int, rows: int, cols: int, stride_r: int, stride_c: int, dst: int, dst_pitch: int,
                side: int, stream: int) -> None:
    """matrix_split_tf32x3: the 3xTF32 operand split of an fp32 matrix (side 0:
    A -> [hi | lo | hi] along its columns; side 1: B -> [hi; hi; lo] along its
    rows)."""
    _check(load().matrix_split_tf32x3(src, int(rows), int(cols), int(stride_r), int(stride_c), dst, int(dst_pitch),
                                      int(side), stream), "matrix_split_tf32x3")


def sum_partials(partials: int, splits: int, rows: int, cols: int, c: int, stride_cm: int, stride_cn: int,
                 dtype: str, stream: int) -> None:
    """matrix_sum_partials: C = sum over s of the fp32 partials [splits][rows][cols]
    of a split-K GEMM, rounded once to C's dtype."""
    _check(load().matrix_sum_partials(partials, int(splits), int(rows), int(cols), c, int(stride_cm), int(stride_cn),
                                      DTYPE_CODES[dtype], stream), "matrix_sum_partials")


def read_and_clear_error_word(device: int) -> int:
    word = ctypes.c_uint32(0)
    _check(load().read_and_clear_error_word(int(device), ctypes.byref(word)), "read_and_clear_error_word")
    return int(word.value)


def describe_error_word(word: int) -> list[str]:
    return [text for bit, text in ERROR_BITS.items() if word & bit]


def set_debug(wait_budget_cycles: int = 0, test_flags: int = 0) -> None:
    _check(load().mgb_set_debug(int(wait_budget_cycles), int(test_flags)), "mgb_set_debug")
