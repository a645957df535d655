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
PRECISION_CODES = {"ieee": 0, "tf32": 1}
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
    "grouped_gemm_fp8_launch",
    "grouped_gemm_launch_noalloc",
    "matmul_launch",
    "matrix_repack",
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
}
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
    scratch_nbytes: int, stream: int,
) -> LaunchInfo:
    """grouped_gemm_offsets_launch: the expert-sorted aggregate layout."""
    info = LaunchInfo()
    cfg = tile_config(config)
    status = load().grouped_gemm_offsets_launch(
        a, b, c, offs, int(problem_count), int(total_rows), int(n), int(k), int(stride_am), int(stride_be),
        int(stride_bk), int(stride_cm), DTYPE_CODES[dtype], PRECISION_CODES[precision], int(bool(swiglu)),
        ctypes.byref(cfg), scratch, int(scratch_nbytes), stream, ctypes.byref(info),
    )
    _check(status, "grouped_gemm_offsets_launch")
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
    allocate device memory (its scratch is a fixed array inside the library).
    The first call on a device must come before any stream capture; calls that
    overlap on the GPU race on the shared array."""
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


def read_and_clear_error_word(device: int) -> int:
    word = ctypes.c_uint32(0)
    _check(load().read_and_clear_error_word(int(device), ctypes.byref(word)), "read_and_clear_error_word")
    return int(word.value)


def describe_error_word(word: int) -> list[str]:
    return [text for bit, text in ERROR_BITS.items() if word & bit]


def set_debug(wait_budget_cycles: int = 0, test_flags: int = 0) -> None:
    _check(load().mgb_set_debug(int(wait_budget_cycles), int(test_flags)), "mgb_set_debug")
