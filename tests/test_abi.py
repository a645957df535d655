"""The C-ABI library loads and exports every symbol include/*.h declares.

No compute calls here: these run without a GPU.  Only the pure host entry
points (status strings, scratch sizing, ABI version, debug knobs) are called.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from kernels import _native

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions() -> set[str]:
    names = set()
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for match in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", text, flags=re.M):
            name = match.group(1)
            if name not in {"if", "while", "for", "switch", "return", "sizeof"}:
                names.add(name)
    return names


def test_header_exists_and_declares_the_boundary():
    assert HEADERS, "include/*.h missing"
    names = declared_functions()
    assert {"grouped_gemm_launch", "matmul_launch", "read_and_clear_error_word"} <= names


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    names = declared_functions()
    assert names == set(_native.EXPORTED_SYMBOLS)
    for name in sorted(names):
        assert hasattr(lib, name), f"{name} not exported"
    exported = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIBRARY_PATH)], capture_output=True,
                              text=True, check=True).stdout
    for name in names:
        assert re.search(rf"\sT\s{name}$", exported, flags=re.M), f"{name} is not a defined text symbol"


def test_library_is_built_for_sm_100a_only():
    """The build recipe compiles every translation unit for sm_100a and nothing
    else (tcgen05 / TMA code has no other target); the GPU tests then show the
    tensor-core kernels running from this library."""
    makefile = (Path(_native.LIBRARY_PATH).parents[1] / "csrc" / "Makefile").read_text()
    arch = re.search(r"^ARCH\s*:=\s*(.+)$", makefile, flags=re.M)
    assert arch and arch.group(1).split() == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "$(ARCH)" in re.search(r"^NVFLAGS\s*:=.*$", makefile, flags=re.M).group(0)
    assert re.search(r"\$\(NVCC\) \$\(ARCH\) -shared", makefile)


def test_noalloc_size_matches_the_header():
    """The Python bound of the no-allocation entry point is the header's
    MGB_NOALLOC_SCRATCH_BYTES."""
    text = "\n".join(h.read_text() for h in HEADERS)
    match = re.search(r"#define\s+MGB_NOALLOC_SCRATCH_BYTES\s+\(1u\s*<<\s*(\d+)\)", text)
    assert match, "MGB_NOALLOC_SCRATCH_BYTES not found in include/*.h"
    assert _native.NOALLOC_SCRATCH_BYTES == 1 << int(match.group(1))


def test_host_only_entry_points():
    lib = _native.load()
    assert lib.mgb_abi_version() == 1
    assert _native.status_text(_native.STATUS_OK) == "ok"
    assert "scratch" in _native.status_text(_native.STATUS_SCRATCH)
    assert _native.status_text(99) == "unknown status"
    # A, B and C tensor maps of 128 bytes per problem, plus E + 1 int64 walk offsets.
    assert _native.scratch_bytes(256, 148) == 256 * 3 * 128 + 257 * 8
    assert _native.scratch_bytes(1, 0) == 3 * 128 + 2 * 8
    assert _native.scratch_bytes(0, 0) == 3 * 128 + 2 * 8
    assert _native.scratch_bytes(2674, 148) <= _native.NOALLOC_SCRATCH_BYTES < _native.scratch_bytes(2675, 148)
    _native.set_debug(1000, 1)
    _native.set_debug(0, 0)


def test_invalid_arguments_are_rejected_before_any_device_call():
    lib = _native.load()
    cfg = _native.TileConfig(16, 128, 64, 4, 4, 3, 1)
    info = _native.LaunchInfo()
    # null tables / non-positive problem count / bad dtype: MGB_ERR_INVALID without touching CUDA
    status = lib.grouped_gemm_launch(None, None, None, None, None, 0, 1, 1, 1, 1, 1, 0, 1, ctypes.byref(cfg), None,
                                     0, None, ctypes.byref(info))
    assert status == _native.STATUS_INVALID
    status = lib.grouped_gemm_launch(None, None, None, None, None, 4, 1, 1, 1, 1, 7, 0, 1, ctypes.byref(cfg), None,
                                     0, None, ctypes.byref(info))
    assert status == _native.STATUS_INVALID
    status = lib.matmul_launch(None, None, None, -1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0, ctypes.byref(cfg), None,
                               ctypes.byref(info))
    assert status == _native.STATUS_INVALID


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_native, "LIBRARY_PATH", tmp_path / "absent.so")
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "_load_error", None)
    with pytest.raises(RuntimeError, match="missing"):
        _native.load()
    assert not _native.available()


def test_expert_parallel_region_layout_is_aligned_and_validated():
    """moe_ep_region_layout is pure host arithmetic: sections in order, 256-byte
    (tables) / 1024-byte (row blocks) aligned, sized for the arguments; bad
    arguments are refused."""
    world, experts, hidden, capacity, slots = 4, 256, 7168, 131072, 32768
    r = _native.ep_region_layout(world, experts, hidden, capacity, slots, 2)
    assert 0 < r.counts < r.send_base < r.recv_offs < r.recv < r.out < r.origin < r.ret < r.bytes
    assert r.counts >= 3 * _native.EP_MAX_WORLD * 4  # the barrier flags sit in front of the tables
    assert r.send_base - r.counts >= 2 * world * experts * 4
    assert r.recv_offs - r.send_base >= experts * 4
    assert r.recv - r.recv_offs >= experts // world * 4
    assert r.out - r.recv >= capacity * hidden * 2 and r.origin - r.out >= capacity * hidden * 2
    assert r.ret - r.origin >= capacity * 8 and r.bytes - r.ret >= slots * hidden * 2
    for offset in (r.counts, r.send_base, r.recv_offs):
        assert offset % 256 == 0
    for offset in (r.recv, r.out, r.origin, r.ret, r.bytes):
        assert offset % 1024 == 0
    for bad in ((0, experts, hidden, capacity, slots, 2), (_native.EP_MAX_WORLD + 1, 256, 8, 8, 8, 2),
                (3, 256, hidden, capacity, slots, 2), (world, experts, 0, capacity, slots, 2),
                (world, experts, hidden, -1, slots, 2), (world, experts, hidden, capacity, -1, 2)):
        with pytest.raises(_native.NativeLaunchError, match="invalid argument"):
            _native.ep_region_layout(*bad)
