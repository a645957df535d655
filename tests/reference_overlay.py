"""A copy of the installed reference (baseline/_ref) with this package's
drop-in modules in place of its two Triton modules.

The reference's drivers import `kernels.grouped_gemm` and `kernels.matmul`
(benchmark_moe.py:12-18, benchmark_shapes.py:8-13, compare_grouped_gemm.py:14,
tests/test_gpu.py:11-17).  The overlay keeps every reference file and replaces
those two modules, adding their helpers and the native library, exactly as a
maintainer would install the drop-in.  The package
files are symlinked, not copied, so a process that loads the library maps the
in-tree libmoe_gemm_b200.so.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REFERENCE_INSTALL = ROOT / "baseline" / "_ref"
KERNELS = ROOT / "moe-gemm-parallel-bench_b200" / "kernels"
DROP_IN = ("grouped_gemm.py", "matmul.py", "_native.py", "_timing.py", "libmoe_gemm_b200.so")


def reference_installed() -> bool:
    return (REFERENCE_INSTALL / "benchmark_moe.py").exists() and (REFERENCE_INSTALL / "tests" / "test_gpu.py").exists()


def build_overlay(dest: Path) -> Path:
    """Copies baseline/_ref to dest/ref and links the drop-in files into its kernels/."""
    target = dest / "ref"
    shutil.copytree(REFERENCE_INSTALL, target, ignore=shutil.ignore_patterns("__pycache__", "*.dist-info"))
    for name in DROP_IN:
        source = KERNELS / name
        if not source.exists():
            raise FileNotFoundError(f"{source} is missing (build the native library first)")
        link = target / "kernels" / name
        if link.exists() or link.is_symlink():
            link.unlink()
        link.symlink_to(source)
    return target


def run_in_overlay(overlay: Path, args: list[str], timeout: int = 900) -> subprocess.CompletedProcess:
    """Runs `python <args>` with the overlay as working directory and only the
    overlay on the import path (the reference's own layout)."""
    env = dict(os.environ)
    env["PYTHONPATH"] = str(overlay)
    env.pop("PYTEST_ADDOPTS", None)
    return subprocess.run([sys.executable, *args], cwd=overlay, env=env, capture_output=True, text=True,
                          timeout=timeout)
