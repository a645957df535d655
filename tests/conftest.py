"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs everywhere (oracle vs golden fixtures, host logic, ABI
exports, gloo multi-rank logic); `-m gpu` needs a CUDA device and runs the
parity tests through the native library.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_DIR = ROOT / "moe-gemm-parallel-bench_b200"
for path in (str(ROOT), str(PACKAGE_DIR)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the native sm_100a library")


def cuda_ready() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except ImportError:
        return False


@pytest.fixture(scope="session")
def golden_cases():
    from tests.golden_data import load_gemm_cases

    return load_gemm_cases()
