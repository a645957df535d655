"""The reference's own unchanged code, driving this package's kernels.

The drop-in keeps the call signatures of the reference's kernels/grouped_gemm.py
and kernels/matmul.py so that its drivers and tests run unchanged on the B200
kernels.  Each test builds an overlay of the installed reference
(baseline/_ref, pip-installed from the reference checkout) with this package's
modules and native library in place of the two Triton modules
(tests/reference_overlay.py), then runs the reference's code in it as a
subprocess:

* tests/test_cpu.py of the reference (CPU: tile heuristics, shape model,
  validation, model configs);
* tests/test_gpu.py of the reference, all of it (GPU);
* benchmark.py --experiment moe on DeepSeek-V3 shapes in hot and in
  rotating-cold mode (run_moe / _run_case, benchmark_moe.py:134-389: NaN
  poisoning, the cold tuner, assert_close, time_cuda) and the reference's
  validate_results over what it wrote;
* benchmark.py --experiment shapes and heatmap (benchmark_shapes._run_one,
  benchmark_shapes.py:65-297);
* compare_grouped_gemm.py on its default cases (run_case,
  compare_grouped_gemm.py:99-161).

The overlay is skipped only when baseline/_ref is absent.
"""

from __future__ import annotations

import csv
import json

import pytest

from tests.conftest import cuda_ready
from tests.reference_overlay import build_overlay, reference_installed, run_in_overlay

needs_reference = pytest.mark.skipif(not reference_installed(), reason="baseline/_ref (the installed reference) absent")

SCHEDULERS = {"single_problem_matmul", "homogeneous_persistent", "generic_persistent"}


@pytest.fixture(scope="module")
def overlay(tmp_path_factory):
    if not reference_installed():
        pytest.skip("baseline/_ref (the installed reference) absent")
    return build_overlay(tmp_path_factory.mktemp("reference_overlay"))


def _ok(proc, what: str) -> str:
    text = proc.stdout + proc.stderr
    assert proc.returncode == 0, f"{what} exited {proc.returncode}:\n{text[-4000:]}"
    return text


def _rows(path) -> list[dict]:
    with open(path, newline="", encoding="utf-8") as handle:
        return list(csv.DictReader(handle))


@needs_reference
def test_reference_cpu_tests_pass_on_the_drop_in(overlay):
    """The reference's whole CPU test file (heuristics, pools, shape model,
    validation, model configs) against this package's modules."""
    text = _ok(run_in_overlay(overlay, ["-m", "pytest", "-q", "-p", "no:cacheprovider", "tests/test_cpu.py"]),
               "reference tests/test_cpu.py")
    assert " passed" in text and " failed" not in text


@needs_reference
def test_overlay_imports_this_package():
    """The overlay's kernels.grouped_gemm is this package's module, and the
    reference's own torch and tutorial providers stay beside it."""
    import tempfile
    from pathlib import Path

    with tempfile.TemporaryDirectory() as tmp:
        ref = build_overlay(Path(tmp))
        probe = ("import kernels.grouped_gemm as g, kernels.matmul as m, kernels.torch_grouped_gemm as t; "
                 "print(g.__file__); print(hasattr(g, 'launch_grouped_mm')); print(t.__file__)")
        text = _ok(run_in_overlay(ref, ["-c", probe]), "import probe")
        lines = text.strip().splitlines()
        assert Path(lines[0]).resolve() == (Path(__file__).resolve().parents[1] / "moe-gemm-parallel-bench_b200" /
                                            "kernels" / "grouped_gemm.py")
        assert lines[1] == "True"
        assert Path(lines[2]).parent == ref / "kernels"


@needs_reference
@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_reference_gpu_tests_pass_on_the_drop_in(overlay):
    """All of the reference's GPU tests (tests/test_gpu.py: the official
    Triton tutorial comparison, odd shapes in every dtype, strided TF32,
    distinct pointers, homogeneous tails, multi-round persistence with guard
    bands, packed gate+up, one-problem dispatch, torch grouped_mm and graph
    replay) with this package in place of the reference's Triton modules."""
    text = _ok(run_in_overlay(overlay, ["-m", "pytest", "-q", "-p", "no:cacheprovider", "-rs", "tests/test_gpu.py"]),
               "reference tests/test_gpu.py")
    assert "12 passed" in text, text[-2000:]


def _moe_run(overlay, results, cache_mode: str):
    args = ["benchmark.py", "--experiment", "moe", "--dtype", "bf16", "--moe-ms", "16,256", "--warmup", "2",
            "--repeat", "5", "--target-timing-ms", "50", "--cache-mode", cache_mode, "--results-dir", str(results),
            "--plots-dir", str(results / "plots"), "--no-plots", "--torch-baseline"]
    return _ok(run_in_overlay(overlay, args, timeout=1500), f"benchmark.py --experiment moe ({cache_mode})")


@needs_reference
@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
@pytest.mark.parametrize("cache_mode", ["hot", "cold"])
def test_reference_moe_driver_runs_on_the_drop_in(overlay, tmp_path, cache_mode):
    """benchmark.py --experiment moe (DeepSeek-V3 defaults, P = 8, bf16,
    M_e in {16, 256}, with the torch grouped_mm provider beside it): every
    grouped row passes the reference's own correctness gate and timing, and
    its validate_results accepts the run."""
    results = tmp_path / "results"
    text = _moe_run(overlay, results, cache_mode)
    assert "Validation: PASS" in text
    for projection in ("w1", "w2"):
        rows = _rows(results / f"moe_{projection}.csv")
        grouped = [r for r in rows if r.get("mode") == "grouped"]
        assert len(grouped) == 4, rows  # EP and TP at two M_e values
        torch_rows = [r for r in rows if r.get("mode") == "torch"]
        assert len(torch_rows) == 4 and all(r["status"] in ("ok", "skipped") for r in torch_rows), torch_rows
        for row in grouped:
            assert row["status"] == "ok", row
            assert row["correct"].lower() == "true", row
            assert row["scheduler"] in SCHEDULERS, row
            assert float(row["tflops"]) > 0
    validation = json.loads((results / "validation.json").read_text())
    assert validation["valid"] is True


@needs_reference
@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_reference_shape_and_heatmap_drivers_run_on_the_drop_in(overlay, tmp_path):
    """benchmark.py --experiment shapes and heatmap: the masked single GEMM
    through launch_matmul with the reference's checker, beside torch.mm."""
    results = tmp_path / "results"
    args = ["benchmark.py", "--experiment", "shapes", "--dtype", "bf16", "--shape-ms", "16,128,1024",
            "--warmup", "2", "--repeat", "5", "--target-timing-ms", "50", "--results-dir", str(results),
            "--plots-dir", str(results / "plots"), "--no-plots"]
    text = _ok(run_in_overlay(overlay, args), "benchmark.py --experiment shapes")
    assert "Validation: PASS" in text
    rows = [r for r in _rows(results / "gemm_shape_sweep.csv") if r.get("provider") == "triton"]
    assert rows and all(r["status"] == "ok" and r["correct"].lower() == "true" for r in rows), rows
    heat = tmp_path / "heat"
    args = ["benchmark.py", "--experiment", "heatmap", "--dtype", "fp16", "--heatmap-ms", "1,17,128",
            "--heatmap-ns", "256,1000", "--heatmap-k", "1024", "--warmup", "2", "--repeat", "5",
            "--target-timing-ms", "50", "--results-dir", str(heat), "--plots-dir", str(heat / "plots"), "--no-plots"]
    text = _ok(run_in_overlay(overlay, args), "benchmark.py --experiment heatmap")
    assert "Validation: PASS" in text
    rows = [r for r in _rows(heat / "gemm_heatmap.csv") if r.get("provider") == "triton"]
    assert len(rows) == 6 and all(r["status"] == "ok" for r in rows), rows


@needs_reference
@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_reference_tutorial_comparison_runs_on_the_drop_in(overlay, tmp_path):
    """compare_grouped_gemm.py on its default cases (homogeneous,
    heterogeneous, persistent rounds): this package's launch_grouped against
    the official Triton tutorial grouped GEMM on identical inputs."""
    output = tmp_path / "comparison.json"
    args = ["compare_grouped_gemm.py", "--repeat", "5", "--warmup", "2", "--target-timing-ms", "50",
            "--output", str(output)]
    _ok(run_in_overlay(overlay, args), "compare_grouped_gemm.py")
    report = json.loads(output.read_text())
    assert report["status"] == "passed", json.dumps(report["cases"])[:2000]
    names = {case["case"]: case for case in report["cases"]}
    assert set(names) == {"homogeneous", "heterogeneous", "persistent_rounds"}
    for case in names.values():
        assert case["status"] == "ok" and case["correct"] is True, case
