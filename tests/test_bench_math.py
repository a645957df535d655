"""The benchmark's shape and roofline arithmetic, on CPU.

`bench.py` builds one step from the reference's EP/TP shape model
(utils/metrics.py:40-72) and scores every launch against the roofline of the
reference's ideal byte model (utils/metrics.py:9-16): time = max(FLOPs / tensor
peak, (A + B + C bytes) / HBM bandwidth).  These tests pin both against the
DeepSeek-V3 P = 8 figures at nominal B200 peaks (2250 TFLOP/s dense bf16,
8 TB/s), so the bench's per-shape fractions rest on the same arithmetic.
"""

from __future__ import annotations

import pytest

NOMINAL = {"bf16_tflops": 2250.0, "bf16_tflops_sustained": 2250.0, "hbm_gbs": 8000.0}


def _bench():
    import bench

    return bench


def test_step_shapes_follow_the_reference_shape_model():
    """One step is 14 launches; EP ranks hold 32 experts at full F, TP ranks all
    256 experts with F cut by 8 (the reference's tests/test_cpu.py:110-114)."""
    bench = _bench()
    w13 = bench.step_shapes(bench.M_VALUES, "W1")
    w2 = bench.step_shapes(bench.M_VALUES, "W2")
    assert len(w13) == len(w2) == 14
    for m in bench.M_VALUES:
        assert ("EP", m, (m, 7168, 4096), 32) in w13
        assert ("TP", m, (m, 7168, 512), 256) in w13
        assert ("EP", m, (m, 2048, 7168), 32) in w2
        assert ("TP", m, (m, 256, 7168), 256) in w2


@pytest.mark.parametrize("projection,par,m,tflops,bound", [
    ("W1", "EP", 16, 127, "hbm"),
    ("W1", "EP", 64, 500, "hbm"),
    ("W1", "EP", 128, 976, "hbm"),
    ("W1", "EP", 256, 1865, "hbm"),
    ("W1", "EP", 512, 2250, "tensor"),
    ("W1", "EP", 1024, 2250, "tensor"),
    ("W1", "TP", 16, 124, "hbm"),
    ("W1", "TP", 1024, 2250, "tensor"),
    ("W2", "EP", 16, 127, "hbm"),
    ("W2", "TP", 16, 120, "hbm"),
    ("W2", "TP", 1024, 1593, "hbm"),
])
def test_roofline_per_launch_at_nominal_peaks(projection, par, m, tflops, bound):
    """Roofline TFLOP/s of one rank launch = FLOPs / max(compute time, byte time)."""
    bench = _bench()
    from moe_parallel import gemm_flops

    (_, _, (mm, k, n), count), = [s for s in bench.step_shapes([m], projection) if s[0] == par]
    ms, got_bound = bench.roofline_ms(mm, k, n, count, NOMINAL)
    achieved = gemm_flops(mm, k, n) * count / (ms * 1e-3) / 1e12
    assert got_bound == bound
    assert achieved == pytest.approx(tflops, rel=5e-3)


@pytest.mark.parametrize("projection,par,m,megabytes", [
    ("W1", "EP", 16, 1891), ("W1", "TP", 1024, 5906), ("W2", "EP", 16, 949), ("W2", "TP", 1024, 4832),
])
def test_ideal_bytes_per_launch(projection, par, m, megabytes):
    """Weights + input + output activations once, bf16 (utils/metrics.py:13-16)."""
    bench = _bench()
    from moe_parallel import ideal_bytes

    (_, _, (mm, k, n), count), = [s for s in bench.step_shapes([m], projection) if s[0] == par]
    assert ideal_bytes(mm, k, n, 2) * count / 1e6 == pytest.approx(megabytes, rel=2e-3)


def test_fused_swiglu_and_fp8_byte_models():
    """SwiGLU writes N/2 output columns; FP8 reads one byte per operand element
    plus fp32 block scales and writes bf16."""
    bench = _bench()
    m, k, n = 64, 7168, 4096
    full, _ = bench.roofline_ms(m, k, n, 1, NOMINAL)
    half, _ = bench.roofline_ms(m, k, n, 1, NOMINAL, out_cols=n // 2)
    assert half < full
    assert bench.fp8_launch_bytes(m, k, n) == m * k + n * k + 4 * (m * 56 + 32 * 56) + 2 * m * n
    fp8, bound = bench.roofline_ms(m, k, n, 1, NOMINAL, fp8=True)
    assert bound == "hbm" and fp8 < full


def test_reference_arm_prints_the_contract_line(capsys):
    """`bench.py --impl reference` times the reference's per-expert
    torch.matmul on the host and prints one JSON line with the arm's keys."""
    import json

    bench = _bench()
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "3", "--m-values", "16"]) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "TFLOP/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
