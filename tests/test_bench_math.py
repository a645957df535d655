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


MEASURED = {"bf16_tflops": 1694.4, "bf16_tflops_sustained": 1434.9, "hbm_gbs": 6468.3, "sm_max_mhz": 1965.0,
            "sustained_sm_mhz": 1380.0}


@pytest.mark.parametrize("mhz,expected,kind", [
    (1965.0, 1694.4, "burst"),        # a short region at boost clock: the burst figure
    (1890.0, 1694.4, "burst"),        # within 5% of the maximum
    (1380.0, 1434.9, "sustained"),    # at the clock the sustained figure was measured at
    (1222.0, 1434.9, "sustained"),    # below it (power-capped step)
    (None, 1694.4, "burst"),          # no clock record: the larger denominator
])
def test_tensor_peak_follows_the_sampled_clock(mhz, expected, kind):
    """The roofline's tensor peak is chosen from the SM clock sampled in the
    timed region, never the sustained figure alone for a boost-clock run."""
    bench = _bench()
    clocks = None if mhz is None else {"sm_mhz": mhz}
    peak, source = bench.tensor_peak(MEASURED, clocks)
    assert peak == pytest.approx(expected)
    assert source.startswith(kind)


def test_tensor_peak_interpolates_between_the_two_figures():
    bench = _bench()
    hi = 0.95 * MEASURED["sm_max_mhz"]
    mid = (hi + MEASURED["sustained_sm_mhz"]) / 2
    peak, source = bench.tensor_peak(MEASURED, {"sm_mhz": mid})
    assert peak == pytest.approx((1694.4 + 1434.9) / 2)
    assert source.startswith("interpolated")


def test_dominant_kernel_fraction_at_burst_clock_matches_the_record():
    """The round's driver record: W13 EP M_e = 1024 at 1.5852 ms with a
    1965 MHz median is 1213.8 TFLOP/s, 0.72 of the burst peak (not 0.846 of
    the sustained one)."""
    bench = _bench()
    from moe_parallel import gemm_flops

    achieved = gemm_flops(1024, 7168, 4096) * 32 / 1.5852e-3 / 1e12
    peak, _ = bench.tensor_peak(MEASURED, {"sm_mhz": 1965.0})
    assert achieved == pytest.approx(1213.8, rel=1e-3)
    assert achieved / peak == pytest.approx(0.716, abs=2e-3)


def test_clock_summary_counts_only_the_timed_region():
    bench = _bench()
    sw_cap, hw_slow = 0x4, 0x8
    samples = [(0.5, 1965.0, 1965.0, 300.0, 0)]  # before the region
    samples += [(1.0 + 0.01 * i, 1400.0 + i, 1965.0, 900.0, sw_cap if i % 2 else 0) for i in range(21)]
    samples += [(5.0, 600.0, 1965.0, 100.0, hw_slow)]  # after it
    rec = bench.summarize_clock_samples(samples, window=(1.0, 1.3), interval_s=0.005)
    assert rec["samples_in_timed_region"] == 21 and rec["samples"] == 21
    assert rec["sm_mhz"] == 1410.0 and rec["sm_mhz_min"] == 1400.0
    assert rec["reasons"] == ["sw_power_cap"] and rec["reason_samples"] == {"sw_power_cap": 10}
    assert rec["power_w_median"] == 900.0


def test_default_step_is_w13_hot_and_w2_rotating_cold():
    """The default line covers both projections the metric names: W13 hot
    and W2 in rotating-cold mode."""
    bench = _bench()
    args = bench.parse_args([])
    projections = bench.selected_projections(args)
    assert projections == ("W1", "W2")
    assert bench.cold_projections(args, projections) == ("W2",)
    text = bench.workload_text(projections, ("W2",))
    assert "one step = 28 grouped launches" in text and "rotating-cold" in text
    only_w13 = bench.parse_args(["--fp8"])
    assert bench.selected_projections(only_w13) == ("W1",)
    with pytest.raises(SystemExit):
        bench.selected_projections(bench.parse_args(["--fp8", "--projection", "W2"]))


@pytest.mark.parametrize("model,parallel,m,ep,tp", [
    # Mixtral-8x7B (E=8, H=4096, F=14336), T=4096 top-2 -> M_e = 1024; EP P=8 is one expert per rank
    ("mixtral-8x7b", 8, 1024, ("W1", 1, (1024, 4096, 28672)), ("W1", 8, (1024, 4096, 3584))),
    ("mixtral-8x7b", 2, 1024, ("W2", 4, (1024, 14336, 4096)), ("W2", 8, (1024, 7168, 4096))),
    # Qwen3-235B-A22B (E=128, H=4096, F=1536), P=8: T=256 -> M_e = 16
    ("qwen3-235b-a22b", 8, 16, ("W1", 16, (16, 4096, 3072)), ("W1", 128, (16, 4096, 384))),
    ("qwen3-235b-a22b", 8, 1024, ("W2", 16, (1024, 1536, 4096)), ("W2", 128, (1024, 192, 4096))),
])
def test_model_table_gives_the_reference_rank_shapes(model, parallel, m, ep, tp):
    """--model / --parallel-size switch the
    step to the reference's rank shapes for that model (utils/metrics.py:40-72)."""
    bench = _bench()
    try:
        bench.set_model(model, parallel)
        assert m in bench.M_VALUES
        for par, (projection, count, shape) in (("EP", ep), ("TP", tp)):
            (_, _, got, experts), = [s for s in bench.step_shapes([m], projection) if s[0] == par]
            assert (got, experts) == (shape, count)
        assert bench.MODELS[model]["label"] in bench.workload_line("W1")
    finally:
        bench.set_model("deepseek-v3", 8)
    with pytest.raises(SystemExit):
        bench.set_model("mixtral-8x7b", 16)  # 16 ranks cannot split 8 experts
    bench.set_model("deepseek-v3", 8)
