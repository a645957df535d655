"""GPU parity of the native kernels against the oracle and the reference's outputs.

Every launch goes through the C ABI (kernels -> ctypes -> libmoe_gemm_b200.so).
Cases follow the reference's own GPU tests (tests/test_gpu.py in the
reference, cited per test) plus the golden outputs of the reference's Triton
kernels and DeepSeek-V3-shaped groups.

Tolerances (written here, applied per case):
* relative Frobenius error vs the float64 oracle: bf16 <= 1e-2 (the target's
  bound), fp16 <= 2e-3, fp32 "ieee" <= 1e-5, fp32 "tf32" <= 5e-3;
* the reference's assert_close (utils/benchmark.py:261-271): fp16 2e-2,
  bf16 5e-2, fp32 2e-3 (rtol = atol);
* exact-integer cases: bit-exact.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from tests.conftest import cuda_ready

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")]

REL_FRO = {"bf16": 1e-2, "fp16": 2e-3, "fp32": 1e-5, "tf32": 5e-3}
ASSERT_CLOSE = {"fp16": 2e-2, "bf16": 5e-2, "fp32": 2e-3}


def _torch():
    import torch

    return torch


def _dtype(name):
    torch = _torch()
    return {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[name]


def _host(t) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def _oracle_check(c, a, b, dtype: str, precision: str = "ieee", gate_up: bool = False):
    from oracle import gemm as oracle

    a64, b64 = _host(a), _host(b)
    expected = oracle.gate_up(a64, b64, dtype) if gate_up else oracle.matmul(a64, b64, dtype)
    got = _host(c)
    assert np.isfinite(got).all(), "output has non-finite values (unwritten or overflow)"
    key = "tf32" if (dtype == "fp32" and precision == "tf32") else dtype
    err = oracle.relative_frobenius(got, expected)
    assert err <= REL_FRO[key], f"relative Frobenius error {err:.3e} > {REL_FRO[key]:.1e}"
    tol = ASSERT_CLOSE[dtype]
    np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)
    return err


def _randn(shape, dtype, gen, scale=0.1):
    torch = _torch()
    return (torch.randn(shape, device="cuda", generator=gen) * scale).to(dtype)


def _workspace(shapes, dtype_name, seed, b_scale=None):
    """Seeded per-expert tensors (A ~ N(0,1)*0.1 unless b_scale given: then
    A ~ N(0,1) and B ~ N(0, b_scale)) wrapped into a grouped workspace."""
    torch = _torch()
    from kernels import workspace_from_tensors

    gen = torch.Generator(device="cuda").manual_seed(seed)
    dtype = _dtype(dtype_name)
    a_list, b_list, c_list = [], [], []
    for m, k, n in shapes:
        if b_scale is None:
            a_list.append(_randn((m, k), dtype, gen))
            b_list.append(_randn((k, n), dtype, gen))
        else:
            a_list.append(_randn((m, k), dtype, gen, 1.0))
            b_list.append(_randn((k, n), dtype, gen, b_scale))
        c_list.append(torch.full((m, n), float("nan"), device="cuda", dtype=dtype))
    return workspace_from_tensors(a_list, b_list, c_list)


def _poison(workspace):
    for c in workspace.c:
        c.fill_(float("nan"))


# --------------------------------------------------------------- plumbing
def test_native_library_is_loaded_and_tensor_core_path_runs():
    """The parity below must come from the native library, not a fallback."""
    torch = _torch()
    from kernels import KernelConfig, check_device_errors, launch_grouped

    ws = _workspace([(16, 256, 256)] * 2, "bf16", seed=1)
    launch_grouped(ws, config=KernelConfig(16, 128, 64, 1, 4, 3), autotune=False)
    torch.cuda.synchronize()
    maps = open("/proc/self/maps").read()
    assert "libmoe_gemm_b200.so" in maps
    assert ws.launch_info["path"].startswith("tcgen05_tma")
    assert ws.launch_info["swap_ab"] == 1
    check_device_errors()
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, "bf16")


# ------------------------------------------------------- golden fixtures
def test_golden_reference_outputs(golden_cases):
    """Native outputs vs the reference's Triton outputs (interpreter-generated)
    and vs the oracle, on the same inputs."""
    torch = _torch()
    from kernels import KernelConfig, check_device_errors, launch_grouped, launch_matmul, workspace_from_tensors

    configs = (KernelConfig(16, 128, 64, 4, 4, 3), KernelConfig(64, 256, 64, 8, 8, 4), KernelConfig(128, 128, 64, 8, 8, 4))
    for case in golden_cases:
        dtype = case["dtype"]
        tol = 2e-3 if dtype == "fp16" else 1e-4
        if case["kind"] == "single_strided":
            a_base = torch.from_numpy(case["a_base"]).cuda()
            b_base = torch.from_numpy(case["b_base"]).cuda()
            c_base = torch.full_like(torch.from_numpy(case["c_base"]).cuda(), float("nan"))
            a, b, c = a_base[:, ::2], b_base[:, ::2], c_base[:, ::2]
            launch_matmul(a, b, c, input_precision="tf32")
            torch.cuda.synchronize()
            expected = torch.from_numpy(case["c_base"])[:, ::2].numpy()
            np.testing.assert_allclose(_host(c), expected, rtol=2e-3, atol=2e-3)
            assert torch.isnan(c_base[:, 1::2]).all(), "strided C: untouched columns were written"
            continue
        a_list = [torch.from_numpy(x).cuda() for x in case["a"]]
        b_list = [torch.from_numpy(x).cuda() for x in case["b"]]
        if case["kind"] == "single":
            c = torch.full((a_list[0].shape[0], b_list[0].shape[1]), float("nan"), device="cuda",
                           dtype=a_list[0].dtype)
            launch_matmul(a_list[0], b_list[0], c, autotune=False)
            torch.cuda.synchronize()
            np.testing.assert_allclose(_host(c), case["c"][0].astype(np.float64), rtol=tol, atol=tol,
                                       err_msg=case["name"])
            continue
        c_list = [torch.empty((a.shape[0], b.shape[1]), device="cuda", dtype=a.dtype) for a, b in zip(a_list, b_list)]
        ws = workspace_from_tensors(a_list, b_list, c_list)
        for cfg in configs:
            _poison(ws)
            launch_grouped(ws, config=cfg, autotune=False)
            torch.cuda.synchronize()
            for e, (a, b, c) in enumerate(ws.problem_tensors()):
                np.testing.assert_allclose(_host(c), case["c"][e].astype(np.float64), rtol=tol, atol=tol,
                                           err_msg=f"{case['name']} problem {e} config {cfg}")
                _oracle_check(c, a, b, dtype, gate_up=case["kind"] == "gate_up")
    check_device_errors()


# ------------------------------------------------ reference test_gpu ports
def test_project_shapes_fp16_vs_fp32_reference():
    """tests/test_gpu.py:34-52: fp16 groups vs an fp32 reference at 2e-3."""
    torch = _torch()
    from kernels import KernelConfig, build_grouped_workspace, launch_grouped

    for shapes in ([(128, 256, 128)] * 3, [(128, 128, 128), (256, 64, 256)]):
        ws = build_grouped_workspace(shapes, torch.float16, seed=123)
        for cfg in (KernelConfig(128, 128, 32, 1, 4, 3), KernelConfig(64, 64, 32, 1, 4, 3),
                    KernelConfig(128, 128, 64, 1, 4, 3), KernelConfig(64, 128, 64, 1, 4, 3)):
            _poison(ws)
            launch_grouped(ws, config=cfg, autotune=False)
            torch.cuda.synchronize()
            for a, b, c in ws.problem_tensors():
                reference = (a.float() @ b.float()).half()
                torch.testing.assert_close(c, reference, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16", "fp32"])
def test_single_odd_shapes_all_dtypes(dtype_name):
    """tests/test_gpu.py:69-86."""
    torch = _torch()
    from kernels import last_matmul_config, launch_matmul, select_config

    gen = torch.Generator(device="cuda").manual_seed(7)
    for m, k, n in ((1, 5, 3), (17, 13, 31), (33, 70, 65), (64, 128, 256), (200, 320, 136)):
        a = _randn((m, k), _dtype(dtype_name), gen)
        b = _randn((k, n), _dtype(dtype_name), gen)
        c = torch.full((m, n), float("nan"), device="cuda", dtype=_dtype(dtype_name))
        fallback = select_config(m, n, k)
        launch_matmul(a, b, c, fallback)
        torch.cuda.synchronize()
        selected = last_matmul_config(fallback)
        assert selected.block_m in (16, 32, 64, 128, 256)
        assert selected.block_n in (32, 64, 128, 256)
        assert selected.block_k in (32, 64, 128)
        _oracle_check(c, a, b, dtype_name)


def test_single_strided_fp32_tf32():
    """tests/test_gpu.py:88-97: strided views, TF32 requested."""
    torch = _torch()
    from kernels import launch_matmul

    gen = torch.Generator(device="cuda").manual_seed(8)
    m, k, n = 17, 70, 65
    a = _randn((m, k * 2), torch.float32, gen)[:, ::2]
    b = _randn((k, n * 2), torch.float32, gen)[:, ::2]
    storage = torch.full((m, n * 2), float("nan"), device="cuda")
    c = storage[:, ::2]
    launch_matmul(a, b, c, input_precision="tf32")
    torch.cuda.synchronize()
    _oracle_check(c, a, b, "fp32", "tf32")
    assert torch.isnan(storage[:, 1::2]).all()


def test_fp32_tf32_tensor_core_path():
    """TMA-aligned fp32 with TF32 runs tcgen05 kind::tf32, both orientations."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped

    ws = _workspace([(40, 256, 384), (40, 256, 384), (40, 256, 384)], "fp32", seed=9)
    for cfg in (KernelConfig(32, 128, 32, 4, 4, 3), KernelConfig(128, 256, 64, 8, 8, 4)):
        _poison(ws)
        launch_grouped(ws, "tf32", cfg, autotune=False)
        torch.cuda.synchronize()
        assert ws.launch_info["path"].startswith("tcgen05_tma")
        for a, b, c in ws.problem_tensors():
            _oracle_check(c, a, b, "fp32", "tf32")


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16", "fp32"])
def test_grouped_distinct_pointers_shapes_and_dtypes(dtype_name):
    """tests/test_gpu.py:99-115: heterogeneous problems -> generic scheduler."""
    torch = _torch()
    from kernels import build_grouped_workspace, launch_grouped, select_config

    shapes = [(1, 5, 3), (17, 13, 31), (9, 70, 65)]
    ws = build_grouped_workspace(shapes, _dtype(dtype_name), seed=99, config=select_config(17, 65, 70))
    assert len({x.data_ptr() for x in ws.a}) == len(shapes)
    launch_grouped(ws)
    torch.cuda.synchronize()
    assert ws.scheduler == "generic_persistent"
    assert ws.config.block_k in (32, 64, 128)
    assert ws.config.num_warps in (2, 4, 8)
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, dtype_name)


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16"])
def test_grouped_heterogeneous_tma_aligned(dtype_name):
    """Heterogeneous but TMA-legal problems: per-problem tensor maps rebuilt on the device."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped

    shapes = [(16, 128, 128), (40, 192, 256), (130, 64, 384), (1, 320, 64), (77, 256, 128)]
    ws = _workspace(shapes, dtype_name, seed=5)
    assert not ws.homogeneous
    for cfg in (KernelConfig(16, 128, 64, 4, 4, 3), KernelConfig(32, 256, 64, 4, 8, 4),
                KernelConfig(64, 128, 64, 8, 4, 4), KernelConfig(128, 64, 64, 8, 4, 3),
                KernelConfig(128, 256, 64, 8, 8, 4), KernelConfig(256, 128, 64, 8, 8, 4),
                KernelConfig(256, 256, 64, 8, 8, 4)):
        _poison(ws)
        launch_grouped(ws, config=cfg, autotune=False)
        torch.cuda.synchronize()
        assert ws.launch_info["path"].startswith("tcgen05_tma"), ws.launch_info
        assert ws.scheduler == "generic_persistent"
        for a, b, c in ws.problem_tensors():
            _oracle_check(c, a, b, dtype_name)


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16"])
def test_pair_tiles_on_ragged_problems(dtype_name):
    """CTA-pair tiles (256 x 256 and 256 x 512) where M, N and K end inside a
    tile: partial M blocks, a K tail shorter than one 64-wide k-block, an N
    block holding 8 valid columns, and a one-row problem."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped

    shapes = [(300, 320, 520), (513, 128, 1024), (1, 64, 512), (256, 72, 264)]
    ws = _workspace(shapes, dtype_name, seed=11)
    for cfg in (KernelConfig(256, 128, 64, 8, 8, 4), KernelConfig(256, 256, 64, 8, 8, 4)):
        _poison(ws)
        launch_grouped(ws, config=cfg, autotune=False)
        torch.cuda.synchronize()
        assert ws.launch_info["path"] == "tcgen05_tma_pair", ws.launch_info
        assert ws.launch_info["tile_n"] == (512 if cfg.block_n == 256 else 256)
        for a, b, c in ws.problem_tensors():
            _oracle_check(c, a, b, dtype_name)


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16"])
@pytest.mark.parametrize("m,k,n", [(256, 320, 512), (200, 200, 384), (256, 128, 1536)])
def test_wide_pair_tile_splits_a_short_last_wave(dtype_name, m, k, n):
    """256 x 512 pair tiles on a homogeneous group whose last wave holds at
    most half as many tiles as the device has clusters: each of those tiles
    runs as two 256-column half items, one per cluster, and the launch uses
    every cluster.  Ragged cases: M, K inside a block, and N = 384, whose
    second half item holds 128 valid columns."""
    torch = _torch()
    from kernels import KernelConfig, check_device_errors, launch_grouped

    clusters = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count // 2
    n_blocks = -(-n // 512)
    tail = max(1, clusters // 4)
    problems = -(-(clusters + tail) // n_blocks)
    tiles = problems * n_blocks
    assert 0 < tiles % clusters <= clusters // 2
    ws = _workspace([(m, k, n)] * problems, dtype_name, seed=21 + n)
    assert ws.homogeneous
    launch_grouped(ws, config=KernelConfig(256, 256, 64, 8, 8, 4), autotune=False)
    torch.cuda.synchronize()
    check_device_errors()
    assert ws.launch_info["path"] == "tcgen05_tma_pair" and ws.launch_info["tile_n"] == 512, ws.launch_info
    assert ws.launch_info["grid"] == 2 * clusters, ws.launch_info
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, dtype_name)


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16"])
def test_wide_pair_tile_split_single_gemm(dtype_name):
    """One masked GEMM on the 256 x 512 pair tile whose tile count leaves a
    short last wave (half items), M ending inside a block."""
    torch = _torch()
    from kernels import KernelConfig, launch_matmul

    clusters = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count // 2
    m_blocks = 3
    n_blocks = -(-(clusters + max(1, clusters // 8)) // m_blocks)
    m, k, n = 256 * m_blocks - 40, 192, 512 * n_blocks
    gen = torch.Generator(device="cuda").manual_seed(5)
    a = _randn((m, k), _dtype(dtype_name), gen)
    b = _randn((k, n), _dtype(dtype_name), gen)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=_dtype(dtype_name))
    launch_matmul(a, b, c, config=KernelConfig(256, 256, 64, 8, 8, 4), autotune=False)
    torch.cuda.synchronize()
    _oracle_check(c, a, b, dtype_name)


def test_grouped_homogeneous_persistent_fast_path():
    """tests/test_gpu.py:117-125."""
    torch = _torch()
    from kernels import build_grouped_workspace, launch_grouped

    ws = build_grouped_workspace([(17, 13, 31)] * 3, torch.float16, seed=101)
    assert ws.homogeneous
    launch_grouped(ws)
    torch.cuda.synchronize()
    assert ws.scheduler == "homogeneous_persistent"
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, "fp16")


@pytest.mark.parametrize("shape", [(1, 1, 1), (17, 33, 65), (33, 64, 136), (130, 128, 256)])
def test_homogeneous_tail_candidates_write_every_output(shape):
    """tests/test_gpu.py:127-154: exact integers for every candidate config."""
    torch = _torch()
    from kernels import build_grouped_workspace, grouped_candidate_configs, launch_grouped

    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        ws = build_grouped_workspace([shape] * 3, dtype)
        for index, (a, b, _) in enumerate(ws.problem_tensors()):
            a.fill_(1)
            b.fill_(index + 1)
        m, k, n = shape
        candidates = grouped_candidate_configs(m, n, k, problem_count=3, sm_count=ws.sm_count)
        assert candidates
        for config in candidates:
            _poison(ws)
            launch_grouped(ws, config=config, autotune=False)
            torch.cuda.synchronize()
            for index, output in enumerate(ws.c):
                torch.testing.assert_close(output, torch.full_like(output, k * (index + 1)), rtol=0, atol=0)


@pytest.mark.parametrize("dtype_name,k,n", [("fp32", 33, 65), ("bf16", 64, 136), ("fp16", 192, 64)])
def test_homogeneous_multiple_rounds_and_guard_storage(dtype_name, k, n):
    """tests/test_gpu.py:156-174: > one persistent round, C swapped after build
    (including c_ptrs), NaN guard bands around every C must survive."""
    torch = _torch()
    from kernels import KernelConfig, build_grouped_workspace, launch_grouped

    config = KernelConfig(16, 32, 32, 4, 4, 2)
    sm_count = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    m = (sm_count + 1) * config.block_m + 1
    ws = build_grouped_workspace([(m, k, n)] * 2, _dtype(dtype_name))
    guards = []
    for index in range(ws.problem_count):
        storage = torch.full((m * n + 32,), float("nan"), device="cuda", dtype=_dtype(dtype_name))
        output = storage[16:-16].view(m, n)
        guards.append(storage)
        ws.c[index] = output
        ws.c_ptrs[index] = output.data_ptr()
    for cfg in (config, KernelConfig(128, 128, 64, 8, 8, 4), KernelConfig(256, 128, 64, 8, 8, 4),
                KernelConfig(256, 256, 64, 8, 8, 4)):
        for c in ws.c:
            c.fill_(float("nan"))
        launch_grouped(ws, config=cfg, autotune=False)
        torch.cuda.synchronize()
        for (a, b, c), storage in zip(ws.problem_tensors(), guards):
            if dtype_name == "fp32":
                reference = (a.double() @ b.double()).float()
                torch.testing.assert_close(c, reference, rtol=1e-4, atol=1e-6)
            else:
                _oracle_check(c, a, b, dtype_name)
            assert torch.isnan(storage[:16]).all()
            assert torch.isnan(storage[-16:]).all()


def test_fused_gate_up_packed_output_in_one_grouped_launch():
    """tests/test_gpu.py:176-188 (plus a TMA-aligned bf16 W13 miniature)."""
    torch = _torch()
    from kernels import build_fused_gate_up_workspace, launch_grouped

    for dtype_name, shapes in (("fp16", [(17, 13, 62)] * 3), ("bf16", [(24, 256, 512)] * 3)):
        ws = build_fused_gate_up_workspace(shapes, _dtype(dtype_name), seed=102)
        assert ws.operation == "gate_up"
        launch_grouped(ws)
        torch.cuda.synchronize()
        assert ws.scheduler == "homogeneous_persistent"
        for a, packed_weight, packed_output in ws.problem_tensors():
            _oracle_check(packed_output, a, packed_weight, dtype_name, gate_up=True)


def _swiglu_check(ws, dtype_name, rows=None, precision="ieee"):
    from oracle import gemm as oracle

    for a, b, c in ws.problem_tensors():
        if rows is not None:
            idx = rows(a.shape[0])
            a, c = a.index_select(0, idx), c.index_select(0, idx)
        expected = oracle.swiglu(_host(a), _host(b), dtype_name)
        got = _host(c)
        assert np.isfinite(got).all(), "output has non-finite values (unwritten or overflow)"
        key = "tf32" if (dtype_name == "fp32" and precision == "tf32") else dtype_name
        err = oracle.relative_frobenius(got, expected)
        assert err <= REL_FRO[key], f"relative Frobenius error {err:.3e} > {REL_FRO[key]:.1e}"
        tol = ASSERT_CLOSE[dtype_name] if key != "tf32" else 5e-3
        np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)


def _swiglu_workspace(shapes, dtype_name, seed, b_scale=None):
    """Per-expert A, packed [gate | up] B and [M, N/2] C for the fused epilogue."""
    torch = _torch()
    from kernels import workspace_from_tensors

    gen = torch.Generator(device="cuda").manual_seed(seed)
    dtype = _dtype(dtype_name)
    a_list, b_list, c_list = [], [], []
    for m, k, n in shapes:
        scale_a, scale_b = (0.1, 0.1) if b_scale is None else (1.0, b_scale)
        a_list.append(_randn((m, k), dtype, gen, scale_a))
        b_list.append(_randn((k, n), dtype, gen, scale_b))
        c_list.append(torch.full((m, n // 2), float("nan"), device="cuda", dtype=dtype))
    return workspace_from_tensors(a_list, b_list, c_list, swiglu=True)


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16"])
def test_fused_swiglu_every_tile_family(dtype_name):
    """silu(A B_gate) * (A B_up) written as [M, F] in one launch: every native
    tile family (swap-AB, 128-row, CTA-pair 256 x 256 and 256 x 512) on a
    heterogeneous group with ragged M and F, against the float64 oracle."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped

    shapes = [(16, 256, 2 * 256), (40, 192, 2 * 136), (130, 320, 2 * 512), (1, 64, 2 * 64), (300, 128, 2 * 520)]
    ws = _swiglu_workspace(shapes, dtype_name, seed=21)
    assert ws.operation == "swiglu" and not ws.homogeneous
    for cfg in (KernelConfig(16, 256, 64, 4, 8, 4), KernelConfig(32, 128, 64, 4, 4, 4),
                KernelConfig(64, 256, 64, 8, 8, 4), KernelConfig(128, 64, 64, 8, 4, 3),
                KernelConfig(128, 256, 64, 8, 8, 4), KernelConfig(256, 128, 64, 8, 8, 4),
                KernelConfig(256, 256, 64, 8, 8, 4)):
        _poison(ws)
        launch_grouped(ws, config=cfg, autotune=False)
        torch.cuda.synchronize()
        assert ws.launch_info["path"].startswith("tcgen05_tma"), ws.launch_info
        _swiglu_check(ws, dtype_name)


@pytest.mark.parametrize("m_e", [16, 128, 1024])
def test_fused_swiglu_deepseek_tp_rank(m_e):
    """DeepSeek-V3 W13 TP rank miniature (4 experts of [M_e, 7168] @ [7168, 512]),
    autotuned launch, A ~ N(0,1), B ~ N(0, 1/sqrt(K)); sampled rows."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped

    ws = _swiglu_workspace([(m_e, 7168, 512)] * 4, "bf16", seed=m_e, b_scale=1.0 / math.sqrt(7168))
    assert ws.homogeneous
    launch_grouped(ws)
    torch.cuda.synchronize()
    check_device_errors()
    rng = np.random.default_rng(m_e)
    rows = lambda m: torch.as_tensor(np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, 16)])), device="cuda")
    _swiglu_check(ws, "bf16", rows=rows)


def test_fused_swiglu_tf32_and_builder():
    """fp32 operands on the TF32 tensor-core path, and the seeded builder."""
    torch = _torch()
    from kernels import build_fused_swiglu_workspace, launch_grouped

    ws = build_fused_swiglu_workspace([(96, 128, 2 * 192)] * 3, torch.float32, seed=4)
    launch_grouped(ws, input_precision="tf32")
    torch.cuda.synchronize()
    assert ws.launch_info["path"].startswith("tcgen05_tma")
    _swiglu_check(ws, "fp32", precision="tf32")
    ws16 = build_fused_swiglu_workspace([(64, 256, 2 * 128)], torch.bfloat16, seed=5)
    launch_grouped(ws16)  # one problem still takes the fused grouped path
    torch.cuda.synchronize()
    assert ws16.scheduler == "homogeneous_persistent"
    _swiglu_check(ws16, "bf16")


def test_fused_swiglu_refuses_the_generic_path():
    torch = _torch()
    from kernels import launch_grouped
    from kernels._native import NativeLaunchError

    ws = _swiglu_workspace([(8, 13, 2 * 16)] * 2, "bf16", seed=1)  # 26-byte A rows: not TMA-addressable
    with pytest.raises(NativeLaunchError, match="unsupported"):
        launch_grouped(ws)
    ws32 = _swiglu_workspace([(8, 64, 2 * 64)] * 2, "fp32", seed=1)  # fp32 "ieee" runs on the SIMT kernel
    with pytest.raises(NativeLaunchError, match="unsupported"):
        launch_grouped(ws32)


# ------------------------------------------- expert-sorted aggregate layout
def _aggregate(sizes, k, n, dtype_name, seed, pad=0, b_scale=0.1):
    """mat_a [T, K] (row pitch K + pad), mat_b [E, K, N] (row pitch N + pad), int32 offs."""
    torch = _torch()
    gen = torch.Generator(device="cuda").manual_seed(seed)
    dtype = _dtype(dtype_name)
    total = int(sum(sizes))
    mat_a = _randn((total, k + pad), dtype, gen, 1.0)[:, :k]
    mat_b = _randn((len(sizes), k, n + pad), dtype, gen, b_scale)[:, :, :n]
    offs = torch.tensor(np.cumsum(sizes), device="cuda", dtype=torch.int32)
    return mat_a, mat_b, offs


def _aggregate_check(out, mat_a, mat_b, sizes, dtype_name, precision="ieee", swiglu=False):
    from oracle import gemm as oracle

    start = 0
    for e, size in enumerate(sizes):
        if size:
            a = _host(mat_a[start:start + size])
            b = _host(mat_b[e])
            expected = oracle.swiglu(a, b, dtype_name) if swiglu else oracle.matmul(a, b, dtype_name)
            got = _host(out[start:start + size])
            assert np.isfinite(got).all(), f"expert {e}: unwritten rows"
            key = "tf32" if (dtype_name == "fp32" and precision == "tf32") else dtype_name
            err = oracle.relative_frobenius(got, expected)
            assert err <= REL_FRO[key], f"expert {e}: relative Frobenius error {err:.3e}"
        start += size


@pytest.mark.parametrize("dtype_name", ["fp16", "bf16"])
def test_aggregate_layout_uneven_experts_every_tile(dtype_name):
    """launch_grouped_mm over tokens sorted by expert with uneven and empty
    groups, for every native tile family; oracle per expert segment."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped_mm

    sizes = [37, 0, 300, 1, 0, 129, 16, 64]
    mat_a, mat_b, offs = _aggregate(sizes, 192, 320, dtype_name, seed=9)
    out = torch.full((sum(sizes), 320), float("nan"), device="cuda", dtype=_dtype(dtype_name))
    for cfg in (None, KernelConfig(16, 256, 64, 4, 8, 4), KernelConfig(64, 128, 64, 8, 4, 4),
                KernelConfig(128, 256, 64, 8, 8, 4), KernelConfig(256, 128, 64, 8, 8, 4),
                KernelConfig(256, 256, 64, 8, 8, 4)):
        out.fill_(float("nan"))
        launch_grouped_mm(mat_a, mat_b, offs, out, config=cfg)
        torch.cuda.synchronize()
        _aggregate_check(out, mat_a, mat_b, sizes, dtype_name)


def test_aggregate_segments_sharing_expert_weights():
    """offs with S = P * E segments (P senders' blocks, each sorted by the E
    experts, as an expert-parallel rank receives them): segment s multiplies
    mat_b[s % E] (grouped_gemm_offsets_launch_ex, b_count = E), for a plain
    and a scattered output."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped_mm, launch_grouped_mm_scatter
    from oracle import gemm as oracle

    experts, k, n = 3, 128, 264
    sizes = [5, 0, 70, 33, 12, 0, 1, 130, 9]  # 3 senders x 3 experts
    gen = torch.Generator(device="cuda").manual_seed(17)
    total = sum(sizes)
    mat_a = _randn((total, k), torch.bfloat16, gen, 1.0)
    mat_b = _randn((experts, k, n), torch.bfloat16, gen, 0.1)
    offs = torch.tensor(np.cumsum(sizes), device="cuda", dtype=torch.int32)
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]])
    for cfg in (KernelConfig(16, 256, 64, 4, 8, 4), KernelConfig(128, 256, 64, 8, 8, 4),
                KernelConfig(256, 128, 64, 8, 8, 4)):
        out = launch_grouped_mm(mat_a, mat_b, offs, config=cfg)
        dst = torch.zeros((total, n), dtype=torch.bfloat16, device="cuda")
        peers = torch.tensor([dst.data_ptr()], dtype=torch.int64, device="cuda")
        origin = torch.arange(total - 1, -1, -1, dtype=torch.int64, device="cuda")  # reversed rows
        launch_grouped_mm_scatter(mat_a, mat_b, offs, origin, peers, 0, n * 2, config=cfg)
        torch.cuda.synchronize()
        host_out, host_dst = _host(out), _host(dst)
        for s_idx, (start, size) in enumerate(zip(starts, sizes)):
            if size == 0:
                continue
            a = _host(mat_a[start:start + size])
            expected = oracle.matmul(a, _host(mat_b[s_idx % experts]), "bf16")
            got = host_out[start:start + size]
            assert oracle.relative_frobenius(got, expected) <= REL_FRO["bf16"], (cfg, s_idx)
            scattered = host_dst[total - start - size:total - start][::-1]
            assert np.array_equal(scattered, got), (cfg, s_idx)


def test_aggregate_layout_padding_precisions_and_swiglu():
    """Padded row pitches (C not TMA-addressable -> staged stores), fp32 on the
    generic kernel and on TF32 tensor cores, the fused SwiGLU epilogue, and a
    cross-check with torch's grouped_mm where it exists."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped_mm

    sizes = [5, 70, 0, 200]
    mat_a, mat_b, offs = _aggregate(sizes, 100, 100, "bf16", seed=2, pad=4)
    out = launch_grouped_mm(mat_a, mat_b, offs)
    torch.cuda.synchronize()
    _aggregate_check(out, mat_a, mat_b, sizes, "bf16")
    grouped_mm = getattr(torch.nn.functional, "grouped_mm", None)
    if grouped_mm is not None:
        try:
            ref = grouped_mm(mat_a, mat_b, offs=offs)
        except RuntimeError:
            ref = None
        if ref is not None:
            torch.testing.assert_close(out.float(), ref.float(), rtol=5e-2, atol=5e-2)
    for precision in ("ieee", "tf32"):
        a32, b32, offs32 = _aggregate(sizes, 64, 96, "fp32", seed=3)
        out32 = launch_grouped_mm(a32, b32, offs32, input_precision=precision)
        torch.cuda.synchronize()
        _aggregate_check(out32, a32, b32, sizes, "fp32", precision=precision)
    sw_sizes = [16, 0, 130, 300]
    a, b, offs_sw = _aggregate(sw_sizes, 256, 2 * 192, "bf16", seed=4, b_scale=1.0 / 16)
    h = launch_grouped_mm(a, b, offs_sw, swiglu=True)
    torch.cuda.synchronize()
    check_device_errors()
    assert h.shape == (sum(sw_sizes), 192)
    _aggregate_check(h, a, b, sw_sizes, "bf16", swiglu=True)


def test_aggregate_layout_graph_replay_follows_device_offsets():
    """Captured once; the routing (offs) changes on the device between
    replays and the output follows it."""
    torch = _torch()
    from kernels import launch_grouped_mm

    sizes = [64, 64, 64, 64]
    mat_a, mat_b, offs = _aggregate(sizes, 128, 256, "bf16", seed=6)
    out = torch.empty((256, 256), device="cuda", dtype=torch.bfloat16)
    launch_grouped_mm(mat_a, mat_b, offs, out)  # eager first call: scratch exists before capture
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch_grouped_mm(mat_a, mat_b, offs, out)
    new_sizes = [10, 0, 200, 46]
    offs.copy_(torch.tensor(np.cumsum(new_sizes), device="cuda", dtype=torch.int32))
    out.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    _aggregate_check(out, mat_a, mat_b, new_sizes, "bf16")
    del graph


# ------------------------------------------------- FP8 block-scaled experts
def _fp8_check(ws, rows=None):
    from oracle import gemm as oracle

    for a, sa, b, sb, c in ws.problem_tensors():
        if rows is not None:
            idx = rows(a.shape[0])
            a, sa, c = a.index_select(0, idx), sa.index_select(0, idx), c.index_select(0, idx)
        expected = oracle.fp8_block_scaled(_host(a), _host(sa), _host(b), _host(sb))
        got = _host(c)
        assert np.isfinite(got).all(), "output has non-finite values (unwritten)"
        err = oracle.relative_frobenius(got, expected)
        assert err <= REL_FRO["bf16"], f"relative Frobenius error {err:.3e}"
        np.testing.assert_allclose(got, expected, rtol=ASSERT_CLOSE["bf16"], atol=ASSERT_CLOSE["bf16"])


def test_fp8_block_scaled_every_tile_ragged_group():
    """e4m3 A [M, K] / B [N, K] with DeepSeek-V3 block scales on every native
    FP8 tile, over a heterogeneous group with partial K, N and M blocks."""
    torch = _torch()
    from kernels import KernelConfig, build_fp8_workspace, check_device_errors, launch_grouped_fp8

    shapes = [(16, 256, 256), (40, 320, 200), (130, 128, 384), (1, 64, 136), (300, 512, 256)]
    ws = build_fp8_workspace(shapes, seed=13)
    assert not ws.homogeneous
    for bm, bn in ((16, 256), (32, 256), (64, 256), (128, 128), (256, 128), (256, 256)):
        for c in ws.c:
            c.fill_(float("nan"))
        launch_grouped_fp8(ws, config=KernelConfig(bm, bn, 128, 4, 8, 4))
        torch.cuda.synchronize()
        check_device_errors()
        path = "tcgen05_tma_pair" if bm == 256 else "tcgen05_tma"
        assert ws.launch_info["path"] == path and ws.launch_info["tile_m"] == bm, ws.launch_info
        assert ws.launch_info["tile_n"] == bn, ws.launch_info
        _fp8_check(ws)


@pytest.mark.parametrize("m_e,k,n", [(16, 7168, 4096), (64, 2048, 7168), (128, 7168, 512), (1024, 256, 7168),
                                     (512, 7168, 4096), (1024, 2048, 7168)])
def test_fp8_block_scaled_deepseek_rank_shapes(m_e, k, n):
    """DeepSeek-V3 W13 / W2 expert shapes (3 experts, the FP8 tile policy);
    oracle on sampled rows."""
    torch = _torch()
    from kernels import build_fp8_workspace, check_device_errors, launch_grouped_fp8

    ws = build_fp8_workspace([(m_e, k, n)] * 3, seed=m_e + k)
    assert ws.homogeneous
    launch_grouped_fp8(ws)
    torch.cuda.synchronize()
    check_device_errors()
    rng = np.random.default_rng(k)
    rows = lambda m: torch.as_tensor(np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, 12)])), device="cuda")
    _fp8_check(ws, rows=rows)


@pytest.mark.parametrize("m_e,k,n", [(512, 7168, 4096), (1024, 2048, 7168), (300, 1024, 384)])
def test_fp8_pair_256_tile_rank_shapes(m_e, k, n):
    """The CTA-pair 256 x 256 FP8 tile (KernelConfig(256, 256, ...)) on
    DeepSeek-V3 W13 / W2 expert shapes, and on a group whose last weight tile
    is half past N (N = 384) with a partial last token tile."""
    torch = _torch()
    from kernels import KernelConfig, build_fp8_workspace, check_device_errors, launch_grouped_fp8

    ws = build_fp8_workspace([(m_e, k, n)] * 3, seed=m_e + n)
    for c in ws.c:
        c.fill_(float("nan"))
    launch_grouped_fp8(ws, config=KernelConfig(256, 256, 128, 8, 8, 4))
    torch.cuda.synchronize()
    check_device_errors()
    assert ws.launch_info["path"] == "tcgen05_tma_pair" and ws.launch_info["tile_n"] == 256, ws.launch_info
    rng = np.random.default_rng(k + 1)
    rows = lambda m: torch.as_tensor(np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, 12)])), device="cuda")
    _fp8_check(ws, rows=rows)


def test_fp8_refuses_unaddressable_rows():
    torch = _torch()
    from kernels import build_fp8_workspace, launch_grouped_fp8
    from kernels._native import NativeLaunchError

    ws = build_fp8_workspace([(8, 24, 64)] * 2, seed=1)  # 24-byte rows: not TMA-addressable
    with pytest.raises(NativeLaunchError, match="unsupported"):
        launch_grouped_fp8(ws)


def test_one_problem_group_dispatches_standard_matmul():
    """tests/test_gpu.py:190-195."""
    torch = _torch()
    from kernels import build_grouped_workspace, launch_grouped

    for dtype, shape in ((torch.float16, (17, 70, 65)), (torch.bfloat16, (96, 256, 384))):
        ws = build_grouped_workspace([shape], dtype, seed=103)
        launch_grouped(ws)
        torch.cuda.synchronize()
        assert ws.scheduler == "single_problem_matmul"
        _oracle_check(ws.c[0], ws.a[0], ws.b[0], "fp16" if dtype == torch.float16 else "bf16")


def test_graph_capture_and_replay_reads_tables_on_device():
    """Launches record into a CUDA graph (utils/benchmark.py:123-151); a replay
    after the inputs change computes the new product (tables and data are
    read on the device at run time)."""
    torch = _torch()
    from kernels import KernelConfig, launch_grouped

    ws = _workspace([(32, 512, 256)] * 4, "bf16", seed=11)
    cfg = KernelConfig(32, 128, 64, 4, 4, 3)
    launch_grouped(ws, config=cfg, autotune=False)  # eager warm-up outside capture
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch_grouped(ws, config=cfg, autotune=False)
    for a in ws.a:
        a.mul_(-1.5)
    _poison(ws)
    graph.replay()
    torch.cuda.synchronize()
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, "bf16")


def test_autotune_applies_the_native_tile_policy_and_caches_it():
    torch = _torch()
    from kernels import build_fused_gate_up_workspace, launch_grouped, native_candidates
    from kernels.grouped_gemm import _GROUPED_BASE_CONFIG_POOL

    ws = build_fused_gate_up_workspace([(16, 1024, 1024)] * 8, torch.bfloat16, seed=3)
    launch_grouped(ws)
    torch.cuda.synchronize()
    first = ws.config
    assert first in native_candidates(16)
    assert first in _GROUPED_BASE_CONFIG_POOL  # a config the reference's tooling knows
    _poison(ws)
    launch_grouped(ws)
    torch.cuda.synchronize()
    assert ws.config == first
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, "bf16", gate_up=True)


# --------------------------------------------------- DeepSeek-V3 shapes
def _sampled_rows_check(ws, dtype_name, rows_per_problem=24, seed=0, gate_up=False):
    """Oracle on a sample of output rows (full K reduction, all N columns)."""
    torch = _torch()
    rng = np.random.default_rng(seed)
    for a, b, c in ws.problem_tensors():
        m = a.shape[0]
        rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=rows_per_problem)]))
        idx = torch.as_tensor(rows, device=a.device)
        _oracle_check(c.index_select(0, idx), a.index_select(0, idx), b, dtype_name, gate_up=gate_up)


@pytest.mark.parametrize("m_e", [16, 64, 128, 256, 1024])
@pytest.mark.parametrize("proj,k,n", [("W13_EP", 7168, 4096), ("W13_TP", 7168, 512), ("W2_EP", 2048, 7168),
                                      ("W2_TP", 256, 7168)])
def test_deepseek_v3_rank_shapes(m_e, proj, k, n):
    """DeepSeek-V3 P=8 rank shapes (utils/metrics.py:40-72) with 3 experts, the autotuned
    launch, A ~ N(0,1), B ~ N(0, 1/sqrt(K)); oracle on sampled rows."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped

    ws = _workspace([(m_e, k, n)] * 3, "bf16", seed=m_e + k, b_scale=1.0 / math.sqrt(k))
    launch_grouped(ws)
    torch.cuda.synchronize()
    check_device_errors()
    assert ws.launch_info["path"].startswith("tcgen05_tma")
    _sampled_rows_check(ws, "bf16", gate_up=proj.startswith("W13"))


def test_full_size_w13_ep_column_checksums():
    """Full DeepSeek-V3 W13 EP rank (32 x [1024, 7168] @ [7168, 4096]):
    size-independent linearity check 1^T C = (1^T A) B per expert, in fp64."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped

    ws = _workspace([(1024, 7168, 4096)] * 32, "bf16", seed=77, b_scale=1.0 / math.sqrt(7168))
    launch_grouped(ws)
    torch.cuda.synchronize()
    check_device_errors()
    for a, b, c in ws.problem_tensors():
        expected = a.double().sum(0) @ b.double()
        got = c.double().sum(0)
        err = float((got - expected).norm() / expected.norm())
        assert err < 1e-2, err


def test_bounded_wait_reports_and_context_survives():
    """Failure detection without a fault: the test hook makes the epilogue
    wait on a barrier nothing arrives on; the wait gives up after its budget,
    the error word reports it, and the context keeps working."""
    torch = _torch()
    from kernels import KernelConfig, _native, check_device_errors, launch_grouped

    ws = _workspace([(16, 256, 256)] * 2, "bf16", seed=12)
    check_device_errors()
    _native.set_debug(wait_budget_cycles=2_000_000, test_flags=1)
    try:
        launch_grouped(ws, config=KernelConfig(16, 128, 64, 4, 4, 3), autotune=False)
        torch.cuda.synchronize()
    finally:
        _native.set_debug(0, 0)
    word = _native.read_and_clear_error_word(torch.cuda.current_device())
    assert word == _native.TEST_WAIT_BIT, _native.describe_error_word(word)
    _poison(ws)
    launch_grouped(ws, config=KernelConfig(16, 128, 64, 4, 4, 3), autotune=False)
    torch.cuda.synchronize()
    check_device_errors()
    for a, b, c in ws.problem_tensors():
        _oracle_check(c, a, b, "bf16")


def test_table_entry_breaking_alignment_is_skipped_not_faulted():
    """A device table entry changed to an address that breaks the TMA
    promise is skipped on the device and reported; nothing is dereferenced."""
    torch = _torch()
    from kernels import KernelConfig, _native, launch_grouped

    ws = _workspace([(16, 256, 256)] * 3, "bf16", seed=13)
    check_ok = _native.read_and_clear_error_word(torch.cuda.current_device())
    del check_ok
    good = int(ws.a_ptrs[1].item())
    ws.a_ptrs[1] = good + 2  # misaligned by 2 bytes, still inside the allocation
    _poison(ws)
    launch_grouped(ws, config=KernelConfig(16, 128, 64, 4, 4, 3), autotune=False)
    torch.cuda.synchronize()
    word = _native.read_and_clear_error_word(torch.cuda.current_device())
    assert word & (1 << 5)
    assert torch.isnan(ws.c[1]).all()
    for e in (0, 2):
        _oracle_check(ws.c[e], ws.a[e], ws.b[e], "bf16")
    ws.a_ptrs[1] = good


@pytest.mark.parametrize("dtype_name,precision,shape", [
    ("fp32", "tf32", (1000, 4095, 127)),
    ("fp32", "tf32", (127, 1000, 4095)),
    ("bf16", "ieee", (1000, 4095, 1000)),
    ("fp16", "ieee", (333, 2047, 515)),
])
def test_masked_large_shapes_repack_onto_tensor_cores(dtype_name, precision, shape):
    """The Qwen3 masked sweep's non-tile-multiple sizes:
    rows the TMA cannot address are repacked and run on the tensor cores."""
    torch = _torch()
    from kernels import launch_matmul
    from kernels.matmul import last_launch_info

    m, k, n = shape
    gen = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = _randn((m, k), _dtype(dtype_name), gen)
    b = _randn((k, n), _dtype(dtype_name), gen)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=_dtype(dtype_name))
    launch_matmul(a, b, c, input_precision=precision)
    torch.cuda.synchronize()
    info = last_launch_info()
    assert info["path"].startswith("tcgen05_tma"), info
    assert info["repacked"], info
    _oracle_check(c, a, b, dtype_name, precision)


@pytest.mark.parametrize("m,k,n,precision,masked", [
    (127, 8191, 4095, "tf32", True),
    (4095, 8191, 127, "ieee", True),
    (127, 2048, 127, "ieee", False),
    (256, 4096, 384, "tf32", False),
])
def test_fp32_split_k_single_gemm(m, k, n, precision, masked):
    """fp32 GEMMs with few output tiles and a long K run as one grouped launch
    over K slices into fp32 partials plus matrix_sum_partials; sampled rows
    against the float64 oracle, and a CUDA-graph replay of the same launch
    gives the same bits."""
    torch = _torch()
    from kernels import check_device_errors, launch_matmul
    from kernels.matmul import last_launch_info
    from oracle import gemm as oracle

    gen = torch.Generator(device="cuda").manual_seed(m + 3 * k + 7 * n)
    if masked:  # rows of k (or n) floats: the TMA cannot address them, so they are repacked first
        a = torch.randn((m, k), device="cuda", generator=gen)
        b = torch.randn((k, n), device="cuda", generator=gen) / math.sqrt(k)
    else:
        a = torch.randn((m, k + 5), device="cuda", generator=gen)[:, :k]
        a = a.contiguous()
        b = torch.randn((k, n), device="cuda", generator=gen) / math.sqrt(k)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    launch_matmul(a, b, c, input_precision=precision)
    torch.cuda.synchronize()
    check_device_errors()
    info = last_launch_info()
    assert info["split_k"] > 1, info
    assert not torch.isnan(c).any()
    rows = torch.tensor(sorted({0, 1, m // 2, m - 1}), device="cuda")
    got = c.index_select(0, rows).double().cpu().numpy()
    expected = oracle.matmul(a.index_select(0, rows).double().cpu().numpy(), b.double().cpu().numpy(), "fp32")
    assert oracle.relative_frobenius(got, expected) <= REL_FRO["tf32" if precision == "tf32" else "fp32"]
    eager = c.clone()
    c.fill_(float("nan"))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            launch_matmul(a, b, c, input_precision=precision)
        graph.replay()
    stream.synchronize()
    check_device_errors()
    assert torch.equal(c, eager)
    del graph


def test_sum_partials_every_output_dtype():
    """matrix_sum_partials adds the partials in order in fp32 and rounds once,
    through C's strides, for fp32, bf16 and fp16 outputs."""
    torch = _torch()
    from kernels import _native

    gen = torch.Generator(device="cuda").manual_seed(5)
    partials = torch.randn((3, 37, 45), device="cuda", generator=gen)
    expected = (partials[0] + partials[1]) + partials[2]
    stream = torch.cuda.current_stream().cuda_stream
    for dtype, name in ((torch.float32, "fp32"), (torch.bfloat16, "bf16"), (torch.float16, "fp16")):
        out = torch.full((45, 37), float("nan"), device="cuda", dtype=dtype).t()  # column-major C
        _native.sum_partials(partials.data_ptr(), 3, 37, 45, out.data_ptr(), out.stride(0), out.stride(1), name,
                             stream)
        torch.cuda.synchronize()
        assert torch.equal(out, expected.to(dtype)), name


@pytest.mark.parametrize("case", [
    # Mixtral-8x7B (E=8, H=4096, F=14336), M_e = 1024: EP P=8 is one expert per rank
    ("mixtral W13 EP P=8", [(1024, 4096, 2 * 14336)], True),
    ("mixtral W2 EP P=8", [(1024, 14336, 4096)], False),
    ("mixtral W13 TP P=4", [(1024, 4096, 2 * 14336 // 4)] * 3, True),
    ("mixtral W2 TP P=2", [(1024, 14336 // 2, 4096)] * 2, False),
    # Qwen3-235B-A22B (E=128, H=4096, F=1536), P=8, T=256 -> M_e=16, T=16384 -> M_e=1024
    ("qwen3 W13 EP M16", [(16, 4096, 3072)] * 4, True),
    ("qwen3 W13 TP M1024", [(1024, 4096, 384)] * 4, True),
    ("qwen3 W2 EP M256", [(256, 1536, 4096)] * 4, False),
    ("qwen3 W2 TP M64", [(64, 192, 4096)] * 4, False),
], ids=lambda c: c[0])
def test_mixtral_and_qwen3_rank_shapes(case):
    """Mixtral and Qwen3 rank shapes (a few
    experts each), autotuned launch, oracle on sampled rows."""
    torch = _torch()
    from kernels import check_device_errors, launch_grouped

    _, shapes, gate_up = case
    k = shapes[0][1]
    ws = _workspace(shapes, "bf16", seed=k + len(shapes), b_scale=1.0 / math.sqrt(k))
    launch_grouped(ws)
    torch.cuda.synchronize()
    check_device_errors()
    assert ws.launch_info["path"].startswith("tcgen05_tma"), ws.launch_info
    assert ws.scheduler == ("single_problem_matmul" if len(shapes) == 1 else "homogeneous_persistent")
    _sampled_rows_check(ws, "bf16", rows_per_problem=8, gate_up=gate_up)
