"""Regenerates the golden fixtures in this directory FROM THE REFERENCE ITSELF.

Run in a container that holds the reference checkout (never on the GPU box;
the fixtures are committed):

    REFERENCE_PATH=/path/to/moe-gemm-parallel-bench python tests/golden/make_golden.py

* configs.json.gz -- outputs of the reference's pure-Python tile heuristics
                    (select_config, matmul_candidate_configs,
                    grouped_candidate_configs; kernels/matmul.py:35-170,
                    kernels/grouped_gemm.py:114-224) and of its EP/TP shape
                    model (utils/metrics.py:40-80) over a grid of inputs.
* gemm_cases.npz -- inputs and outputs of the reference's Triton kernels
                    (_homogeneous_grouped_kernel_impl, _generic_grouped_kernel_impl,
                    _matmul_kernel_impl) executed by Triton's CPU interpreter
                    (TRITON_INTERPRET=1) on seeded inputs.  fp16 and fp32 only:
                    the interpreter mis-reads bfloat16 memory, so bf16 parity
                    rests on the oracle, which these cases pin.
"""

from __future__ import annotations

import gzip
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if "REFERENCE_PATH" not in os.environ:
    raise SystemExit("set REFERENCE_PATH to the reference checkout (see the module docstring)")
REFERENCE = Path(os.environ["REFERENCE_PATH"])


def _import_reference():
    # The reference builds its Triton kernels only when a CUDA driver answers
    # (kernels/grouped_gemm.py:236-263); the interpreter needs none, so report
    # an sm_100 target and let the module define them.
    import triton
    from triton.backends.compiler import GPUTarget

    class _InterpreterTarget:
        def get_current_target(self):
            return GPUTarget("cuda", 100, 32)

    torch.cuda.is_available = lambda: True
    triton.runtime.driver.set_active(_InterpreterTarget())
    sys.path.insert(0, str(REFERENCE))
    import kernels.grouped_gemm as grouped
    import kernels.matmul as matmul
    import utils.metrics as metrics

    return grouped, matmul, metrics


def config_fixtures(grouped, matmul, metrics) -> dict:
    def cfg(c):
        return [c.block_m, c.block_n, c.block_k, c.group_size_m, c.num_warps, c.num_stages, c.cta_multiplier]

    dims = (1, 16, 17, 32, 33, 64, 65, 127, 128, 129, 1000, 4095, 8191)
    select = [[m, n, k, cfg(matmul.select_config(m, n, k))] for m in dims for n in dims for k in (1, 8191, 8192)]
    matmul_cands = []
    for m in (1, 16, 17, 33, 64, 65, 129, 512, 4095):
        for n in (3, 32, 64, 65, 128, 512, 8192):
            for k in (1, 32, 128, 4096):
                matmul_cands.append([m, n, k, [cfg(c) for c in matmul.matmul_candidate_configs(m, n, k)]])
    grouped_cands = []
    for m in (1, 16, 17, 33, 64, 128, 129, 512, 1024):
        for n in (3, 64, 65, 256, 4096, 7168):
            for k in (1, 64, 256, 7168):
                for problems, sms in ((1, 148), (3, 0), (32, 148), (256, 120)):
                    got = grouped.grouped_candidate_configs(m, n, k, problem_count=problems, sm_count=sms)
                    grouped_cands.append([m, n, k, problems, sms, [cfg(c) for c in got]])
    shapes = []
    for proj in ("W1", "W2"):
        for par in ("EP", "TP"):
            for m, h, f, e, p in ((17, 7168, 2048, 256, 8), (16, 7168, 2048, 256, 8), (1024, 4096, 14336, 8, 8),
                                  (64, 4096, 1536, 128, 8), (64, 1024, 512, 8, 1)):
                shapes.append([proj, par, m, h, f, e, p, [list(s) for s in metrics.moe_shapes(proj, par, m, h, f, e, p)[:1]],
                               len(metrics.moe_shapes(proj, par, m, h, f, e, p)),
                               metrics.verify_ep_tp_flops(proj, m, h, f, e, p)])
    return {
        "matmul_pool": [cfg(c) for c in matmul._MATMUL_CONFIG_POOL],
        "grouped_base_pool": [cfg(c) for c in grouped._GROUPED_BASE_CONFIG_POOL],
        "select_config": select,
        "matmul_candidate_configs": matmul_cands,
        "grouped_candidate_configs": grouped_cands,
        "moe_shapes": shapes,
    }


def _tensor(values: np.ndarray, dtype: str) -> torch.Tensor:
    torch_dtype = {"fp16": torch.float16, "fp32": torch.float32}[dtype]
    return torch.from_numpy(np.ascontiguousarray(values)).to(torch_dtype)


def _inputs(rng, shapes, dtype):
    a_list = [_tensor(rng.standard_normal((m, k)) * 0.1, dtype) for m, k, _ in shapes]
    b_list = [_tensor(rng.standard_normal((k, n)) * 0.1, dtype) for _, k, n in shapes]
    return a_list, b_list


def run_grouped(grouped, matmul, a_list, b_list, config, homogeneous: bool, precision: str = "ieee"):
    """The reference's fixed-config grouped launch (kernels/grouped_gemm.py:684-760) on host tensors."""
    c_list = [torch.full((a.shape[0], b.shape[1]), float("nan"), dtype=a.dtype) for a, b in zip(a_list, b_list)]
    ptrs = [torch.tensor([x.data_ptr() for x in xs], dtype=torch.int64) for xs in (a_list, b_list, c_list)]
    shapes = [(a.shape[0], a.shape[1], b.shape[1]) for a, b in zip(a_list, b_list)]
    tiles = sum(-(-m // config.block_m) * -(-n // config.block_n) for m, _, n in shapes)
    grid = (max(1, min(tiles, 4 * config.cta_multiplier)),)  # a small persistent grid: several rounds per CTA
    common = dict(SHAPE_SIGNATURE=0, DEVICE_SIGNATURE=0, SM_COUNT=4, BLOCK_M=config.block_m, BLOCK_N=config.block_n,
                  BLOCK_K=config.block_k, GROUP_M=config.group_size_m, CTA_MULTIPLIER=config.cta_multiplier,
                  INPUT_PRECISION=precision, num_warps=config.num_warps, num_stages=config.num_stages)
    if homogeneous:
        m, k, n = shapes[0]
        grouped._homogeneous_grouped_kernel_impl[grid](
            *ptrs, a_list[0], b_list[0], c_list[0], M=m, N=n, K=k, MAX_M=m, MAX_N=n, MAX_K=k,
            PROBLEM_COUNT=len(shapes), **common)
    else:
        dims = torch.tensor([[m, n, k] for m, k, n in shapes], dtype=torch.int32)
        strides = torch.tensor([[a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1)]
                                for a, b, c in zip(a_list, b_list, c_list)], dtype=torch.int64)
        grouped._generic_grouped_kernel_impl[grid](
            *ptrs, dims, strides, a_list[0], b_list[0], c_list[0], len(shapes),
            MAX_M=max(s[0] for s in shapes), MAX_N=max(s[2] for s in shapes), MAX_K=max(s[1] for s in shapes),
            **common)
    return c_list


def run_matmul(matmul, a, b, c, config, precision: str = "ieee"):
    """The reference's fixed-config single launch (kernels/matmul.py:369-392) on host tensors."""
    m, k = a.shape
    n = b.shape[1]
    grid = (-(-m // config.block_m) * -(-n // config.block_n),)
    matmul._matmul_kernel_impl[grid](
        a, b, c, m, n, k, a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1),
        DEVICE_SIGNATURE=0, BLOCK_M=config.block_m, BLOCK_N=config.block_n, BLOCK_K=config.block_k,
        GROUP_M=config.group_size_m, INPUT_PRECISION=precision, num_warps=config.num_warps,
        num_stages=config.num_stages)
    return c


def gemm_fixtures(grouped, matmul) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    index = []
    KC = matmul.KernelConfig

    def record(name, kind, dtype, a_list, b_list, c_list, extra=None):
        entry = {"name": name, "kind": kind, "dtype": dtype, "problems": len(a_list), **(extra or {})}
        index.append(entry)
        for e, (a, b, c) in enumerate(zip(a_list, b_list, c_list)):
            np_dtype = np.float16 if dtype == "fp16" else np.float32
            out[f"{name}/a{e}"] = a.numpy().astype(np_dtype)
            out[f"{name}/b{e}"] = b.numpy().astype(np_dtype)
            out[f"{name}/c{e}"] = c.numpy().astype(np_dtype)

    rng = np.random.default_rng(20251201)
    hetero = [(1, 5, 3), (17, 13, 31), (9, 70, 65)]  # tests/test_gpu.py:99-115
    for dtype in ("fp32", "fp16"):
        a_list, b_list = _inputs(rng, hetero, dtype)
        cfg = matmul.select_config(17, 65, 70)
        record(f"grouped_generic_{dtype}", "grouped", dtype, a_list, b_list,
               run_grouped(grouped, matmul, a_list, b_list, cfg, homogeneous=False))
    # Homogeneous tails (tests/test_gpu.py:117-125, :127-154) with a multi-round grid.
    for dtype, shape, cfg in (("fp32", (17, 33, 65), KC(16, 32, 32, 4, 4, 2)),
                              ("fp16", (17, 13, 31), KC(16, 32, 32, 4, 2, 2))):
        a_list, b_list = _inputs(rng, [shape] * 3, dtype)
        record(f"grouped_homog_{dtype}", "grouped", dtype, a_list, b_list,
               run_grouped(grouped, matmul, a_list, b_list, cfg, homogeneous=True))
    # Packed gate+up (tests/test_gpu.py:176-188).
    a_list, b_list = _inputs(rng, [(17, 13, 62)] * 3, "fp16")
    record("gate_up_fp16", "gate_up", "fp16", a_list, b_list,
           run_grouped(grouped, matmul, a_list, b_list, KC(16, 64, 32, 4, 2, 2), homogeneous=True))
    # The tutorial-comparison shapes (tests/test_gpu.py:34-52).
    a_list, b_list = _inputs(rng, [(128, 256, 128)] * 2, "fp16")
    record("tutorial_homog_fp16", "grouped", "fp16", a_list, b_list,
           run_grouped(grouped, matmul, a_list, b_list, KC(64, 64, 32, 1, 4, 3), homogeneous=True))
    # TMA-aligned miniature MoE groups: narrow M over several K blocks, and an
    # M tail past one 128-row tile.
    for name, shapes, cfg in (("moe_narrow_fp16", [(16, 256, 256)] * 2, KC(16, 64, 64, 4, 4, 3)),
                              ("moe_tail_fp16", [(130, 192, 128)] * 2, KC(64, 64, 64, 4, 4, 3)),
                              ("moe_hetero_fp16", [(16, 128, 128), (40, 192, 128), (130, 64, 256)],
                               KC(32, 64, 64, 4, 4, 3))):
        a_list, b_list = _inputs(rng, shapes, "fp16")
        record(name, "grouped", "fp16", a_list, b_list,
               run_grouped(grouped, matmul, a_list, b_list, cfg, homogeneous=len(set(shapes)) == 1))
    # Single GEMM odd shapes (tests/test_gpu.py:69-86).
    for dtype in ("fp32", "fp16"):
        for m, k, n in ((1, 5, 3), (17, 13, 31), (33, 70, 65)):
            a_list, b_list = _inputs(rng, [(m, k, n)], dtype)
            c = torch.full((m, n), float("nan"), dtype=a_list[0].dtype)
            run_matmul(matmul, a_list[0], b_list[0], c, matmul.select_config(m, n, k))
            record(f"single_{dtype}_{m}x{k}x{n}", "single", dtype, a_list, b_list, [c])
    # Strided fp32 views with TF32 requested (tests/test_gpu.py:88-97).
    m, k, n = 17, 70, 65
    a_base = _tensor(rng.standard_normal((m, 2 * k)) * 0.1, "fp32")
    b_base = _tensor(rng.standard_normal((k, 2 * n)) * 0.1, "fp32")
    c_base = torch.full((m, 2 * n), float("nan"))
    run_matmul(matmul, a_base[:, ::2], b_base[:, ::2], c_base[:, ::2], matmul.select_config(m, n, k), "tf32")
    index.append({"name": "single_fp32_strided_tf32", "kind": "single_strided", "dtype": "fp32", "problems": 1})
    out["single_fp32_strided_tf32/a_base"] = a_base.numpy()
    out["single_fp32_strided_tf32/b_base"] = b_base.numpy()
    out["single_fp32_strided_tf32/c_base"] = c_base.numpy()
    out["_index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    return out


def main() -> None:
    grouped, matmul, metrics = _import_reference()
    with gzip.open(HERE / "configs.json.gz", "wt") as handle:
        handle.write(json.dumps(config_fixtures(grouped, matmul, metrics)) + "\n")
    np.savez_compressed(HERE / "gemm_cases.npz", **gemm_fixtures(grouped, matmul))
    print("wrote", HERE / "configs.json.gz", HERE / "gemm_cases.npz")


if __name__ == "__main__":
    main()
