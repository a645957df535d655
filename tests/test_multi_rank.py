"""Multi-rank host logic on CPU: world_size 2 over gloo.

The GPU runs put one rank of the P-way EP/TP layer on each GPU with no
collective in the timed region, then gather outputs for verification
(bench.py).  Here the same shard plans, gather and reassembly run as two gloo
processes whose per-rank GEMMs come from the CPU oracle; rank 0 checks the
reassembled layer against the global product.  A second test makes a rank
fail on the host before the gather and checks that the survivor's collective
ends with an error instead of waiting forever.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for path in (str(ROOT), str(ROOT / "moe-gemm-parallel-bench_b200")):
        if path not in sys.path:
            sys.path.insert(0, path)


def _layer(seed=0, e=4, f=8, h=6, m=5):
    rng = np.random.default_rng(seed)
    a = [rng.standard_normal((m, h)) for _ in range(e)]
    w13 = [rng.standard_normal((h, 2 * f)) for _ in range(e)]
    return a, w13, (e, f, h, m)


def _worker(rank, world, port, mode, result_path):
    _setup_paths()
    from moe_parallel import assemble_w13_tp, ep_owner, rank_plan, shard_weight
    from oracle import gemm as oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    a, w13, (e, f, h, m) = _layer()
    if mode == "fail" and rank == 1:
        # A rank that dies on the host between steps: it never joins the gather.
        os._exit(3)
    ep = rank_plan("W1", "EP", rank, world, e, f, h)
    tp = rank_plan("W1", "TP", rank, world, e, f, h)
    ep_out = torch.zeros((e, m, 2 * f), dtype=torch.float64)
    for x in ep.experts:
        ep_out[x] = torch.from_numpy(oracle.matmul(a[x], w13[x], "fp32"))
    tp_out = torch.stack([torch.from_numpy(oracle.matmul(a[x], shard_weight(w13[x], tp), "fp32"))
                          for x in tp.experts])
    gathered_ep = [torch.empty_like(ep_out) for _ in range(world)]
    gathered_tp = [torch.empty_like(tp_out) for _ in range(world)]
    try:
        dist.all_gather(gathered_ep, ep_out)
        dist.all_gather(gathered_tp, tp_out)
    except RuntimeError as exc:
        Path(result_path).write_text(f"collective failed: {type(exc).__name__}")
        os._exit(0)
    if rank == 0:
        worst = 0.0
        for x in range(e):
            expected = oracle.matmul(a[x], w13[x], "fp32")
            got_ep = gathered_ep[ep_owner(x, world, e)][x].numpy()
            got_tp = assemble_w13_tp([gathered_tp[r][x].numpy() for r in range(world)], world)
            worst = max(worst, oracle.relative_frobenius(got_ep, expected),
                        oracle.relative_frobenius(got_tp, expected))
        Path(result_path).write_text(f"ok {worst}")
    dist.destroy_process_group()


def test_two_gloo_ranks_gather_and_reassemble(tmp_path):
    result = tmp_path / "result.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, "ok", str(result))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    text = result.read_text()
    assert text.startswith("ok")
    assert float(text.split()[1]) < 1e-7


def test_rank_death_before_gather_ends_the_collective_with_an_error(tmp_path):
    result = tmp_path / "result.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, "fail", str(result))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode is not None for p in procs), "a rank is still waiting"
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    assert result.read_text().startswith("collective failed")
