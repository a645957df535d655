"""Expert-parallel MoE layer: routing, dispatch / combine over peer memory and
the grouped GEMMs between them.

CPU: the layout restatement (every slot lands once, sorted by local expert
then source rank), the layer oracle against a per-slot loop, capacity and
handle exchange over two gloo ranks.  GPU: the layer on one rank against the
oracle (uniform, skewed and dropped routing, zero tokens, repeated forwards,
CUDA-graph replay, capacity overflow reported rather than written out of
bounds), the standalone route / permute / combine kernels, and two ranks on
two GPUs when the box has them.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

from oracle import moe_layer as oracle_moe
from oracle.gemm import bf16_round, relative_frobenius
from tests.conftest import cuda_ready

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parents[1]
BF16_TOL = 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for path in (str(ROOT), str(ROOT / "moe-gemm-parallel-bench_b200")):
        if path not in sys.path:
            sys.path.insert(0, path)


def _routing(rng, tokens, experts, top_k, skew=False, drop=0.0):
    """topk_ids [T, k] int32 (distinct experts per token) and weights [T, k] fp32."""
    if skew:
        p = np.linspace(1.0, 8.0, experts) ** 3
        p /= p.sum()
    else:
        p = None
    ids = np.stack([rng.choice(experts, size=top_k, replace=False, p=p) for _ in range(tokens)]) \
        if tokens else np.zeros((0, top_k), dtype=np.int64)
    ids = ids.astype(np.int32)
    if drop:
        ids[rng.random(ids.shape) < drop] = -1
    weights = rng.random((tokens, top_k)).astype(np.float32)
    weights /= np.maximum(weights.sum(axis=1, keepdims=True), 1e-6)
    return ids, weights


def _weights(rng, experts, hidden, ffn):
    w13 = bf16_round((rng.standard_normal((experts, hidden, 2 * ffn)) / np.sqrt(hidden)).astype(np.float32))
    w2 = bf16_round((rng.standard_normal((experts, ffn, hidden)) / np.sqrt(ffn)).astype(np.float32))
    return w13, w2


def _tokens(rng, tokens, hidden):
    return bf16_round(rng.standard_normal((tokens, hidden)).astype(np.float32))


# ---------------------------------------------------------------- CPU tests


@pytest.mark.parametrize("world,experts", [(1, 8), (2, 8), (4, 16), (8, 256)])
def test_ep_layout_places_every_slot_once(world, experts):
    rng = np.random.default_rng(world * 100 + experts)
    counts = rng.integers(0, 9, size=(world, experts))
    counts[0, :] = 0  # a rank that sends nothing
    local = experts // world
    layouts = [oracle_moe.ep_layout(counts, r) for r in range(world)]
    for owner in range(world):
        _, recv_offs = layouts[owner]
        taken = np.zeros(int(recv_offs[-1]) if local else 0, dtype=np.int64)
        for r in range(world):
            send_base, _ = layouts[r]
            for e in range(owner * local, (owner + 1) * local):
                rows = send_base[e] + np.arange(counts[r, e])
                el = e - owner * local
                lo = recv_offs[el - 1] if el else 0
                assert np.all((rows >= lo) & (rows < recv_offs[el])), "row outside its expert's segment"
                taken[rows] += 1
        assert np.all(taken == 1), "receive rows must be covered exactly once"


def test_ep_layout_orders_source_ranks_inside_an_expert():
    counts = np.array([[2, 1, 0, 3], [1, 4, 2, 0]])
    base0, offs0 = oracle_moe.ep_layout(counts, 0)
    base1, offs1 = oracle_moe.ep_layout(counts, 1)
    # owner 0 holds experts 0, 1: e0 rows [rank0: 0-1 | rank1: 2], e1 rows [rank0: 3 | rank1: 4-7]
    assert list(base0[:2]) == [0, 3] and list(base1[:2]) == [2, 4]
    assert list(offs0) == [3, 8] and list(offs1) == [2, 5]
    clamped, offs_c = oracle_moe.ep_layout(counts, 1, capacity=3)
    assert list(clamped[:2]) == [2, 3] and list(offs_c) == [2, 3]


def test_layer_oracle_matches_a_per_slot_loop():
    rng = np.random.default_rng(5)
    t, h, f, e, k = 9, 16, 8, 4, 2
    x = _tokens(rng, t, h)
    w13, w2 = _weights(rng, e, h, f)
    ids, w = _routing(rng, t, e, k, drop=0.2)
    got = oracle_moe.moe_layer(x, ids, w, w13, w2)
    expected = np.zeros((t, h))
    for i in range(t):
        for j in range(k):
            ex = ids[i, j]
            if ex < 0:
                continue
            gate = x[i] @ w13[ex][:, :f].astype(np.float64)
            up = x[i] @ w13[ex][:, f:].astype(np.float64)
            hid = bf16_round((gate / (1 + np.exp(-gate)) * up).astype(np.float32)).astype(np.float64)
            expected[i] += w[i, j] * bf16_round((hid @ w2[ex]).astype(np.float32))
    assert relative_frobenius(got, expected) < 1e-2
    counts = oracle_moe.route_counts(ids, e)
    assert counts.sum() == int((ids >= 0).sum())


def test_capacity_and_expected_rows():
    _setup_paths()
    from expert_parallel import ep_capacity, expected_rows_per_expert

    assert ep_capacity(128, 8, 8) == 8192
    assert expected_rows_per_expert(128, 8, 32) == 32
    assert expected_rows_per_expert(1, 1, 32) == 1
    with pytest.raises(ValueError):
        ep_capacity(-1, 8, 8)


def _gloo_handles(rank, world, port, result_path):
    _setup_paths()
    import torch.distributed as dist
    from expert_parallel import exchange_handles

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    handles = exchange_handles(bytes([rank + 1]) * 64, rank, world)
    dist.destroy_process_group()
    if rank == 0:
        Path(result_path).write_text(",".join(str(h[0]) for h in handles))


def test_handle_exchange_keeps_rank_order_over_gloo(tmp_path):
    import torch.multiprocessing as mp

    result = tmp_path / "handles.txt"
    mp.start_processes(_gloo_handles, args=(2, _free_port(), str(result)), nprocs=2, start_method="spawn")
    assert result.read_text() == "1,2"


# ---------------------------------------------------------------- GPU tests


def _layer_case(seed, tokens, experts, hidden, ffn, top_k, **routing):
    rng = np.random.default_rng(seed)
    x = _tokens(rng, tokens, hidden)
    w13, w2 = _weights(rng, experts, hidden, ffn)
    ids, w = _routing(rng, tokens, experts, top_k, **routing)
    return x, w13, w2, ids, w


def _to_gpu(x, w13, w2, ids, w, device="cuda"):
    bf = torch.bfloat16
    return (torch.from_numpy(x).to(device, bf), torch.from_numpy(w13).to(device, bf),
            torch.from_numpy(w2).to(device, bf), torch.from_numpy(ids).to(device),
            torch.from_numpy(w).to(device))


@pytest.mark.parametrize("tokens,experts,hidden,ffn,top_k,routing", [
    (96, 8, 256, 128, 2, {}),
    (200, 16, 512, 256, 4, {"skew": True}),
    (64, 8, 256, 192, 2, {"drop": 0.25}),
    (300, 32, 1024, 512, 8, {}),
])
@pytest.mark.parametrize("fused_return", [True, False])
@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_single_rank_layer_matches_oracle(tokens, experts, hidden, ffn, top_k, routing, fused_return):
    _setup_paths()
    from expert_parallel import ExpertParallelMoE

    x, w13, w2, ids, w = _layer_case(1, tokens, experts, hidden, ffn, top_k, **routing)
    gx, g13, g2, gids, gw = _to_gpu(x, w13, w2, ids, w)
    with ExpertParallelMoE(g13, g2, experts, max_tokens=tokens, top_k=top_k, fused_return=fused_return) as layer:
        out = layer(gx, gids, gw)
        layer.check_errors()
        expected = oracle_moe.moe_layer(x, ids, w, w13, w2)
        err = relative_frobenius(out.float().cpu().numpy(), expected)
        assert err < BF16_TOL, err
        counts = oracle_moe.route_counts(ids, experts)
        assert layer.recv_offs.cpu().tolist() == np.cumsum(counts).tolist()


@pytest.mark.parametrize("tile", ["swap16x256", "swap32x256", "swap64x256", "tok128x256", "tok128x64",
                                  "pair256x256", "pair256x512"])
@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_scatter_epilogue_every_tile_family(tile):
    """W2-style aggregate GEMM whose rows go to per-row destinations: equal to
    the plain launch's rows, permuted, with dropped rows left untouched."""
    _setup_paths()
    from kernels import KernelConfig, launch_grouped_mm, launch_grouped_mm_scatter

    shapes = {"swap16x256": (16, 256), "swap32x256": (32, 256), "swap64x256": (64, 256), "tok128x256": (128, 256),
              "tok128x64": (128, 64), "pair256x256": (256, 128), "pair256x512": (256, 256)}
    bm, bn = shapes[tile]
    cfg = KernelConfig(bm, bn, 64, 8, 4, 4)
    rng = np.random.default_rng(4)
    sizes = [0, 37, 300, 5, 129, 64]
    k, n = 192, 776
    total = sum(sizes)
    gen = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn((total, k), device="cuda", generator=gen).to(torch.bfloat16)
    b = (torch.randn((len(sizes), k, n), device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    offs = torch.tensor(np.cumsum(sizes), dtype=torch.int32, device="cuda")
    ref = launch_grouped_mm(a, b, offs, config=cfg)
    perm = rng.permutation(total)
    origin_host = perm.astype(np.int64)
    origin_host[rng.random(total) < 0.1] = -1  # dropped rows
    pitch = n + 8  # padded destination rows
    dst = torch.full((total, pitch), 7.0, dtype=torch.bfloat16, device="cuda")
    peers = torch.tensor([dst.data_ptr()], dtype=torch.int64, device="cuda")
    launch_grouped_mm_scatter(a, b, offs, torch.from_numpy(origin_host).cuda(), peers, 0, pitch * 2, config=cfg)
    torch.cuda.synchronize()
    host_dst, host_ref = dst.float().cpu().numpy(), ref.float().cpu().numpy()
    kept = origin_host >= 0
    assert np.array_equal(host_dst[origin_host[kept], :n], host_ref[kept])
    untouched = np.setdiff1d(np.arange(total), origin_host[kept])
    assert np.all(host_dst[untouched] == 7.0) and np.all(host_dst[:, n:] == 7.0)


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_nccl_baseline_layer_single_rank_matches_oracle():
    _setup_paths()
    from expert_parallel import NcclAllToAllMoE

    tokens, experts, hidden, ffn, top_k = 150, 16, 512, 256, 4
    x, w13, w2, ids, w = _layer_case(9, tokens, experts, hidden, ffn, top_k, drop=0.1)
    gx, g13, g2, gids, gw = _to_gpu(x, w13, w2, ids, w)
    layer = NcclAllToAllMoE(g13, g2, experts, max_tokens=tokens, top_k=top_k)
    out = layer(gx, gids, gw)
    layer.check_errors()
    err = relative_frobenius(out.float().cpu().numpy(), oracle_moe.moe_layer(x, ids, w, w13, w2))
    assert err < BF16_TOL, err


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_repeated_forwards_zero_tokens_and_graph_replay():
    _setup_paths()
    from expert_parallel import ExpertParallelMoE

    experts, hidden, ffn, top_k, max_tokens = 8, 256, 128, 2, 128
    rng = np.random.default_rng(7)
    w13, w2 = _weights(rng, experts, hidden, ffn)
    g13 = torch.from_numpy(w13).cuda().to(torch.bfloat16)
    g2 = torch.from_numpy(w2).cuda().to(torch.bfloat16)
    with ExpertParallelMoE(g13, g2, experts, max_tokens=max_tokens, top_k=top_k) as layer:
        for tokens, routing in ((50, {}), (0, {}), (128, {"skew": True}), (1, {})):
            x = _tokens(rng, tokens, hidden)
            ids, w = _routing(rng, tokens, experts, top_k, **routing)
            out = layer(torch.from_numpy(x).cuda().to(torch.bfloat16), torch.from_numpy(ids).cuda(),
                        torch.from_numpy(w).cuda())
            layer.check_errors()
            if tokens:
                err = relative_frobenius(out.float().cpu().numpy(), oracle_moe.moe_layer(x, ids, w, w13, w2))
                assert err < BF16_TOL, (tokens, err)
        # Static buffers, one eager call, then capture and replay with new routing.
        tokens = 96
        sx = torch.empty((tokens, hidden), dtype=torch.bfloat16, device="cuda")
        sids = torch.empty((tokens, top_k), dtype=torch.int32, device="cuda")
        sw = torch.empty((tokens, top_k), dtype=torch.float32, device="cuda")
        sout = torch.empty((tokens, hidden), dtype=torch.bfloat16, device="cuda")
        x, (ids, w) = _tokens(rng, tokens, hidden), _routing(rng, tokens, experts, top_k)
        sx.copy_(torch.from_numpy(x)), sids.copy_(torch.from_numpy(ids)), sw.copy_(torch.from_numpy(w))
        layer(sx, sids, sw, sout)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
            layer(sx, sids, sw, sout)
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(2):
            x, (ids, w) = _tokens(rng, tokens, hidden), _routing(rng, tokens, experts, top_k, skew=True)
            sx.copy_(torch.from_numpy(x)), sids.copy_(torch.from_numpy(ids)), sw.copy_(torch.from_numpy(w))
            graph.replay()
            torch.cuda.synchronize()
            layer.check_errors()
            err = relative_frobenius(sout.float().cpu().numpy(), oracle_moe.moe_layer(x, ids, w, w13, w2))
            assert err < BF16_TOL, err
        del graph


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_capacity_overflow_is_reported_and_kept_rows_are_right():
    _setup_paths()
    from expert_parallel import ExpertParallelMoE

    tokens, experts, hidden, ffn, top_k = 64, 8, 256, 128, 2
    x, w13, w2, ids, w = _layer_case(3, tokens, experts, hidden, ffn, top_k)
    gx, g13, g2, gids, gw = _to_gpu(x, w13, w2, ids, w)
    capacity = 40
    with ExpertParallelMoE(g13, g2, experts, max_tokens=tokens, top_k=top_k, capacity=capacity) as layer:
        out = layer(gx, gids, gw)
        with pytest.raises(RuntimeError, match="capacity"):
            layer.check_errors()
        # Rows land in expert order; slot (t, j) survives iff its row < capacity.
        position = layer.position[: tokens * top_k].cpu().numpy().reshape(tokens, top_k)
        send_base, _ = oracle_moe.ep_layout(oracle_moe.route_counts(ids, experts)[None, :], 0, capacity)
        kept = ids.copy()
        kept[send_base[ids] + position >= capacity] = -1
        err = relative_frobenius(out.float().cpu().numpy(), oracle_moe.moe_layer(x, kept, w, w13, w2))
        assert err < BF16_TOL, err


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_route_permute_combine_kernels():
    _setup_paths()
    from kernels import _native, launch_grouped_mm

    tokens, experts, hidden, ffn, top_k = 77, 8, 256, 128, 2
    x, w13, w2, ids, w = _layer_case(11, tokens, experts, hidden, ffn, top_k, drop=0.1)
    gx, g13, g2, gids, gw = _to_gpu(x, w13, w2, ids, w)
    stream = torch.cuda.current_stream().cuda_stream
    counts = torch.empty(experts, dtype=torch.int32, device="cuda")
    position = torch.empty(tokens * top_k, dtype=torch.int32, device="cuda")
    _native.route_layout(gids.data_ptr(), tokens, top_k, experts, counts.data_ptr(), position.data_ptr(), stream)
    expected_counts = oracle_moe.route_counts(ids, experts)
    assert counts.cpu().tolist() == expected_counts.tolist()
    pos = position.cpu().numpy().reshape(tokens, top_k)
    assert np.all(pos[ids < 0] == -1)
    for e in range(experts):
        assert sorted(pos[ids == e].tolist()) == list(range(expected_counts[e]))
    starts = torch.cumsum(counts, 0, dtype=torch.int32) - counts
    rows = int(expected_counts.sum())
    sorted_rows = torch.zeros((rows, hidden), dtype=torch.bfloat16, device="cuda")
    _native.permute(gx.data_ptr(), hidden, gids.data_ptr(), position.data_ptr(), starts.data_ptr(), tokens, top_k,
                    experts, hidden, sorted_rows.data_ptr(), hidden, 2, stream)
    host_sorted = sorted_rows.float().cpu().numpy()
    for (t, j), e in np.ndenumerate(ids):
        if e >= 0:
            assert np.array_equal(host_sorted[int(starts[e]) + pos[t, j]], x[t])
    offs = torch.cumsum(counts, 0, dtype=torch.int32)
    h = launch_grouped_mm(sorted_rows, g13, offs, swiglu=True)
    y = launch_grouped_mm(h, g2, offs)
    out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device="cuda")
    _native.combine(y.data_ptr(), hidden, gids.data_ptr(), gw.data_ptr(), position.data_ptr(), starts.data_ptr(),
                    tokens, top_k, experts, hidden, out.data_ptr(), hidden, stream)
    err = relative_frobenius(out.float().cpu().numpy(), oracle_moe.moe_layer(x, ids, w, w13, w2))
    assert err < BF16_TOL, err


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")
def test_peer_that_never_arrives_times_out_and_reports():
    """A two-rank configuration on one GPU whose second rank never runs (its
    region is a second local allocation nothing signals from): every barrier
    gives up after its 50 ms deadline and reports error bit 9, the exchange
    drops every slot instead of writing anywhere, and the context stays usable."""
    _setup_paths()
    from kernels import _native, launch_grouped_mm

    world, experts, hidden, top_k, tokens = 2, 4, 64, 2, 8
    slots = tokens * top_k
    capacity = world * slots
    layout = _native.ep_region_layout(world, experts, hidden, capacity, slots, 2)
    own, _ = _native.ep_shared_alloc(layout.bytes, with_handle=False)
    silent, _ = _native.ep_shared_alloc(layout.bytes, with_handle=False)
    try:
        _native.read_and_clear_error_word(0)
        peers = torch.tensor([own, silent], dtype=torch.int64, device="cuda")
        cfg = _native.EpConfig(0, world, experts, 2, hidden, capacity, 50_000_000, slots)
        gen = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn((tokens, hidden), device="cuda", generator=gen).to(torch.bfloat16)
        ids = torch.randint(0, experts, (tokens, top_k), device="cuda", generator=gen, dtype=torch.int32)
        w = torch.rand((tokens, top_k), device="cuda", generator=gen)
        counts = torch.zeros(experts, dtype=torch.int32, device="cuda")
        position = torch.empty(slots, dtype=torch.int32, device="cuda")
        out = torch.full((tokens, hidden), 7.0, dtype=torch.bfloat16, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        _native.route_layout(ids.data_ptr(), tokens, top_k, experts, counts.data_ptr(), position.data_ptr(), stream)
        _native.ep_exchange_counts(counts.data_ptr(), peers.data_ptr(), cfg, stream)
        _native.ep_dispatch(x.data_ptr(), hidden, ids.data_ptr(), position.data_ptr(), tokens, top_k,
                            peers.data_ptr(), cfg, stream)
        _native.ep_combine(ids.data_ptr(), w.data_ptr(), position.data_ptr(), tokens, top_k, peers.data_ptr(), cfg,
                           out.data_ptr(), hidden, stream)
        torch.cuda.synchronize()
        word = _native.read_and_clear_error_word(0)
        assert word & (1 << 9), _native.describe_error_word(word)
        assert torch.count_nonzero(out.float()) == 0, "a failed exchange must drop every slot"
        send_base = torch.as_tensor(_view_int32(own + layout.send_base, experts))
        assert torch.all(send_base == capacity)
        # The context still computes.
        a = torch.randn((96, 64), device="cuda", generator=gen).to(torch.bfloat16)
        b = torch.randn((2, 64, 128), device="cuda", generator=gen).to(torch.bfloat16)
        offs = torch.tensor([40, 96], dtype=torch.int32, device="cuda")
        got = launch_grouped_mm(a, b, offs)
        expected = torch.cat((a[:40].float() @ b[0].float(), a[40:].float() @ b[1].float()))
        assert torch.allclose(got.float(), expected, rtol=2e-2, atol=2e-2)
        assert _native.read_and_clear_error_word(0) == 0
    finally:
        torch.cuda.synchronize()
        _native.ep_shared_free(own)
        _native.ep_shared_free(silent)


def _view_int32(ptr, count):
    from expert_parallel import _view

    return _view(ptr, (count,), "<i4", torch.device("cuda", 0))


def _two_rank_worker(rank, world, port, result_dir):
    _setup_paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from expert_parallel import ExpertParallelMoE, NcclAllToAllMoE

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    experts, hidden, ffn, top_k, max_tokens = 16, 512, 256, 4, 160
    rng = np.random.default_rng(21)
    w13, w2 = _weights(rng, experts, hidden, ffn)
    local = experts // world
    mine = slice(rank * local, (rank + 1) * local)
    g13 = torch.from_numpy(w13[mine]).cuda().to(torch.bfloat16)
    g2 = torch.from_numpy(w2[mine]).cuda().to(torch.bfloat16)
    worst, lines = 0.0, []
    variants = ((ExpertParallelMoE, {"fused_return": True}), (ExpertParallelMoE, {"fused_return": False}),
                (NcclAllToAllMoE, {}))
    for cls, options in variants:
        with cls(g13, g2, experts, max_tokens=max_tokens, top_k=top_k, **options) as layer:
            for step, (tokens, routing) in enumerate(((120, {}), (160, {"skew": True}), (0 if rank else 33, {}),
                                                      (77, {"drop": 0.2}))):
                trng = np.random.default_rng(1000 * step + rank)
                x = _tokens(trng, tokens, hidden)
                ids, w = _routing(trng, tokens, experts, top_k, **routing)
                out = layer(torch.from_numpy(x).cuda().to(torch.bfloat16), torch.from_numpy(ids).cuda(),
                            torch.from_numpy(w).cuda())
                layer.check_errors()
                if tokens:
                    err = relative_frobenius(out.float().cpu().numpy(), oracle_moe.moe_layer(x, ids, w, w13, w2))
                    worst = max(worst, err)
                    lines.append(f"{cls.__name__} {options} step {step} tokens {tokens} err {err:.3e}")
    dist.destroy_process_group()
    Path(result_dir, f"rank{rank}.txt").write_text(f"{worst}\n" + "\n".join(lines))


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_dispatch_and_combine_over_peer_memory(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_two_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    for rank in range(2):
        text = (tmp_path / f"rank{rank}.txt").read_text()
        assert float(text.splitlines()[0]) < BF16_TOL, text
