"""Float64 restatement of one MoE expert layer around the grouped GEMMs -- test
infrastructure only (tests, smoke, bench checks; never the product path).

The reference times the expert GEMMs alone: routing, token permutation and
the expert-parallel all-to-all are outside its scope (README.md:14, :35), and
SiLU(gate) * up is applied after its packed W13 GEMM outside the timed region
(README.md:55-57; the [gate | up] packing is kernels/grouped_gemm.py:575-594).
The layer built around those GEMMs computes, for token t routed to experts
e_t0 .. e_t(k-1) with weights w_tj,

    h_tj   = bf16( SiLU(x_t W13[e][:, :F]) * (x_t W13[e][:, F:]) )
    y_tj   = bf16( h_tj W2[e] )
    out[t] = bf16( sum_j w_tj * y_tj )

(bf16 intermediates because the fused W13 epilogue and the W2 GEMM store
bf16; slots whose expert id is outside [0, E) are dropped).  Parity for this
layer is unpinned against the reference, which has no such layer; the GEMM
pieces it is built from are pinned by the grouped GEMM fixtures.

``ep_layout`` restates where an expert-parallel rank's rows go: each owner's
receive rows are sorted by local expert, then by source rank.
"""

from __future__ import annotations

import numpy as np

from .gemm import bf16_round


def route_counts(topk_ids: np.ndarray, num_experts: int) -> np.ndarray:
    """Slots per expert (ids outside [0, E) dropped)."""
    ids = np.asarray(topk_ids).reshape(-1)
    kept = ids[(ids >= 0) & (ids < num_experts)]
    return np.bincount(kept, minlength=num_experts).astype(np.int64)


def ep_layout(counts_all: np.ndarray, rank: int, capacity: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """(send_base [E], recv_offs [E_l]) of `rank` from every rank's counts [world, E]:
    the slots of rank r for expert e start at (rows of e's lower-numbered local
    experts on the owner) + (rows of e from ranks below r); recv_offs are the
    cumulative row ends of this rank's local experts.  Both clamp at capacity."""
    counts_all = np.asarray(counts_all, dtype=np.int64)
    world, experts = counts_all.shape
    if experts % world:
        raise ValueError("experts must be a multiple of world")
    local = experts // world
    totals = counts_all.sum(axis=0)
    send_base = np.zeros(experts, dtype=np.int64)
    for e in range(experts):
        first = (e // local) * local
        send_base[e] = totals[first:e].sum() + counts_all[:rank, e].sum()
    mine = totals[rank * local:(rank + 1) * local]
    recv_offs = np.cumsum(mine)
    if capacity is not None:
        send_base = np.minimum(send_base, capacity)
        recv_offs = np.minimum(recv_offs, capacity)
    return send_base, recv_offs


def _silu(v: np.ndarray) -> np.ndarray:
    return v / (1.0 + np.exp(-v))


def moe_layer(x: np.ndarray, topk_ids: np.ndarray, topk_weights: np.ndarray, w13: np.ndarray,
              w2: np.ndarray) -> np.ndarray:
    """out [T, H] (float64 holding bf16 values) for x [T, H], topk_ids /
    topk_weights [T, k], w13 [E, H, 2F] packed [gate | up], w2 [E, F, H]."""
    x = np.asarray(x, dtype=np.float64)
    ids = np.asarray(topk_ids)
    weights = np.asarray(topk_weights, dtype=np.float64)
    experts, _, two_f = w13.shape
    half = two_f // 2
    tokens = x.shape[0]
    out = np.zeros((tokens, w2.shape[2]), dtype=np.float64)
    for e in range(experts):
        rows, slots = np.nonzero(ids == e)
        if rows.size == 0:
            continue
        xe = x[rows]
        b = np.asarray(w13[e], dtype=np.float64)
        h = bf16_round((_silu(xe @ b[:, :half]) * (xe @ b[:, half:])).astype(np.float32)).astype(np.float64)
        y = bf16_round((h @ np.asarray(w2[e], dtype=np.float64)).astype(np.float32)).astype(np.float64)
        np.add.at(out, rows, weights[rows, slots][:, None] * y)
    return bf16_round(out.astype(np.float32)).astype(np.float64)
