"""EP / TP rank plans for an MoE expert layer, and reassembly of rank outputs.

The reference models one rank of a P-way expert-parallel (EP) or
tensor-parallel (TP) layer as a list of GEMM shapes (utils/metrics.py:40-72):

* EP rank r owns experts [r*E/P, (r+1)*E/P) with the full FFN width:
  W13 = [M_e, H] @ [H, 2F] (packed [gate | up]) and W2 = [M_e, F] @ [F, H].
* TP rank r owns every expert but only FFN columns [r*F/P, (r+1)*F/P) of W1
  and of W3, packed as [gate_r | up_r] (N = 2F/P), and the matching rows of
  W2 (K = F/P); a TP rank's W2 output is a partial sum.

Here every rank is a real process on its own GPU.  The timed region has no
collective; after timing, rank outputs are gathered (NCCL all_gather) and
reassembled by the functions below so rank 0 can check them against the
global product.
"""

from __future__ import annotations

from dataclasses import dataclass


def gemm_flops(m: int, k: int, n: int) -> int:
    """Useful FLOPs of one GEMM (utils/metrics.py:9-10)."""
    return 2 * m * k * n


def ideal_bytes(m: int, k: int, n: int, itemsize: int) -> int:
    """One-read / one-write traffic of one GEMM (utils/metrics.py:13-16)."""
    return itemsize * (m * k + k * n + m * n)


def moe_shapes(projection: str, parallel_type: str, m: int, hidden: int, ffn: int, experts: int,
               parallel_size: int) -> list[tuple[int, int, int]]:
    """One rank's (M, K, N) GEMMs after uniform routing (utils/metrics.py:40-72)."""
    if experts % parallel_size:
        raise ValueError("num_experts must be divisible by parallel_size")
    if ffn % parallel_size:
        raise ValueError("ffn_size must be divisible by parallel_size")
    if parallel_type not in ("EP", "TP"):
        raise ValueError(f"unknown parallel type {parallel_type}")
    local_experts = experts // parallel_size if parallel_type == "EP" else experts
    local_ffn = ffn if parallel_type == "EP" else ffn // parallel_size
    if projection == "W1":
        shape = (m, hidden, 2 * local_ffn)
    elif projection == "W2":
        shape = (m, local_ffn, hidden)
    else:
        raise ValueError(f"unknown projection {projection}")
    return [shape] * local_experts


def verify_ep_tp_flops(projection: str, m: int, hidden: int, ffn: int, experts: int, parallel_size: int) -> int:
    """EP and TP ranks do exactly the same useful work (utils/metrics.py:75-80)."""
    ep = sum(gemm_flops(*s) for s in moe_shapes(projection, "EP", m, hidden, ffn, experts, parallel_size))
    tp = sum(gemm_flops(*s) for s in moe_shapes(projection, "TP", m, hidden, ffn, experts, parallel_size))
    if ep != tp:
        raise ValueError(f"per-rank FLOPs differ: EP={ep}, TP={tp}")
    return ep


@dataclass(frozen=True)
class RankPlan:
    projection: str       # "W1" (packed W13 gate+up) or "W2" (down)
    parallel_type: str    # "EP" or "TP"
    rank: int
    parallel_size: int
    experts: tuple[int, ...]  # global expert ids this rank computes, in launch order
    ffn_slice: tuple[int, int]  # [start, stop) of the FFN dimension this rank holds
    ffn: int
    hidden: int

    @property
    def local_ffn(self) -> int:
        return self.ffn_slice[1] - self.ffn_slice[0]


def rank_plan(projection: str, parallel_type: str, rank: int, parallel_size: int, experts: int, ffn: int,
              hidden: int) -> RankPlan:
    if not 0 <= rank < parallel_size:
        raise ValueError(f"rank {rank} outside [0, {parallel_size})")
    moe_shapes(projection, parallel_type, 1, hidden, ffn, experts, parallel_size)  # divisibility checks
    if parallel_type == "EP":
        per = experts // parallel_size
        owned = tuple(range(rank * per, (rank + 1) * per))
        ffn_slice = (0, ffn)
    else:
        owned = tuple(range(experts))
        width = ffn // parallel_size
        ffn_slice = (rank * width, (rank + 1) * width)
    return RankPlan(projection, parallel_type, rank, parallel_size, owned, ffn_slice, ffn, hidden)


def shard_weight(global_weight, plan: RankPlan):
    """This rank's weight from one expert's global weight (any 2-D array type).

    W1: global [H, 2F] packed [gate | up] -> EP: itself; TP: [gate_r | up_r].
    W2: global [F, H] -> EP: itself; TP: rows of the rank's FFN slice.
    """
    start, stop = plan.ffn_slice
    f = plan.ffn
    if plan.parallel_type == "EP":
        return global_weight
    if plan.projection == "W1":
        gate = global_weight[:, start:stop]
        up = global_weight[:, f + start:f + stop]
        return _concat_columns(gate, up)
    return global_weight[start:stop, :]


def _concat_columns(left, right):
    try:
        import torch

        if isinstance(left, torch.Tensor):
            return torch.cat((left, right), dim=1).contiguous()
    except ImportError:
        pass
    import numpy as np

    return np.concatenate((left, right), axis=1)


def ep_owner(expert: int, parallel_size: int, experts: int) -> int:
    return expert // (experts // parallel_size)


def assemble_w13_tp(rank_outputs: list, parallel_size: int):
    """[gate | up] for the full FFN width from every TP rank's [gate_r | up_r]."""
    if len(rank_outputs) != parallel_size:
        raise ValueError("need one output per TP rank")
    width = rank_outputs[0].shape[1] // 2
    gates = [out[:, :width] for out in rank_outputs]
    ups = [out[:, width:] for out in rank_outputs]
    ordered = gates + ups
    result = ordered[0]
    for piece in ordered[1:]:
        result = _concat_columns(result, piece)
    return result


def assemble_w2_tp(rank_partials: list):
    """Full W2 output: the sum of every TP rank's partial product."""
    total = rank_partials[0]
    for part in rank_partials[1:]:
        total = total + part
    return total
