"""One rank of an expert-parallel (EP) MoE expert layer on B200.

The reference benchmarks one rank's expert GEMMs and models expert
parallelism only as the shapes a rank would see (utils/metrics.py:40-72);
routing, permutation and the all-to-all are outside its scope (README.md:14,
:35).  This module runs the whole layer around those GEMMs, one process per
GPU:

    route      moe_route_layout: slots per expert, each slot's position
    exchange   moe_ep_exchange_counts: counts to every rank over peer memory,
               then where each rank's rows land on each owner
    dispatch   moe_ep_dispatch: token rows copied straight into the owners'
               receive rows (one bulk shared -> global copy per slot over
               NVLink, sorted by local expert)
    W13        grouped GEMM, fused SiLU(gate) * up epilogue, over the receive
               rows in the aggregate layout (offs = per-expert row ends on the
               device, so no host synchronisation)
    W2         grouped GEMM whose epilogue stores every output row straight
               into the source rank's return rows (peer stores from the GEMM
               epilogue, row destinations from the origin table the dispatch
               wrote), so the return crosses NVLink while W2 still computes
    combine    moe_ep_combine: every token sums its k returned rows
               (local), weighted; with ``fused_return=False`` W2 writes the
               owner's out rows and the combine reads them (peer loads)

Rank r owns experts [r E / P, (r + 1) E / P) (utils/metrics.py:40-72 EP
split).  Each rank's region is a plain device allocation mapped by its peers
through CUDA IPC; handles travel once over the process group at construction.
With P = 1 the same kernels run locally (the single-GPU MoE layer).
"""

from __future__ import annotations

import math

try:
    import torch
    import torch.distributed as dist
except ImportError:  # pragma: no cover - host helpers stay importable
    torch = None
    dist = None

from kernels import _native
from kernels.grouped_gemm import check_device_errors, launch_grouped_mm, launch_grouped_mm_scatter
from kernels.matmul import KernelConfig, native_candidates


def ep_capacity(max_tokens: int, top_k: int, world: int) -> int:
    """Receive rows per rank that never drop a slot: every rank's tokens may
    all pick this rank's experts."""
    if max_tokens < 0 or top_k <= 0 or world <= 0:
        raise ValueError("max_tokens >= 0, top_k > 0 and world > 0 are required")
    return world * max_tokens * top_k


def expected_rows_per_expert(tokens: int, top_k: int, local_experts: int) -> int:
    """Average receive rows per local expert under uniform routing: every rank
    sends tokens * top_k slots, a rank receives P * tokens * top_k / E of them
    for each of its E / P experts."""
    return max(1, math.ceil(tokens * top_k / local_experts))


def exchange_handles(handle: bytes, rank: int, world: int, group=None) -> list[bytes]:
    """Every rank's IPC handle, in rank order (one all_gather_object)."""
    if world == 1:
        return [handle]
    gathered: list = [None] * world
    dist.all_gather_object(gathered, handle, group=group)
    if gathered[rank] != handle:
        raise RuntimeError("handle exchange returned another rank's handle in this rank's slot")
    return list(gathered)


class _DeviceArray:
    """Zero-copy view of raw device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3}


def _view(ptr: int, shape: tuple[int, ...], typestr: str, device):
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=device)


class ExpertParallelMoE:
    """This rank's share of an EP MoE expert layer.

    ``w13`` [E_l, H, 2F] (packed [gate | up] per local expert) and ``w2``
    [E_l, F, H], bf16 on this rank's GPU; ``num_experts`` global E = P * E_l.
    ``max_tokens`` bounds the tokens per forward on any rank; ``capacity``
    (receive rows, default ``ep_capacity``) may be set lower to save memory,
    in which case slots beyond it are dropped and reported.  ``group`` is the
    process group of the P ranks (None: the default group, or a single rank
    when torch.distributed is not initialised).  ``fused_return`` selects the
    W2 epilogue that returns rows to the source ranks (default) over the
    combine that pulls them.
    """

    def __init__(self, w13, w2, num_experts: int, *, max_tokens: int, top_k: int, group=None,
                 capacity: int | None = None, timeout_s: float = 10.0, fused_return: bool = True):
        if torch is None or not torch.cuda.is_available():
            raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
        _native.load()
        if w13.ndim != 3 or w2.ndim != 3:
            raise ValueError("expected w13 [E_l, H, 2F] and w2 [E_l, F, H]")
        local, hidden, two_f = w13.shape
        if w2.shape != (local, two_f // 2, hidden) or two_f % 2:
            raise ValueError(f"w2 must be [{local}, {two_f // 2}, {hidden}] for w13 {tuple(w13.shape)}")
        if w13.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
            raise ValueError("expert weights must be bfloat16")
        if w13.device != w2.device or not w13.is_cuda:
            raise ValueError("w13 and w2 must be on this rank's CUDA device")
        if dist is not None and dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        if num_experts != local * self.world:
            raise ValueError(f"num_experts {num_experts} != {self.world} ranks x {local} local experts")
        if self.world > _native.EP_MAX_WORLD:
            raise ValueError(f"at most {_native.EP_MAX_WORLD} ranks")
        self.group = group
        self.device = w13.device
        self.w13, self.w2 = w13.contiguous(), w2.contiguous()
        self.num_experts, self.local_experts = num_experts, local
        self.hidden, self.ffn = hidden, two_f // 2
        self.max_tokens, self.top_k = max_tokens, top_k
        self.capacity = ep_capacity(max_tokens, top_k, self.world) if capacity is None else int(capacity)
        self.max_slots = max_tokens * top_k
        self.fused_return = bool(fused_return)
        self.config = _native.EpConfig(self.rank, self.world, num_experts, 2, hidden, self.capacity,
                                       int(timeout_s * 1e9), self.max_slots)
        self.region = _native.ep_region_layout(self.world, num_experts, hidden, self.capacity, self.max_slots, 2)
        self._peer_ptrs: list[int] = []
        self._base = 0
        with torch.cuda.device(self.device):
            self._base, handle = _native.ep_shared_alloc(self.region.bytes, with_handle=self.world > 1)
            try:
                handles = exchange_handles(handle, self.rank, self.world, group)
                for r, h in enumerate(handles):
                    self._peer_ptrs.append(self._base if r == self.rank else _native.ep_peer_open(h))
            except Exception:
                self.close()
                raise
            self.peers = torch.tensor(self._peer_ptrs, dtype=torch.int64, device=self.device)
            rows = max(1, self.capacity)
            self.recv = _view(self._base + self.region.recv, (rows, hidden), "<i2", self.device).view(torch.bfloat16)
            self.out_rows = _view(self._base + self.region.out, (rows, hidden), "<i2", self.device).view(torch.bfloat16)
            self.recv_offs = _view(self._base + self.region.recv_offs, (local,), "<i4", self.device)
            self.send_base = _view(self._base + self.region.send_base, (num_experts,), "<i4", self.device)
            self.origin = _view(self._base + self.region.origin, (rows,), "<i8", self.device)
            self.hidden_rows = torch.empty((rows, self.ffn), dtype=torch.bfloat16, device=self.device)
            self.counts = torch.zeros(num_experts, dtype=torch.int32, device=self.device)
            self.position = torch.empty(max(1, max_tokens * top_k), dtype=torch.int32, device=self.device)

    def tile_configs(self, tokens: int) -> tuple[KernelConfig, KernelConfig]:
        """Native tiles of the two grouped GEMMs for `tokens` per rank."""
        rows = expected_rows_per_expert(tokens, self.top_k, self.local_experts)
        return (native_candidates(rows, self.hidden, split_tail=False)[0],
                native_candidates(rows, self.ffn, split_tail=False)[0])

    def forward(self, x, topk_ids, topk_weights, out=None, *, configs=None, phase_events=None):
        """out [T, H] bf16 = sum_j topk_weights[t, j] * expert_{topk_ids[t, j]}(x[t]).

        ``x`` [T, H] bf16, ``topk_ids`` [T, k] int32 (ids outside [0, E) are
        dropped), ``topk_weights`` [T, k] float32, all on this rank's GPU and
        contiguous.  Every rank must call forward the same number of times,
        with T = 0 too.  Launches only; ``check_device_errors`` reports
        barrier timeouts and dropped rows.  ``phase_events``: four CUDA events
        recorded after dispatch, W13, W2 and combine (phase timing)."""
        tokens = x.shape[0]
        if x.ndim != 2 or x.shape[1] != self.hidden or x.dtype != torch.bfloat16 or (tokens and x.stride(1) != 1):
            raise ValueError(f"x must be [T, {self.hidden}] bf16 with contiguous rows")
        if tuple(topk_ids.shape) != (tokens, self.top_k) or topk_ids.dtype != torch.int32:
            raise ValueError(f"topk_ids must be [{tokens}, {self.top_k}] int32")
        if tuple(topk_weights.shape) != (tokens, self.top_k) or topk_weights.dtype != torch.float32:
            raise ValueError(f"topk_weights must be [{tokens}, {self.top_k}] float32")
        if tokens and not (topk_ids.is_contiguous() and topk_weights.is_contiguous()):
            raise ValueError("topk_ids and topk_weights must be contiguous")
        if tokens > self.max_tokens:
            raise ValueError(f"{tokens} tokens exceed max_tokens={self.max_tokens}")
        if len({x.device, topk_ids.device, topk_weights.device, self.device}) != 1:
            raise ValueError("inputs must be on the layer's device")
        if out is None:
            out = torch.empty((tokens, self.hidden), dtype=torch.bfloat16, device=self.device)
        elif (tuple(out.shape) != (tokens, self.hidden) or out.dtype != torch.bfloat16 or
              (tokens and out.stride(1) != 1)):
            raise ValueError(f"out must be [{tokens}, {self.hidden}] bf16 with contiguous rows")
        cfg13, cfg2 = configs or self.tile_configs(tokens)
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _native.route_layout(topk_ids.data_ptr(), tokens, self.top_k, self.num_experts, self.counts.data_ptr(),
                                 self.position.data_ptr(), stream)
            _native.ep_exchange_counts(self.counts.data_ptr(), self.peers.data_ptr(), self.config, stream)
            x_pitch = x.stride(0) if tokens else self.hidden
            _native.ep_dispatch(x.data_ptr(), x_pitch, topk_ids.data_ptr(), self.position.data_ptr(), tokens,
                                self.top_k, self.peers.data_ptr(), self.config, stream)
            marks = list(phase_events or ())
            if marks:
                marks.pop(0).record()
            if self.capacity > 0:
                launch_grouped_mm(self.recv, self.w13, self.recv_offs, self.hidden_rows, swiglu=True, config=cfg13)
                if marks:
                    marks.pop(0).record()
                if self.fused_return:
                    launch_grouped_mm_scatter(self.hidden_rows, self.w2, self.recv_offs, self.origin, self.peers,
                                              self.region.ret, self.hidden * 2, config=cfg2)
                else:
                    launch_grouped_mm(self.hidden_rows, self.w2, self.recv_offs, self.out_rows, config=cfg2)
            elif marks:
                marks.pop(0).record()
            if marks:
                marks.pop(0).record()
            _native.ep_combine(topk_ids.data_ptr(), topk_weights.data_ptr(), self.position.data_ptr(), tokens,
                               self.top_k, self.peers.data_ptr(), self.config, out.data_ptr(),
                               out.stride(0) if tokens else self.hidden, stream,
                               returned=self.fused_return and self.capacity > 0)
            if marks:
                marks.pop(0).record()
        return out

    __call__ = forward

    def launches_per_forward(self) -> int:
        """Native kernels one forward launches: route (1), exchange (1),
        dispatch (1), two grouped GEMMs (map builder + GEMM each), barrier and
        combine (2); the route's counter reset is a memset, not a kernel."""
        return 3 + (4 if self.capacity > 0 else 0) + 2

    def check_errors(self) -> None:
        check_device_errors(self.device)

    def close(self) -> None:
        """Unmaps the peers' regions and frees this rank's (collective when P > 1)."""
        if not self._base:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            if self.world > 1 and dist.is_initialized():
                dist.barrier(group=self.group)
            for r, ptr in enumerate(self._peer_ptrs):
                if r != self.rank:
                    _native.ep_peer_close(ptr)
            self._peer_ptrs = []
            for name in ("recv", "out_rows", "recv_offs", "send_base", "origin"):
                self.__dict__.pop(name, None)
            _native.ep_shared_free(self._base)
            self._base = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class NcclAllToAllMoE:
    """The same layer with the exchange done by NCCL ``all_to_all_single`` --
    the library baseline the peer-memory path is measured against.

    Per forward: route and permute the slots into expert order (native
    kernels), all-to-all the per-expert counts, copy the split sizes to the
    host (the variable-split all-to-all needs them there), all-to-all the
    rows, regroup them from source-major to expert-major (one gather), the
    same two grouped GEMMs, the reverse gather and all-to-all, and the native
    weighted combine.  Same arguments and results as ExpertParallelMoE.
    """

    def __init__(self, w13, w2, num_experts: int, *, max_tokens: int, top_k: int, group=None):
        if torch is None or not torch.cuda.is_available():
            raise RuntimeError("CUDA PyTorch and the native sm_100a library are required")
        _native.load()
        local, hidden, two_f = w13.shape
        if w2.shape != (local, two_f // 2, hidden) or two_f % 2 or w13.dtype != torch.bfloat16:
            raise ValueError("expected bf16 w13 [E_l, H, 2F] and w2 [E_l, F, H]")
        if dist is not None and dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        if num_experts != local * self.world:
            raise ValueError(f"num_experts {num_experts} != {self.world} ranks x {local} local experts")
        self.group, self.device = group, w13.device
        self.w13, self.w2 = w13.contiguous(), w2.contiguous()
        self.num_experts, self.local_experts = num_experts, local
        self.hidden, self.ffn, self.top_k, self.max_tokens = hidden, two_f // 2, top_k, max_tokens
        self.counts = torch.zeros(num_experts, dtype=torch.int32, device=self.device)
        self.position = torch.empty(max(1, max_tokens * top_k), dtype=torch.int32, device=self.device)
        self.sorted_rows = torch.empty((max(1, max_tokens * top_k), hidden), dtype=torch.bfloat16, device=self.device)
        self.returned = torch.empty_like(self.sorted_rows)

    def tile_configs(self, tokens: int) -> tuple[KernelConfig, KernelConfig]:
        rows = expected_rows_per_expert(tokens, self.top_k, self.local_experts)
        return (native_candidates(rows, self.hidden, split_tail=False)[0],
                native_candidates(rows, self.ffn, split_tail=False)[0])

    def _all_to_all(self, out, inp, out_splits=None, in_splits=None):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x, topk_ids, topk_weights, out=None, *, configs=None, phase_events=None):
        tokens, k, E, El, P = x.shape[0], self.top_k, self.num_experts, self.local_experts, self.world
        if tokens > self.max_tokens or tuple(topk_ids.shape) != (tokens, k) or topk_ids.dtype != torch.int32:
            raise ValueError("x / topk_ids do not match the layer")
        if out is None:
            out = torch.empty((tokens, self.hidden), dtype=torch.bfloat16, device=self.device)
        cfg13, cfg2 = configs or self.tile_configs(tokens)
        marks = list(phase_events or ())
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _native.route_layout(topk_ids.data_ptr(), tokens, k, E, self.counts.data_ptr(),
                                 self.position.data_ptr(), stream)
            starts = torch.cumsum(self.counts, 0, dtype=torch.int32) - self.counts
            _native.permute(x.data_ptr(), x.stride(0) if tokens else self.hidden, topk_ids.data_ptr(),
                            self.position.data_ptr(), starts.data_ptr(), tokens, k, E, self.hidden,
                            self.sorted_rows.data_ptr(), self.hidden, 2, stream)
            recv_counts = torch.empty_like(self.counts)
            self._all_to_all(recv_counts, self.counts)
            splits = torch.stack((self.counts.view(P, El).sum(1), recv_counts.view(P, El).sum(1))).cpu()
            send_splits, recv_splits = splits[0].tolist(), splits[1].tolist()
            received = sum(recv_splits)
            recv_rows = torch.empty((received, self.hidden), dtype=torch.bfloat16, device=self.device)
            self._all_to_all(recv_rows, self.sorted_rows[: sum(send_splits)], recv_splits, send_splits)
            # Source-major [src][expert] segments -> expert-major rows.
            per = recv_counts.view(P, El).to(torch.int64)
            expert_start = torch.cumsum(per.sum(0), 0) - per.sum(0)
            src_before = torch.cumsum(per, 0) - per
            seg_dest = (expert_start[None, :] + src_before).reshape(-1)
            seg_src = (torch.cumsum(per.reshape(-1), 0) - per.reshape(-1))
            seg_len = per.reshape(-1)
            seg_of_row = torch.repeat_interleave(torch.arange(P * El, device=self.device), seg_len,
                                                 output_size=received)
            dest = seg_dest[seg_of_row] + torch.arange(received, device=self.device) - seg_src[seg_of_row]
            grouped = torch.empty_like(recv_rows)
            grouped.index_copy_(0, dest, recv_rows)
            offs = torch.cumsum(per.sum(0), 0).to(torch.int32)
            if marks:
                marks.pop(0).record()
            if received:
                h = launch_grouped_mm(grouped, self.w13, offs, swiglu=True, config=cfg13)
                if marks:
                    marks.pop(0).record()
                y = launch_grouped_mm(h, self.w2, offs, config=cfg2)
                if marks:
                    marks.pop(0).record()
                back = y.index_select(0, dest)
            else:
                for _ in range(2):
                    if marks:
                        marks.pop(0).record()
                back = recv_rows
            self._all_to_all(self.returned[: sum(send_splits)], back, send_splits, recv_splits)
            _native.combine(self.returned.data_ptr(), self.hidden, topk_ids.data_ptr(), topk_weights.data_ptr(),
                            self.position.data_ptr(), starts.data_ptr(), tokens, k, E, self.hidden,
                            out.data_ptr(), out.stride(0) if tokens else self.hidden, stream)
            if marks:
                marks.pop(0).record()
        return out

    __call__ = forward

    def check_errors(self) -> None:
        check_device_errors(self.device)

    def close(self) -> None:
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
