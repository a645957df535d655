"""Benchmark of the MoE expert grouped GEMM on B200 (one JSON line on rank 0).

Workload: DeepSeek-V3 (H = 7168, F = 2048, E = 256, top-8) P = 8 rank shapes
in bf16 for M_e in {16, 32, 64, 128, 256, 512, 1024}, both projections the
metric names:
  W13 gate+up, hot:  EP 32 x [M_e, 7168] @ [7168, 4096]
                     TP 256 x [M_e, 7168] @ [7168, 512]
  W2 down, rotating-cold (two resident workspace sets, step s runs set s % 2):
                     EP 32 x [M_e, 2048] @ [2048, 7168]
                     TP 256 x [M_e, 256] @ [256, 7168]   (partial sums)
A step is one pass of the hot path over that batch: 28 grouped launches, each
one launch_grouped call (kernels/grouped_gemm.py:618-760 in the reference).

With --gpus N (torchrun, one process per GPU) GPU r runs rank r of the P = 8
layout: per-GPU work is fixed (weak scaling) and the timed region holds no
collective.  After timing, rank outputs are all-gathered over NCCL and rank 0
checks EP expert outputs, TP W13 [gate_r | up_r] slices and TP W2 partial sums
against a float64 product of the global per-expert weights.

Inputs: A ~ N(0, 1), B ~ N(0, 1/sqrt(K)), seeded per global expert, so EP and
TP ranks hold consistent slices of one layer.  Weights (0.94-1.88 GB per
projection and parallel type) dwarf the 126 MB L2, so no flush is needed.

Beside the timed step: each launch alone next to torch.nn.functional.grouped_mm
on the same inputs (the reference's torch provider,
kernels/torch_grouped_gemm.py:162-174), end to end through launch_grouped with
host buffers, and the reference's host computation (per-expert torch.matmul,
benchmark_moe.py:259-266) on a bounded sample.

--impl reference times that host computation alone and prints the same line
with "impl": "reference".
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PACKAGE_DIR = ROOT / "moe-gemm-parallel-bench_b200"
for _p in (str(ROOT), str(PACKAGE_DIR)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

# MoE dimensions of the reference's bundled model configs (model_configs/*.json:
# hidden_size, moe_intermediate_size or intermediate_size, routed experts,
# experts per token) and the tokens-per-expert sweep BASELINE.json names for each.
MODELS = {
    "deepseek-v3": {"hidden": 7168, "ffn": 2048, "experts": 256, "topk": 8,
                    "m_values": (16, 32, 64, 128, 256, 512, 1024), "label": "DeepSeek-V3"},
    "mixtral-8x7b": {"hidden": 4096, "ffn": 14336, "experts": 8, "topk": 2, "m_values": (1024,),
                     "label": "Mixtral-8x7B"},
    "qwen3-235b-a22b": {"hidden": 4096, "ffn": 1536, "experts": 128, "topk": 8, "m_values": (16, 64, 256, 1024),
                        "label": "Qwen3-235B-A22B"},
}
MODEL = "deepseek-v3"
HIDDEN, FFN, EXPERTS, TOPK, PARALLEL = 7168, 2048, 256, 8, 8
M_VALUES = MODELS[MODEL]["m_values"]


def set_model(name: str, parallel: int) -> None:
    """Makes `name` (a MODELS key) and P = `parallel` the workload of this process."""
    global MODEL, HIDDEN, FFN, EXPERTS, TOPK, PARALLEL, M_VALUES
    if name not in MODELS:
        raise SystemExit(f"unknown --model {name!r}; one of {sorted(MODELS)}")
    spec = MODELS[name]
    if spec["experts"] % parallel or spec["ffn"] % parallel:
        raise SystemExit(f"--parallel-size {parallel} must divide {spec['experts']} experts and F = {spec['ffn']}")
    MODEL, PARALLEL = name, parallel
    HIDDEN, FFN, EXPERTS, TOPK = spec["hidden"], spec["ffn"], spec["experts"], spec["topk"]
    M_VALUES = spec["m_values"]
METRIC = "grouped-GEMM TFLOP/s per B200 (EP vs TP, W13 & W2) and % of roofline"
# Used only when MEASURED_PEAKS.json is absent: an earlier measurement on this
# pool (copy bandwidth; cuBLAS bf16 burst, and sustained at ~1.3 GHz under the
# 1 kW cap).
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                  "sm_max_mhz": 1965.0, "sustained_sm_mhz": 1300.0}
PROJECTION_NAME = {"W1": "W13", "W2": "W2"}


def workload_line(projection: str, m_values=None) -> str:
    """One projection's rank shapes under the current model and P."""
    label = MODELS[MODEL]["label"]
    ms = "{" + ",".join(str(m) for m in (m_values or M_VALUES)) + "}"
    ep, tp = EXPERTS // PARALLEL, EXPERTS
    if projection == "W1":
        return (f"{label} W13 gate+up bf16, P={PARALLEL} rank shapes: EP {ep} x [M_e,{HIDDEN}]@[{HIDDEN},{2 * FFN}] "
                f"and TP {tp} x [M_e,{HIDDEN}]@[{HIDDEN},{2 * FFN // PARALLEL}], M_e in {ms}")
    return (f"{label} W2 down bf16, P={PARALLEL} rank shapes: EP {ep} x [M_e,{FFN}]@[{FFN},{HIDDEN}] and "
            f"TP {tp} x [M_e,{FFN // PARALLEL}]@[{FFN // PARALLEL},{HIDDEN}] (partial sums), M_e in {ms}")


def projection_dims(projection: str) -> dict:
    """(K, N) of one expert GEMM per parallel type for a projection."""
    if projection == "W1":
        return {"EP": (HIDDEN, 2 * FFN), "TP": (HIDDEN, 2 * FFN // PARALLEL)}
    return {"EP": (FFN, HIDDEN), "TP": (FFN // PARALLEL, HIDDEN)}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("native", "reference", "reference-gpu"), default="native",
                   help="reference: the reference's CPU path (the driver's reference arm); reference-gpu: the "
                        "reference's own Triton grouped GEMM and torch grouped_mm provider on this GPU, per shape, "
                        "next to the native kernels on identical inputs (one line per projection)")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--skip-cpu-baseline", action="store_true")
    p.add_argument("--skip-grouped-mm", action="store_true",
                   help="leave out the per-shape torch grouped_mm side-by-side")
    p.add_argument("--m-values", type=str, default=None,
                   help="tokens per expert (default: the model's sweep from BASELINE.json)")
    p.add_argument("--model", choices=sorted(MODELS), default="deepseek-v3",
                   help="MoE dimensions: deepseek-v3 (configs[1]/[2], the benchmark line), mixtral-8x7b "
                        "(configs[3]), qwen3-235b-a22b (configs[4])")
    p.add_argument("--parallel-size", type=int, default=8,
                   help="P of the EP/TP layout; GPU r runs rank r of it")
    p.add_argument("--masked-sweep", action="store_true",
                   help="configs[4]'s masked single-GEMM sweep over {127,1000,4095,8191}^3 in fp32 (TF32 inputs "
                        "and full fp32 products) next to torch.mm, one JSON line")
    p.add_argument("--projection", choices=("both", "W1", "W2"), default="both",
                   help="both: W13 and W2 in one step (the benchmark line); W1: packed W13 gate+up only "
                        "(BASELINE configs[1]); W2: down projection only (configs[2])")
    p.add_argument("--cache-mode", choices=("default", "hot", "cold"), default="default",
                   help="default: W13 hot and W2 rotating-cold (configs[1] and [2]); hot: one workspace set; "
                        "cold: two resident workspace sets for every projection, alternated step by step")
    p.add_argument("--layout", choices=("tables", "aggregate"), default="tables",
                   help="W1: per-expert pointer tables (the reference's workspaces) or the expert-sorted "
                        "aggregate layout (launch_grouped_mm: A [E*M_e, K], B [E, K, N], int32 offsets)")
    p.add_argument("--fp8", action="store_true",
                   help="W1: e4m3 experts with DeepSeek-V3 block scales (grouped_gemm_fp8_launch, bf16 output)")
    p.add_argument("--fused-swiglu", action="store_true",
                   help="W1 only: launch with the fused SwiGLU epilogue (C = silu(gate) * up, [M_e, F_local])")
    p.add_argument("--parallel", type=str, default="EP,TP", help="subset of EP,TP to build and launch")
    p.add_argument("--expert-limit", type=int, default=None,
                   help="at most this many experts per workspace (smaller cases for ncu captures)")
    p.add_argument("--moe-layer", action="store_true",
                   help="time the whole expert-parallel MoE layer (route, dispatch, W13 SwiGLU, W2, combine)")
    p.add_argument("--layer-tokens", type=int, default=4096, help="tokens per rank for --moe-layer")
    p.add_argument("--layer-experts", type=int, default=EXPERTS,
                   help="global experts for --moe-layer (fewer: a smaller case for profiling)")
    p.add_argument("--ep-transport", choices=("peer", "peer-pull", "nccl"), default="peer",
                   help="--moe-layer exchange: peer-memory kernels with W2 returning rows from its epilogue, "
                        "peer-memory kernels with the combine pulling rows, or the NCCL all_to_all_single baseline")
    p.add_argument("--ref-providers", type=str, default="triton,torch_grouped_mm",
                   help="--impl reference-gpu: subset of triton,torch_grouped_mm to time beside the native launch")
    return p.parse_args(argv)


def load_peaks() -> tuple[dict, str]:
    """Roofline denominators: MEASURED_PEAKS.json (driver-written on this
    pool's B200s) or the fallback figures.  `sustained_sm_mhz` is the median
    SM clock under which the sustained bf16 figure was measured."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        peaks = {k: float(data[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}
        peaks["sm_max_mhz"] = float(data.get("sm_max_mhz") or FALLBACK_PEAKS["sm_max_mhz"])
        under_load = data.get("clocks_under_load") or {}
        peaks["sustained_sm_mhz"] = float(under_load.get("sm_mhz_median") or FALLBACK_PEAKS["sustained_sm_mhz"])
        return peaks, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def tensor_peak(peaks: dict, clocks: dict | None) -> tuple[float, str]:
    """Dense bf16 tensor peak that applies to a timed region, chosen from the
    SM clock sampled inside it.

    The burst figure (cuBLAS timed alone, boost clock) applies when the
    region's median clock is within 5% of the maximum; the sustained figure
    (seconds under the 1 kW cap) when the median is at or below the clock it
    was measured at; between the two, the linear interpolation in clock.
    Without a clock record the burst figure applies: it is the larger
    denominator, so the fraction is never overstated."""
    burst, sustained = peaks["bf16_tflops"], peaks["bf16_tflops_sustained"]
    hi = 0.95 * peaks.get("sm_max_mhz", FALLBACK_PEAKS["sm_max_mhz"])
    lo = peaks.get("sustained_sm_mhz", FALLBACK_PEAKS["sustained_sm_mhz"])
    mhz = (clocks or {}).get("sm_mhz")
    if not mhz:
        return burst, "burst (no clock record)"
    if mhz >= hi or hi <= lo:
        return burst, f"burst (timed-region median SM clock {mhz:.0f} MHz)"
    if mhz <= lo:
        return sustained, f"sustained (timed-region median SM clock {mhz:.0f} MHz <= {lo:.0f} MHz)"
    peak = sustained + (burst - sustained) * (mhz - lo) / (hi - lo)
    return peak, (f"interpolated between sustained ({lo:.0f} MHz) and burst ({hi:.0f} MHz) at the "
                  f"timed-region median SM clock {mhz:.0f} MHz")


def progress(message: str) -> None:
    """Progress markers on stderr (stdout carries only the JSON line)."""
    if os.environ.get("MGB_BENCH_VERBOSE"):
        print(f"[bench {time.strftime('%H:%M:%S')}] {message}", file=sys.stderr, flush=True)


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def step_shapes(m_values, projection: str = "W1") -> list[tuple[str, int, tuple[int, int, int], int]]:
    """(parallel_type, M_e, (M, K, N), experts) for the 14 launches of one
    projection's step."""
    from moe_parallel import moe_shapes

    out = []
    for m in m_values:
        for par in ("EP", "TP"):
            shapes = moe_shapes(projection, par, m, HIDDEN, FFN, EXPERTS, PARALLEL)
            out.append((par, m, shapes[0], len(shapes)))
    return out


def fp8_launch_bytes(m: int, k: int, n: int) -> int:
    """One read of e4m3 A and B, their fp32 block scales, one bf16 write of C."""
    kb, nb = -(-k // 128), -(-n // 128)
    return m * k + n * k + 4 * (m * kb + nb * kb) + 2 * m * n


def roofline_ms(m: int, k: int, n: int, count: int, peaks: dict, tc_peak: float | None = None,
                out_cols: int | None = None, fp8: bool = False) -> tuple[float, str]:
    """Roofline time of one launch: max(FLOPs / tensor peak, algorithmic bytes
    / HBM bandwidth) (utils/metrics.py:9-16).  `tc_peak` is the bf16 tensor
    peak in TFLOP/s (default: the burst figure); `out_cols` is C's width when
    it is not N (the fused SwiGLU epilogue writes N/2 columns).  FP8 launches
    count their e4m3 / scale / bf16 bytes and twice the bf16 tensor peak (the
    dense e4m3 rate of the tensor cores is twice the bf16 one)."""
    from moe_parallel import gemm_flops, ideal_bytes

    flops = gemm_flops(m, k, n) * count
    if fp8:
        nbytes = fp8_launch_bytes(m, k, n) * count
    elif out_cols is None:
        nbytes = ideal_bytes(m, k, n, 2) * count
    else:
        nbytes = 2 * (m * k + k * n + m * out_cols) * count
    peak = peaks["bf16_tflops"] if tc_peak is None else tc_peak
    tc = flops / ((2 * peak if fp8 else peak) * 1e12) * 1e3
    hbm = nbytes / (peaks["hbm_gbs"] * 1e9) * 1e3
    return (tc, "tensor") if tc >= hbm else (hbm, "hbm")


# ------------------------------------------------------------- clocks
NVML_REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
                0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}


def summarize_clock_samples(samples, window=None, interval_s: float | None = None) -> dict | None:
    """Clock record of a timed region from (time, sm_mhz, max_mhz, power_w,
    reason_bits) samples: median SM clock and power of the samples inside
    `window` (wall-clock bounds), every clock-event reason seen active there,
    and how many samples saw each."""
    inside = [s for s in samples if window is None or window[0] <= s[0] <= window[1]]
    rows = inside or list(samples)
    if not rows:
        return None
    counts = {name: sum(1 for s in rows if s[4] & bit) for bit, name in NVML_REASONS.items()}
    return {"sm_mhz": statistics.median(s[1] for s in rows), "sm_mhz_min": min(s[1] for s in rows),
            "sm_max_mhz": max(s[2] for s in rows), "reasons": sorted(n for n, c in counts.items() if c),
            "reason_samples": {n: c for n, c in counts.items() if c},
            "power_w_median": round(statistics.median(s[3] for s in rows), 1),
            "power_w_max": round(max(s[3] for s in rows), 1),
            "samples": len(rows), "samples_in_timed_region": len(inside),
            "source": "NVML" + (f", every {interval_s * 1e3:.0f} ms" if interval_s else "")}


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, polled through NVML
    on a background thread (every `interval_s`) while the timed region runs.
    Only samples inside the wall-clock window given to mark() count."""

    def __init__(self, device_index: int, interval_s: float = 0.005):
        self.device_index = device_index
        self.interval_s = interval_s
        self.samples: list[tuple[float, float, float, float, int]] = []
        self.window: tuple[float, float] | None = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self) -> bool:
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
            try:
                self._handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
            except pynvml.NVMLError:
                visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
                ids = [v for v in visible.split(",") if v.strip()]
                index = int(ids[self.device_index]) if ids and ids[self.device_index].isdigit() else self.device_index
                self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            return True
        except Exception:  # no NVML (CPU host) or no such device: no clock record
            self._nvml = None
            return False

    def _poll(self) -> None:
        nv, h = self._nvml, self._handle
        max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                power = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((time.time(), sm, max_mhz, power, reasons))
            except nv.NVMLError:
                pass
            self._stop.wait(self.interval_s)

    def start(self) -> None:
        if self._open():
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
            time.sleep(0.05)

    def mark(self, begin: float, end: float) -> None:
        """Wall-clock bounds of the timed region."""
        self.window = (begin, end)

    def stop(self) -> dict | None:
        if self._thread is None:
            return None
        self._stop.set()
        self._thread.join(timeout=5)
        return summarize_clock_samples(self.samples, self.window, self.interval_s)


# ------------------------------------------------------------- workload
def expert_weight(expert: int, device):
    """Global W13 weight of one expert, [H, 2F] = [gate | up], B ~ N(0, 1/sqrt(H))."""
    import torch

    gen = torch.Generator(device=device).manual_seed(1_000_003 * (expert + 1))
    w = torch.randn((HIDDEN, 2 * FFN), device=device, generator=gen, dtype=torch.float32)
    return w.mul_(1.0 / math.sqrt(HIDDEN)).to(torch.bfloat16)


@dataclass
class RankStep:
    """One projection's tensors on this rank: the grouped launches of a step
    (`workspaces`: (parallel, M_e, workspace)), their activations and outputs
    per M_e, and per launch the same operands in torch grouped_mm's layout
    (`stacks`: (parallel, M_e) -> (A [E * M_e, K], B [E, K, N], int32 offs))."""

    projection: str
    ep: object
    tp: object
    activations: dict
    outputs: dict
    workspaces: list
    stacks: dict = field(default_factory=dict)


def uniform_offsets(count: int, m: int, device):
    import torch

    return torch.arange(1, count + 1, device=device, dtype=torch.int32) * m


def build_rank(rank: int, m_values, device, parallel=("EP", "TP"), expert_limit=None, swiglu: bool = False
               ) -> RankStep:
    """Per-rank W13 tensors and the grouped workspaces of one step (14 by
    default).  With `swiglu` the outputs are the fused SwiGLU activations
    [M_e, F_local]."""
    import torch

    from kernels import workspace_from_tensors
    from moe_parallel import rank_plan, shard_weight

    ep = rank_plan("W1", "EP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    tp = rank_plan("W1", "TP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    ep_experts = ep.experts[:expert_limit] if expert_limit else ep.experts
    tp_experts = tp.experts[:expert_limit] if expert_limit else tp.experts
    w_ep = torch.empty((len(ep_experts), HIDDEN, 2 * FFN), device=device, dtype=torch.bfloat16) \
        if "EP" in parallel else None
    w_tp = torch.empty((len(tp_experts), HIDDEN, 2 * tp.local_ffn), device=device, dtype=torch.bfloat16) \
        if "TP" in parallel else None
    for e in range(EXPERTS):
        use_ep, use_tp = e in ep_experts and w_ep is not None, e in tp_experts and w_tp is not None
        if not (use_ep or use_tp):
            continue
        w = expert_weight(e, device)
        if use_ep:
            w_ep[ep_experts.index(e)].copy_(w)
        if use_tp:
            w_tp[tp_experts.index(e)].copy_(shard_weight(w, tp))
        del w
    step = RankStep("W1", ep, tp, {}, {}, [])
    width = 1 if swiglu else 2
    for m in m_values:
        gen = torch.Generator(device=device).manual_seed(7919 * m)
        a_all = torch.randn((EXPERTS, m, HIDDEN), device=device, generator=gen).to(torch.bfloat16)
        step.activations[m] = a_all
        c_ep = torch.empty((len(ep_experts), m, width * FFN), device=device, dtype=torch.bfloat16)
        c_tp = torch.empty((len(tp_experts), m, tp.local_ffn * width), device=device, dtype=torch.bfloat16)
        step.outputs[m] = (c_ep, c_tp)
        if w_ep is not None:
            ws_ep = workspace_from_tensors([a_all[e] for e in ep_experts], list(w_ep), list(c_ep), swiglu=swiglu)
            ws_ep.operation = "swiglu" if swiglu else "gate_up"
            step.workspaces.append(("EP", m, ws_ep))
            lo = ep_experts[0]
            step.stacks[("EP", m)] = (a_all[lo:lo + len(ep_experts)].reshape(-1, HIDDEN), w_ep,
                                      uniform_offsets(len(ep_experts), m, device))
        if w_tp is not None:
            ws_tp = workspace_from_tensors([a_all[e] for e in tp_experts], list(w_tp), list(c_tp), swiglu=swiglu)
            ws_tp.operation = "swiglu" if swiglu else "gate_up"
            step.workspaces.append(("TP", m, ws_tp))
            step.stacks[("TP", m)] = (a_all[:len(tp_experts)].reshape(-1, HIDDEN), w_tp,
                                      uniform_offsets(len(tp_experts), m, device))
    return step


def expert_down_weight(expert: int, device, seed: int = 0):
    """Global W2 (down) weight of one expert, [F, H], B ~ N(0, 1/sqrt(F))."""
    import torch

    gen = torch.Generator(device=device).manual_seed(2_000_029 * (expert + 1) + seed)
    w = torch.randn((FFN, HIDDEN), device=device, generator=gen, dtype=torch.float32)
    return w.mul_(1.0 / math.sqrt(FFN)).to(torch.bfloat16)


def expert_intermediate(expert: int, m: int, device, seed: int = 0):
    """Global W2 input of one expert (the SiLU(gate) * up activations), [M, F]."""
    import torch

    gen = torch.Generator(device=device).manual_seed(7919 * m + 104_729 * (expert + 1) + seed)
    return torch.randn((m, FFN), device=device, generator=gen).to(torch.bfloat16)


def build_rank_w2(rank: int, m_values, device, parallel=("EP", "TP"), expert_limit=None, seed: int = 0
                  ) -> RankStep:
    """W2 (down projection) rank tensors: EP experts with the full F, TP every
    expert with the rank's F/P slice (rows of W2, columns of the input), whose
    [M, 7168] outputs are partial sums."""
    import torch

    from kernels import workspace_from_tensors
    from moe_parallel import rank_plan, shard_weight

    ep = rank_plan("W2", "EP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    tp = rank_plan("W2", "TP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    ep_experts = ep.experts[:expert_limit] if expert_limit else ep.experts
    tp_experts = tp.experts[:expert_limit] if expert_limit else tp.experts
    lo, hi = tp.ffn_slice
    w_ep = torch.empty((len(ep_experts), FFN, HIDDEN), device=device, dtype=torch.bfloat16) \
        if "EP" in parallel else None
    w_tp = torch.empty((len(tp_experts), hi - lo, HIDDEN), device=device, dtype=torch.bfloat16) \
        if "TP" in parallel else None
    for e in range(EXPERTS):
        use_ep, use_tp = e in ep_experts and w_ep is not None, e in tp_experts and w_tp is not None
        if not (use_ep or use_tp):
            continue
        w = expert_down_weight(e, device, seed)
        if use_ep:
            w_ep[ep_experts.index(e)].copy_(w)
        if use_tp:
            w_tp[tp_experts.index(e)].copy_(shard_weight(w, tp))
        del w
    step = RankStep("W2", ep, tp, {}, {}, [])
    for m in m_values:
        a_ep = torch.empty((len(ep_experts), m, FFN), device=device, dtype=torch.bfloat16)
        a_tp = torch.empty((len(tp_experts), m, hi - lo), device=device, dtype=torch.bfloat16)
        for i, e in enumerate(tp_experts if w_tp is not None else ()):
            full = expert_intermediate(e, m, device, seed)
            a_tp[i].copy_(full[:, lo:hi])
        for i, e in enumerate(ep_experts if w_ep is not None else ()):
            a_ep[i].copy_(expert_intermediate(e, m, device, seed))
        step.activations[m] = [a_ep, a_tp]
        c_ep = torch.empty((len(ep_experts), m, HIDDEN), device=device, dtype=torch.bfloat16)
        c_tp = torch.empty((len(tp_experts), m, HIDDEN), device=device, dtype=torch.bfloat16)
        step.outputs[m] = (c_ep, c_tp)
        if w_ep is not None:
            ws_ep = workspace_from_tensors(list(a_ep), list(w_ep), list(c_ep))
            ws_ep.operation = "down"
            step.workspaces.append(("EP", m, ws_ep))
            step.stacks[("EP", m)] = (a_ep.view(-1, FFN), w_ep, uniform_offsets(len(ep_experts), m, device))
        if w_tp is not None:
            ws_tp = workspace_from_tensors(list(a_tp), list(w_tp), list(c_tp))
            ws_tp.operation = "down"
            step.workspaces.append(("TP", m, ws_tp))
            step.stacks[("TP", m)] = (a_tp.view(-1, hi - lo), w_tp, uniform_offsets(len(tp_experts), m, device))
    return step


def verify_w2_outputs(rank, world, ep, tp, outputs, device, m_values, seed: int = 0) -> dict:
    """W2 after timing: sampled rows of every rank's EP outputs and TP partial
    sums are all-gathered over NCCL; rank 0 checks EP rows against the full
    float64 product and rank r's TP partial against its F/P slice of it (with
    all 8 ranks present, the partials' sum against the full product too)."""
    import torch
    import torch.distributed as dist

    from moe_parallel import ep_owner

    per = EXPERTS // PARALLEL
    sampled = sorted({0, per - 1} | {r * per + (r % per) for r in range(world)})
    checks = [m_values[0], m_values[-1]]
    width = FFN // PARALLEL
    worst = 0.0
    for m in checks:
        rows = torch.tensor(sorted({0, m - 1, m // 2}), device=device)
        c_ep, c_tp = outputs[m]
        payload = torch.zeros((len(sampled), len(rows), 2 * HIDDEN), device=device, dtype=torch.float32)
        for i, e in enumerate(sampled):
            if ep_owner(e, PARALLEL, EXPERTS) == rank:
                payload[i, :, :HIDDEN] = c_ep[ep.experts.index(e)].index_select(0, rows).float()
            payload[i, :, HIDDEN:] = c_tp[e].index_select(0, rows).float()
        gathered = [torch.empty_like(payload) for _ in range(world)] if world > 1 else [payload]
        if world > 1:
            dist.all_gather(gathered, payload)
        if rank != 0:
            continue
        for i, e in enumerate(sampled):
            a = expert_intermediate(e, m, device, seed).index_select(0, rows).double()
            w = expert_down_weight(e, device, seed).double()
            full = a @ w
            owner = ep_owner(e, PARALLEL, EXPERTS)
            if owner < world:
                got = gathered[owner][i, :, :HIDDEN].double()
                worst = max(worst, float((got - full).norm() / full.norm()))
            for r in range(world):
                part = a[:, r * width:(r + 1) * width] @ w[r * width:(r + 1) * width]
                got = gathered[r][i, :, HIDDEN:].double()
                worst = max(worst, float((got - part).norm() / part.norm()))
            if world == PARALLEL:
                summed = sum(gathered[r][i, :, HIDDEN:].double() for r in range(world))
                worst = max(worst, float((summed - full).norm() / full.norm()))
    return {"checked_experts": sampled, "checked_m": checks, "max_rel_frobenius": worst, "passed": worst <= 1e-2}


class AggregateLaunch:
    """One launch_grouped_mm call of the step (expert-sorted aggregate layout),
    standing in for a grouped workspace: same shapes, counts and launch info."""

    def __init__(self, mat_a, mat_b, offs, out, shape, count, swiglu):
        self.mat_a, self.mat_b, self.offs, self.out = mat_a, mat_b, offs, out
        self.shapes = (shape,)
        self.problem_count = count
        self.max_m = shape[0]
        self.swiglu = swiglu
        self.config = None
        self.launch_info = None

    def run(self, config=None) -> None:
        from kernels import last_aggregate_launch_info, launch_grouped_mm

        launch_grouped_mm(self.mat_a, self.mat_b, self.offs, self.out, config=config, swiglu=self.swiglu)
        self.launch_info = last_aggregate_launch_info()
        self.config = config or "native policy"


def build_rank_aggregate(rank: int, m_values, device, parallel=("EP", "TP"), expert_limit=None,
                         swiglu: bool = False) -> RankStep:
    """W13 rank tensors in the expert-sorted aggregate layout: per M_e one
    activation block [E, M_e, 7168] (EP ranks use their experts' contiguous
    slice), stacked weights [E, 7168, N] and uniform int32 offsets."""
    import torch

    from moe_parallel import rank_plan, shard_weight

    ep = rank_plan("W1", "EP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    tp = rank_plan("W1", "TP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    ep_experts = ep.experts[:expert_limit] if expert_limit else ep.experts
    tp_experts = tp.experts[:expert_limit] if expert_limit else tp.experts
    w_ep = torch.empty((len(ep_experts), HIDDEN, 2 * FFN), device=device, dtype=torch.bfloat16) \
        if "EP" in parallel else None
    w_tp = torch.empty((len(tp_experts), HIDDEN, 2 * tp.local_ffn), device=device, dtype=torch.bfloat16) \
        if "TP" in parallel else None
    for e in range(EXPERTS):
        if not ((e in ep_experts and w_ep is not None) or (e in tp_experts and w_tp is not None)):
            continue
        w = expert_weight(e, device)
        if e in ep_experts and w_ep is not None:
            w_ep[ep_experts.index(e)].copy_(w)
        if e in tp_experts and w_tp is not None:
            w_tp[tp_experts.index(e)].copy_(shard_weight(w, tp))
        del w
    width = 1 if swiglu else 2
    step = RankStep("W1", ep, tp, {}, {}, [])
    activations, outputs, launches = step.activations, step.outputs, step.workspaces
    for m in m_values:
        gen = torch.Generator(device=device).manual_seed(7919 * m)
        a_all = torch.randn((EXPERTS, m, HIDDEN), device=device, generator=gen).to(torch.bfloat16)
        activations[m] = a_all
        c_ep = torch.empty((len(ep_experts), m, width * FFN), device=device, dtype=torch.bfloat16)
        c_tp = torch.empty((len(tp_experts), m, width * tp.local_ffn), device=device, dtype=torch.bfloat16)
        outputs[m] = (c_ep, c_tp)
        if w_ep is not None:
            lo = ep_experts[0]
            a_ep = a_all[lo:lo + len(ep_experts)].reshape(-1, HIDDEN)
            offs = torch.arange(1, len(ep_experts) + 1, device=device, dtype=torch.int32) * m
            launches.append(("EP", m, AggregateLaunch(a_ep, w_ep, offs, c_ep.view(-1, c_ep.shape[-1]),
                                                      (m, HIDDEN, 2 * FFN), len(ep_experts), swiglu)))
        if w_tp is not None:
            a_tp = a_all[:len(tp_experts)].reshape(-1, HIDDEN)
            offs = torch.arange(1, len(tp_experts) + 1, device=device, dtype=torch.int32) * m
            launches.append(("TP", m, AggregateLaunch(a_tp, w_tp, offs, c_tp.view(-1, c_tp.shape[-1]),
                                                      (m, HIDDEN, 2 * tp.local_ffn), len(tp_experts), swiglu)))
    return step


def build_rank_fp8(rank: int, m_values, device, parallel=("EP", "TP"), expert_limit=None) -> RankStep:
    """W13 rank tensors quantized to e4m3 with DeepSeek-V3 block scales: each
    expert's packed weight (the EP weight or the TP [gate_r | up_r] slice) is
    stored [N, K] and quantized per 128 x 128 block; the activations per token
    and 128-deep K block.  Outputs are bf16 [M_e, N]."""
    import torch

    from kernels import fp8_workspace_from_tensors, quantize_activations, quantize_weight
    from moe_parallel import rank_plan, shard_weight

    ep = rank_plan("W1", "EP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    tp = rank_plan("W1", "TP", rank, PARALLEL, EXPERTS, FFN, HIDDEN)
    ep_experts = ep.experts[:expert_limit] if expert_limit else ep.experts
    tp_experts = tp.experts[:expert_limit] if expert_limit else tp.experts
    weights = {"EP": {}, "TP": {}}
    for e in range(EXPERTS):
        use_ep, use_tp = e in ep_experts and "EP" in parallel, e in tp_experts and "TP" in parallel
        if not (use_ep or use_tp):
            continue
        w = expert_weight(e, device)
        if use_ep:
            weights["EP"][e] = quantize_weight(w.t())
        if use_tp:
            weights["TP"][e] = quantize_weight(shard_weight(w, tp).t())
        del w
    step = RankStep("W1", ep, tp, {}, {}, [])
    activations, outputs, workspaces = step.activations, step.outputs, step.workspaces
    for m in m_values:
        gen = torch.Generator(device=device).manual_seed(7919 * m)
        a_all = torch.randn((EXPERTS, m, HIDDEN), device=device, generator=gen).to(torch.bfloat16)
        qa, sa = quantize_activations(a_all.view(-1, HIDDEN))
        qa, sa = qa.view(EXPERTS, m, HIDDEN), sa.view(EXPERTS, m, -1)
        activations[m] = [qa, sa]
        c_ep = torch.empty((len(ep_experts), m, 2 * FFN), device=device, dtype=torch.bfloat16)
        c_tp = torch.empty((len(tp_experts), m, 2 * tp.local_ffn), device=device, dtype=torch.bfloat16)
        outputs[m] = (c_ep, c_tp)
        for par, experts, c in (("EP", ep_experts, c_ep), ("TP", tp_experts, c_tp)):
            if par not in parallel:
                continue
            ws = fp8_workspace_from_tensors([qa[e] for e in experts], [weights[par][e][0] for e in experts],
                                            [sa[e] for e in experts], [weights[par][e][1] for e in experts], list(c))
            workspaces.append((par, m, ws))
    return step


def verify_fp8_outputs(world, workspaces, m_values, device) -> dict:
    """After timing: every rank checks sampled experts and rows of its FP8
    launches against the float64 product of the dequantized operands; the
    worst relative error is max-reduced over the ranks."""
    import torch
    import torch.distributed as dist

    from kernels.fp8 import dequantize_activations, dequantize_weight

    worst = 0.0
    checks = {m_values[0], m_values[-1]}
    for par, m, ws in workspaces:
        if m not in checks:
            continue
        for e in sorted({0, ws.problem_count - 1}):
            rows = torch.tensor(sorted({0, m // 2, m - 1}), device=device)
            a = dequantize_activations(ws.a[e].index_select(0, rows), ws.sa[e].index_select(0, rows)).double()
            b = dequantize_weight(ws.b[e], ws.sb[e]).double()
            ref = a @ b.t()
            got = ws.c[e].index_select(0, rows).double()
            worst = max(worst, float((got - ref).norm() / ref.norm()))
    t = torch.tensor([worst], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    worst = float(t.item())
    return {"checked_m": sorted(checks), "max_rel_frobenius": worst, "passed": worst <= 1e-2,
            "reference": "float64 product of the dequantized e4m3 operands"}


def launch(ws) -> None:
    """One launch of the step through the public API, with the native tile
    policy (launch_grouped's autotune=True path)."""
    from kernels import launch_grouped

    if isinstance(ws, AggregateLaunch):
        ws.run()
    elif getattr(ws, "operation", "") == "fp8_block_scaled":
        from kernels import launch_grouped_fp8

        launch_grouped_fp8(ws)
    else:
        launch_grouped(ws)


def graph_of_steps(rings, steps: int, stream, first_step: int = 0):
    """One CUDA graph holding `steps` passes of the step's launches, with an
    event pair around every launch (read after the timed replay).  `rings`
    holds one or two lists of (projection, parallel, M_e, workspace); step s
    launches rings[s % len(rings)] (rotating-cold alternates two resident
    workspace sets)."""
    import torch

    events = []
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for step in range(first_step, first_step + steps):
            for proj, par, m, ws in rings[step % len(rings)]:
                start = torch.cuda.Event(enable_timing=True, external=True)
                end = torch.cuda.Event(enable_timing=True, external=True)
                start.record()
                launch(ws)
                end.record()
                events.append((proj, par, m, start, end))
    return graph, events


def step_graphs(rings, steps: int, stream):
    """Graphs that together replay exactly `steps` steps: (graphs, replay
    order, events).  One graph of `chunk` steps replayed steps / chunk times;
    with two rings and an odd step count, two one-step graphs alternated."""
    if len(rings) == 1 or steps % 2 == 0:
        chunk = max(d for d in range(1, 11) if steps % d == 0 and (len(rings) == 1 or d % 2 == 0))
        graph, events = graph_of_steps(rings, chunk, stream)
        return [graph], [0] * (steps // chunk), events
    graphs, events = [], []
    for phase in range(2):
        graph, ev = graph_of_steps(rings, 1, stream, first_step=phase)
        graphs.append(graph)
        events += ev
    return graphs, [s % 2 for s in range(steps)], events


def verify_rank_outputs(rank, world, ep, tp, activations, outputs, device, m_values, swiglu: bool = False) -> dict:
    """After timing: NCCL all_gather of sampled output rows from every rank;
    rank 0 checks EP expert rows and TP [gate_r | up_r] slices against the
    float64 product of the global weights (regenerated for sampled experts).
    With `swiglu` the outputs are silu(gate) * up: EP rows against the full
    activation, TP rank r against its F/P column slice of it."""
    import torch
    import torch.distributed as dist

    from moe_parallel import ep_owner

    per = EXPERTS // PARALLEL
    sampled_experts = sorted({0, per - 1} | {r * per + (r % per) for r in range(world)})
    rows_idx = {m: sorted({0, m - 1, m // 2}) for m in m_values}
    checks = [m_values[0], m_values[-1]]
    ep_w, tp_w = (FFN, tp.local_ffn) if swiglu else (2 * FFN, 2 * tp.local_ffn)
    width = ep_w + tp_w
    worst = 0.0
    for m in checks:
        rows = torch.tensor(rows_idx[m], device=device)
        c_ep, c_tp = outputs[m]
        payload = torch.zeros((len(sampled_experts), len(rows), width), device=device, dtype=torch.float32)
        for i, e in enumerate(sampled_experts):
            if ep_owner(e, PARALLEL, EXPERTS) == rank:
                payload[i, :, :ep_w] = c_ep[ep.experts.index(e)].index_select(0, rows).float()
            payload[i, :, ep_w:] = c_tp[e].index_select(0, rows).float()
        gathered = [torch.empty_like(payload) for _ in range(world)] if world > 1 else [payload]
        if world > 1:
            dist.all_gather(gathered, payload)
        if rank != 0:
            continue
        local = tp.local_ffn
        for i, e in enumerate(sampled_experts):
            ref = activations[m][e].index_select(0, rows).double() @ expert_weight(e, device).double()
            if swiglu:
                gate, up = ref[:, :FFN], ref[:, FFN:]
                ref = gate / (1.0 + torch.exp(-gate)) * up
            owner = ep_owner(e, PARALLEL, EXPERTS)
            if owner < world:
                got = gathered[owner][i, :, :ep_w].double()
                worst = max(worst, float((got - ref).norm() / ref.norm()))
            for r in range(world):
                if swiglu:
                    sl = ref[:, r * local:(r + 1) * local]
                else:
                    sl = torch.cat((ref[:, r * local:(r + 1) * local], ref[:, FFN + r * local:FFN + (r + 1) * local]), 1)
                got = gathered[r][i, :, ep_w:].double()
                worst = max(worst, float((got - sl).norm() / sl.norm()))
    return {"checked_experts": sampled_experts, "checked_m": checks, "max_rel_frobenius": worst,
            "passed": worst <= 1e-2}


# ------------------------------------------------------------- CPU leg
def m_values_of(args) -> list[int]:
    """Tokens per expert of the run: --m-values, else the model's sweep."""
    return [int(v) for v in args.m_values.split(",")] if args.m_values else list(M_VALUES)


def selected_projections(args) -> tuple[str, ...]:
    """Projections of the step: both by default (the metric names W13 and W2);
    the W13-only modes (--fp8, --fused-swiglu, --layout aggregate) run W1."""
    w13_only = args.fp8 or args.fused_swiglu or args.layout == "aggregate"
    if args.projection == "both":
        return ("W1",) if w13_only else ("W1", "W2")
    if w13_only and args.projection != "W1":
        raise SystemExit("--fp8 / --fused-swiglu / --layout aggregate apply to the W1 (packed gate+up) projection")
    return (args.projection,)


def cold_projections(args, projections) -> tuple[str, ...]:
    """Projections that alternate two resident workspace sets step by step."""
    if args.cache_mode == "hot":
        return ()
    if args.cache_mode == "cold":
        return tuple(projections)
    return tuple(p for p in projections if p == "W2")


def workload_text(projections, cold=(), m_values=None) -> str:
    parts = []
    for proj in projections:
        mode = "rotating-cold (two resident workspace sets, step s runs set s % 2)" if proj in cold else "hot"
        parts.append(f"{workload_line(proj, m_values)}, {mode}")
    launches = 2 * len(m_values or M_VALUES) * len(projections)
    return "; ".join(parts) + f"; one step = {launches} grouped launches"


def cpu_problems(m_values, experts_per_launch: int, seed: int, projections=("W1",)):
    """Host bf16 problems for a sample of the step: `experts_per_launch`
    experts of every launch shape; weights are shared across the M_e values."""
    import torch

    gen = torch.Generator().manual_seed(seed)
    a_list, b_list = [], []
    for projection in projections:
        dims = projection_dims(projection)
        weights = {par: [(torch.randn((k, n), generator=gen) / math.sqrt(k)).to(torch.bfloat16)
                         for _ in range(experts_per_launch)] for par, (k, n) in dims.items()}
        for m in m_values:
            for par, (k, _n) in dims.items():
                acts = torch.randn((experts_per_launch, m, k), generator=gen).to(torch.bfloat16)
                for j in range(experts_per_launch):
                    a_list.append(acts[j])
                    b_list.append(weights[par][j])
    return a_list, b_list


def time_cpu(m_values, experts_per_launch: int, passes: int, budget_s: float, projections=("W1",)) -> dict:
    import torch

    from oracle.cpu_baseline import host_threads, per_expert_mm

    a_list, b_list = cpu_problems(m_values, experts_per_launch, seed=5, projections=projections)
    threads = host_threads()
    torch.set_num_threads(threads)
    per_expert_mm(a_list, b_list)  # warm-up pass
    flops = sum(2 * a.shape[0] * a.shape[1] * b.shape[1] for a, b in zip(a_list, b_list))
    samples = []
    start_all = time.perf_counter()
    for _ in range(max(1, passes)):
        t0 = time.perf_counter()
        per_expert_mm(a_list, b_list)
        samples.append(time.perf_counter() - t0)
        if time.perf_counter() - start_all > budget_s:
            break
    median = statistics.median(samples)
    shapes = 14 * len(projections)
    return {"value": round(flops / median / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": (f"per-expert torch.matmul (benchmark_moe.py:259-266) on host bf16 tensors, "
                       f"{experts_per_launch} expert(s) of each of the step's {shapes} launch shapes "
                       f"({len(a_list)} GEMMs, {flops / 1e9:.1f} GFLOP per pass), median of {len(samples)} passes"),
            "seconds_per_pass": median}


def reference_arm(args, rank: int, world: int) -> None:
    """The reference's host computation of the path (per-expert torch.matmul),
    one expert of each launch shape per step, every host thread."""
    if rank != 0:
        return
    import torch

    from oracle.cpu_baseline import host_threads, per_expert_mm

    m_values = m_values_of(args)
    projections = selected_projections(args)
    threads = host_threads()
    torch.set_num_threads(threads)
    a_list, b_list = cpu_problems(m_values, 1, seed=11, projections=projections)
    flops = sum(2 * a.shape[0] * a.shape[1] * b.shape[1] for a, b in zip(a_list, b_list))
    for _ in range(args.warmup):
        per_expert_mm(a_list, b_list)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        per_expert_mm(a_list, b_list)
    elapsed = time.perf_counter() - t0
    value = flops * args.steps / elapsed / 1e12
    sample = (f"per-expert torch.matmul (benchmark_moe.py:259-266) on host bf16 tensors, one expert of each of "
              f"the step's {14 * len(projections)} launch shapes ({len(a_list)} GEMMs, "
              f"{flops / 1e9:.1f} GFLOP per step)")
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload_text(projections, cold_projections(args, projections), m_values),
                   "sample": sample,
                   "parallelism": "host CPU, rank 0 only"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- main
LAYER_WORKLOAD = ("DeepSeek-V3 MoE expert layer bf16 (H=7168, F=2048, E=256 experts split over the ranks, top-8): "
                  "per rank T tokens routed uniformly at random; one step = route + count exchange + dispatch "
                  "(peer stores) + W13 grouped GEMM with fused SwiGLU + W2 grouped GEMM + weighted combine "
                  "(peer loads)")


def layer_reference(x, ids, weights, device):
    """fp32 reference of the layer for a few tokens from regenerated global
    expert weights (bf16 intermediates as the layer stores them)."""
    import torch

    out = torch.zeros((x.shape[0], HIDDEN), dtype=torch.float32, device=device)
    for t in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            w13 = expert_weight(e, device).float()
            w2 = expert_down_weight(e, device).float()
            xt = x[t:t + 1].float()
            gate, up = xt @ w13[:, :FFN], xt @ w13[:, FFN:]
            h = (torch.nn.functional.silu(gate) * up).to(torch.bfloat16).float()
            out[t] += float(weights[t, j]) * (h @ w2).to(torch.bfloat16).float()[0]
    return out.to(torch.bfloat16).float()


def moe_layer_bench(args, rank: int, world: int, local_rank: int, device) -> None:
    """--moe-layer: the whole EP layer per step, one JSON line on rank 0."""
    import torch
    import torch.distributed as dist

    from expert_parallel import ExpertParallelMoE, NcclAllToAllMoE
    from kernels import check_device_errors

    peaks, peak_source = load_peaks()
    tokens, top_k, experts = args.layer_tokens, TOPK, args.layer_experts
    if experts % world or experts < top_k:
        raise SystemExit("--layer-experts must be a multiple of the ranks and at least top-k")
    local = experts // world
    progress(f"building {local} local experts")
    w13 = torch.empty((local, HIDDEN, 2 * FFN), dtype=torch.bfloat16, device=device)
    w2 = torch.empty((local, FFN, HIDDEN), dtype=torch.bfloat16, device=device)
    for i in range(local):
        w13[i] = expert_weight(rank * local + i, device)
        w2[i] = expert_down_weight(rank * local + i, device)
    gen = torch.Generator(device=device).manual_seed(31337 + rank)
    x = torch.randn((tokens, HIDDEN), device=device, generator=gen).to(torch.bfloat16)
    scores = torch.rand((tokens, experts), device=device, generator=gen)
    top = scores.topk(top_k, dim=1)
    ids = top.indices.to(torch.int32).contiguous()
    weights = torch.softmax(top.values, dim=1).float().contiguous()
    out = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=device)
    if args.ep_transport == "nccl":
        layer = NcclAllToAllMoE(w13, w2, experts, max_tokens=tokens, top_k=top_k)
    else:
        layer = ExpertParallelMoE(w13, w2, experts, max_tokens=tokens, top_k=top_k,
                                  fused_return=args.ep_transport == "peer")
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    progress(f"tiles {layer.tile_configs(tokens)}")
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            layer(x, ids, weights, out)
    stream.synchronize()
    check_device_errors(local_rank)

    sampler = ClockSampler(local_rank)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall_begin = time.time()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            layer(x, ids, weights, out)
        end.record(stream)
    torch.cuda.synchronize(device)
    sampler.mark(wall_begin, time.time())
    clocks = sampler.stop()
    elapsed = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    max_ms = float(elapsed.item())
    check_device_errors(local_rank)

    # Phase split from a few more steps (dispatch incl. route and exchange,
    # W13, W2, combine incl. its barrier).
    phases = {"dispatch": [], "w13": [], "w2": [], "combine": []}
    with torch.cuda.stream(stream):
        for _ in range(5):
            begin = torch.cuda.Event(enable_timing=True)
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            begin.record(stream)
            layer(x, ids, weights, out, phase_events=marks)
            stream.synchronize()
            prev = begin
            for name, ev in zip(phases, marks):
                phases[name].append(prev.elapsed_time(ev))
                prev = ev
    phase_ms = {k: round(statistics.median(v), 4) for k, v in phases.items()}

    progress("end-to-end pass")
    host_x = torch.empty(x.shape, dtype=x.dtype, pin_memory=True).copy_(x)
    host_ids = torch.empty(ids.shape, dtype=ids.dtype, pin_memory=True).copy_(ids)
    host_w = torch.empty(weights.shape, dtype=weights.dtype, pin_memory=True).copy_(weights)
    host_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    e2e_steps = max(1, args.e2e_steps)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e_start.record(stream)
        for _ in range(e2e_steps):
            x.copy_(host_x, non_blocking=True)
            ids.copy_(host_ids, non_blocking=True)
            weights.copy_(host_w, non_blocking=True)
            layer(x, ids, weights, out)
            host_out.copy_(out, non_blocking=True)
        e_end.record(stream)
    torch.cuda.synchronize(device)
    e2e_t = torch.tensor([e_start.elapsed_time(e_end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_t.item())
    check_device_errors(local_rank)

    progress("verification")
    sample = torch.arange(0, tokens, max(1, tokens // 8), device=device)[:8]
    expected = layer_reference(x[sample], ids[sample].cpu(), weights[sample].cpu(), device)
    got = out[sample].float()
    err = torch.tensor([float((got - expected).norm() / expected.norm().clamp_min(1e-30))], device=device,
                       dtype=torch.float64)
    if world > 1:
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    # Native kernels per forward; the NCCL baseline adds torch and NCCL kernels
    # (cumsum, index gather / scatter, all-to-alls) that are not counted.
    launches = (7 if args.ep_transport == "nccl" else layer.launches_per_forward()) * args.steps
    layer.close()

    if rank == 0:
        slots = tokens * top_k
        step_flops = world * slots * 2 * (HIDDEN * 2 * FFN + FFN * HIDDEN)
        value = step_flops * args.steps / (max_ms * 1e-3) / 1e12
        ms_step = max_ms / args.steps
        gemm_ms = phase_ms["w13"] + phase_ms["w2"]
        tc_peak, tc_source = tensor_peak(peaks, clocks)
        # Per rank and GEMM: FLOPs on the tensor cores, or the expert weights
        # plus input and output rows through HBM, whichever takes longer.
        rows = slots  # rows a rank receives under uniform routing
        gemm_flops = rows * 2 * (HIDDEN * 2 * FFN + FFN * HIDDEN)
        gemm_bytes = 2 * (local * (HIDDEN * 2 * FFN + FFN * HIDDEN) + rows * (HIDDEN + FFN) * 2)
        t_tensor = gemm_flops / (tc_peak * 1e12)
        t_hbm = gemm_bytes / (peaks["hbm_gbs"] * 1e9)
        bound = "tensor" if t_tensor >= t_hbm else "hbm"
        if bound == "tensor":
            achieved, peak, unit = gemm_flops / (gemm_ms * 1e-3) / 1e12, tc_peak, "TFLOP/s"
        else:
            achieved, peak, unit = gemm_bytes / (gemm_ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
        moved = slots * HIDDEN * 2
        line = {
            "metric": "MoE expert layer TFLOP/s (route + dispatch + W13 SwiGLU + W2 + combine), whole job",
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded tokens, uniform "
            "random top-8 routing, random-init expert weights)",
            "config": {"workload": LAYER_WORKLOAD, "tokens_per_rank": tokens, "experts": experts,
                       "experts_per_rank": local,
                       "exchange": {"peer": "peer-memory dispatch kernel; W2 epilogue stores rows back to the "
                                            "source ranks (NVLink stores); local combine",
                                    "peer-pull": "peer-memory dispatch kernel; combine loads rows from the owners "
                                                 "(NVLink loads)",
                                    "nccl": "NCCL all_to_all_single (baseline; host sync for split sizes)"}[
                                        args.ep_transport],
                       "rows_per_expert_avg": slots / local, "parallelism": f"ep{world}",
                       "l2": "weights (2.8 GB per 32 experts) exceed L2; no flush"},
            "phases_ms": phase_ms,
            "roofline": {"bound": bound, "kernel": "W13 + W2 grouped GEMMs", "achieved": round(achieved, 1),
                         "peak": peak, "unit": unit, "frac": round(achieved / peak, 3),
                         "peak_source": f"{peak_source} {tc_source}" if bound == "tensor" else peak_source,
                         "traffic": None,
                         "gemm_share": round(gemm_ms / sum(phase_ms.values()), 3),
                         "gemm_roofline_ms": round(max(t_tensor, t_hbm) * 1e3, 4)},
            "exchange": {"dispatch_gbs": round(moved / (phase_ms["dispatch"] * 1e-3) / 1e9, 1),
                         "combine_gbs": round(moved / (phase_ms["combine"] * 1e-3) / 1e9, 1),
                         "bytes_per_rank": moved},
            "e2e": {"value": round(step_flops * e2e_steps / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": host_x.numel() * 2 + host_ids.numel() * 4 + host_w.numel() * 4,
                    "d2h_bytes_per_step": host_out.numel() * 2},
            "gpu_launches": launches, "clocks": clocks,
            "verify": {"sampled_tokens": int(sample.numel()), "max_rel_err": float(err.item()), "tol": 1e-2,
                       "ok": float(err.item()) < 1e-2},
        }
        print(json.dumps(line), flush=True)


REF_DIR = ROOT / "baseline" / "_ref"


def load_reference_package():
    """The unmodified reference's `kernels` package from baseline/_ref,
    imported as `refkernels` so it sits beside this package's `kernels`
    (its modules import `utils.benchmark`, found on baseline/_ref)."""
    import importlib.util

    init = REF_DIR / "kernels" / "__init__.py"
    if not init.exists():
        raise FileNotFoundError(f"{init} is missing (install the reference into baseline/_ref)")
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    spec = importlib.util.spec_from_file_location("refkernels", init, submodule_search_locations=[str(init.parent)])
    module = importlib.util.module_from_spec(spec)
    sys.modules["refkernels"] = module
    spec.loader.exec_module(module)
    return module


def reference_gpu_arm(args, rank: int, world: int) -> None:
    """--impl reference-gpu: per step shape, the reference's Triton persistent
    grouped GEMM (its launch_grouped with its hot autotune,
    kernels/grouped_gemm.py:618-760) and its torch.nn.functional.grouped_mm
    provider (kernels/torch_grouped_gemm.py:121-176), both from the unmodified
    reference in baseline/_ref, next to this package's native launch on the
    same seeded inputs (the reference's build_grouped_workspace draw, restated
    by kernels.build_grouped_workspace).  Native and Triton outputs are compared
    (relative Frobenius).  Rank 0 only; one JSON line per projection, each with
    the clock record of its run."""
    if rank != 0:
        return
    import torch

    torch.cuda.set_device(0)
    try:
        ref = load_reference_package()
    except Exception as exc:  # the reference is not installed or does not import here
        print(json.dumps({"impl": "reference-gpu", "unavailable": f"{type(exc).__name__}: {exc}"}))
        return
    from kernels import build_grouped_workspace, check_device_errors, launch_grouped

    m_values = m_values_of(args)
    parallel = [p for p in ("EP", "TP") if p in args.parallel.split(",")]
    counts = {"EP": EXPERTS // PARALLEL, "TP": EXPERTS}
    providers = args.ref_providers.split(",")

    def median_ms(fn, reps: int = 10) -> float:
        fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end))
        return statistics.median(times)

    for projection in selected_projections(args):
        dims = projection_dims(projection)
        sampler = ClockSampler(0)
        sampler.start()
        wall_begin = time.time()
        rows = []
        for m in m_values:
            for par in parallel:
                k, n = dims[par]
                shapes = [(m, k, n)] * counts[par]
                flops = 2 * m * k * n * counts[par]
                row = {"parallel": par, "M_e": m, "experts": counts[par]}
                progress(f"{projection} {par} M_e={m}: native")
                ws = build_grouped_workspace(shapes, torch.bfloat16, seed=0)
                launch_grouped(ws)
                torch.cuda.synchronize()
                check_device_errors(0)
                row["native_ms"] = round(median_ms(lambda: launch_grouped(ws)), 4)
                row["native_tile"] = f"{ws.launch_info.get('tile_m')}x{ws.launch_info.get('tile_n')}" \
                    f"{' pair' if ws.launch_info.get('path') == 'tcgen05_tma_pair' else ''}"
                native_c = [c.clone() for c in ws.c[:4]]
                del ws
                progress(f"{projection} {par} M_e={m}: reference Triton (hot autotune)")
                try:
                    if "triton" not in providers:
                        raise RuntimeError("not requested (--ref-providers)")
                    rws = ref.build_grouped_workspace(shapes, torch.bfloat16, seed=0)
                    ref.launch_grouped(rws)
                    torch.cuda.synchronize()
                    row["triton_ms"] = round(median_ms(lambda: ref.launch_grouped(rws)), 4)
                    row["triton_config"] = str(getattr(rws, "config", None))
                    errs = []
                    for ours, theirs in zip(native_c, rws.c[:4]):
                        diff = (ours.float() - theirs.float()).norm() / theirs.float().norm().clamp_min(1e-30)
                        errs.append(float(diff))
                    row["rel_err_native_vs_triton"] = max(errs)
                    del rws
                except Exception as exc:
                    row["triton_unavailable"] = f"{type(exc).__name__}: {str(exc)[:200]}"
                torch.cuda.empty_cache()
                progress(f"{projection} {par} M_e={m}: torch grouped_mm")
                try:
                    if "torch_grouped_mm" not in providers:
                        raise RuntimeError("not requested (--ref-providers)")
                    tws = ref.build_torch_grouped_workspace(shapes, torch.bfloat16, seed=0)
                    row["torch_grouped_mm_ms"] = round(median_ms(lambda: ref.launch_torch_grouped(tws)), 4)
                    del tws
                except Exception as exc:
                    row["torch_grouped_mm_unavailable"] = f"{type(exc).__name__}: {str(exc)[:200]}"
                torch.cuda.empty_cache()
                for key in ("native", "triton", "torch_grouped_mm"):
                    if f"{key}_ms" in row:
                        row[f"{key}_tflops"] = round(flops / row[f"{key}_ms"] / 1e9, 1)
                for key in ("triton", "torch_grouped_mm"):
                    if f"{key}_ms" in row:
                        row[f"native_speedup_vs_{key}"] = round(row[f"{key}_ms"] / row["native_ms"], 3)
                rows.append(row)
                print(json.dumps(row), file=sys.stderr, flush=True)
        sampler.mark(wall_begin, time.time())
        clocks = sampler.stop()
        totals = {key: round(sum(r.get(f"{key}_ms", float("nan")) for r in rows), 4)
                  for key in ("native", "triton", "torch_grouped_mm")}
        wins = {key: sum(1 for r in rows if r.get(f"native_speedup_vs_{key}", 0) > 1.0)
                for key in ("triton", "torch_grouped_mm")}
        print(json.dumps({
            "impl": "reference-gpu", "metric": METRIC, "unit": "TFLOP/s", "n_gpus": 1, "dtype": "bf16",
            "projection": PROJECTION_NAME[projection],
            "data": "synthetic (the reference's seeded build_grouped_workspace draw, N(0,1)*0.1)",
            "config": {"workload": workload_line(projection, m_values),
                       "timing": "hot; median of 10 CUDA-event-timed launches per shape after the first call "
                                 "(the reference's autotune runs in that first call)"},
            "providers": {"native": "this package (C ABI, native tile policy)",
                          "triton": "reference kernels/grouped_gemm.py launch_grouped (Triton, hot autotune)",
                          "torch_grouped_mm": "reference kernels/torch_grouped_gemm.py "
                                              "(torch.nn.functional.grouped_mm)"},
            "step_ms": totals, "native_wins": wins, "shapes": len(rows), "per_shape": rows, "clocks": clocks,
        }), flush=True)


def paired_ms(fn_a, fn_b, reps: int = 15) -> tuple[float, float]:
    """Median CUDA-event times of `fn_a` and `fn_b` launched alternately
    (a, b, a, b, ...) back to back on the current stream, hot, after three
    untimed rounds.  Alternating gives both the same clock and power state,
    which drifts over a run of heavy launches on a power-capped GPU."""
    import torch

    for _ in range(3):
        fn_a()
        fn_b()
    torch.cuda.synchronize()
    pairs_a, pairs_b = [], []
    for _ in range(reps):
        for fn, pairs in ((fn_a, pairs_a), (fn_b, pairs_b)):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            pairs.append((start, end))
    torch.cuda.synchronize()
    return (statistics.median(s.elapsed_time(e) for s, e in pairs_a),
            statistics.median(s.elapsed_time(e) for s, e in pairs_b))


def alternating_ms(fns, reps: int = 15) -> float:
    """Median CUDA-event time of one call when the calls in `fns` take turns
    (f0, f1, f0, f1, ...), after three untimed rounds: a rotating-cold launch
    timed alone, each call on the other resident workspace set."""
    import torch

    for _ in range(3):
        for fn in fns:
            fn()
    torch.cuda.synchronize()
    pairs = []
    for _ in range(reps):
        for fn in fns:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            pairs.append((start, end))
    torch.cuda.synchronize()
    return statistics.median(s.elapsed_time(e) for s, e in pairs)


def grouped_mm_side_by_side(steps: dict, device, cold_sets: dict | None = None) -> dict:
    """Per launch of the step: this package's launch alone and
    torch.nn.functional.grouped_mm on the same operands (the call of the
    reference's torch provider, kernels/torch_grouped_gemm.py:162-174: A
    [E * M_e, K], B [E, K, N], int32 cumulative offsets), timed alternately
    (paired_ms); the relative Frobenius difference of their outputs on the
    first two experts rides along.

    For projections in `cold_sets` (projection -> the second resident
    workspace set) the launch is also timed alone with its two workspace sets
    taking turns (`alone_cold_ms`), as the rotating-cold step runs it."""
    import torch

    out = {}
    for proj, rank_step in steps.items():
        other = (cold_sets or {}).get(proj)
        others = {(par, m): ws for par, m, ws in other.workspaces} if other is not None else {}
        for par, m, ws in rank_step.workspaces:
            if (par, m) not in rank_step.stacks:
                continue
            a2d, b3d, offs = rank_step.stacks[(par, m)]
            holder = {}

            def run_grouped_mm():
                holder.pop("c", None)  # lets the caching allocator reuse the previous output's storage
                holder["c"] = torch.nn.functional.grouped_mm(a2d, b3d, offs=offs)

            native_ms, gm_ms = paired_ms(lambda: launch(ws), run_grouped_mm)
            m_rows = ws.shapes[0][0]
            compared = min(2, ws.problem_count)
            ours = torch.cat([ws.c[i] for i in range(compared)]).float()
            theirs = holder["c"][:compared * m_rows].float()
            diff = float((ours - theirs).norm() / theirs.norm().clamp_min(1e-30))
            holder.clear()
            row = {"alone_ms": round(native_ms, 4), "grouped_mm_ms": round(gm_ms, 4),
                   "vs_grouped_mm": round(gm_ms / native_ms, 3), "rel_diff_vs_grouped_mm": float(f"{diff:.3e}")}
            if (par, m) in others:
                ws_other = others[(par, m)]
                row["alone_cold_ms"] = round(alternating_ms([lambda: launch(ws), lambda: launch(ws_other)]), 4)
            out[(proj, par, m)] = row
            torch.cuda.empty_cache()
    return out


def paired_graph_ms(fn_a, fn_b, calls: int = 10, reps: int = 5) -> tuple[float, float]:
    """Per-call device time of `fn_a` and `fn_b`, each captured `calls` times
    into a CUDA graph and the two graphs replayed alternately `reps` times
    (median replay / calls): the device time without host launch overhead,
    the way the reference times its shape sweep (utils/benchmark.py
    time_cuda, CUDA-graph replay)."""
    import torch

    for fn in (fn_a, fn_b):  # eager first calls: tile choice, one-time set-up
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graphs = []
    with torch.cuda.stream(stream):
        for fn in (fn_a, fn_b):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(calls):
                    fn()
            graphs.append(graph)
        for graph in graphs:
            graph.replay()
        stream.synchronize()
        times = ([], [])
        for _ in range(reps):
            for graph, out in zip(graphs, times):
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                graph.replay()
                end.record(stream)
                out.append((start, end))
        stream.synchronize()
    result = tuple(statistics.median(s.elapsed_time(e) for s, e in out) / calls for out in times)
    del graphs
    return result


SWEEP_SIZES = (127, 1000, 4095, 8191)


def masked_sweep_bench(args) -> None:
    """--masked-sweep: BASELINE configs[4]'s masked single GEMM (the
    reference's launch_matmul, kernels/matmul.py:332-392) over every
    {127, 1000, 4095, 8191}^3 shape in fp32, with TF32 inputs and with full
    fp32 products ("ieee": the 3xTF32 split with promoted accumulation on the
    tensor cores), each timed alternately with torch.mm (cuBLAS) at the same
    precision.  Rank 0 / cuda:0 only; one JSON line."""
    import itertools

    import torch

    from kernels import check_device_errors, launch_matmul
    from kernels.matmul import last_launch_info

    torch.cuda.set_device(0)
    rows = []
    totals = {"tf32": [0.0, 0.0, 0.0], "ieee": [0.0, 0.0, 0.0]}  # flops, native ms, torch ms
    sampler = ClockSampler(0)
    sampler.start()
    wall_begin = time.time()
    for m, k, n in itertools.product(SWEEP_SIZES, SWEEP_SIZES, SWEEP_SIZES):
        gen = torch.Generator(device="cuda").manual_seed(m * 7 + k * 3 + n)
        a = torch.randn((m, k), device="cuda", generator=gen)
        b = torch.randn((k, n), device="cuda", generator=gen) / math.sqrt(k)
        c = torch.empty((m, n), device="cuda")
        c_ref = torch.empty((m, n), device="cuda")
        row = {"m": m, "k": k, "n": n}
        for precision in ("tf32", "ieee"):
            def native():
                launch_matmul(a, b, c, input_precision=precision)

            def reference():
                torch.backends.cuda.matmul.allow_tf32 = precision == "tf32"
                torch.mm(a, b, out=c_ref)

            native_ms, torch_ms = paired_graph_ms(native, reference)
            info = last_launch_info()
            flops = 2 * m * n * k
            diff = float((c.double() - c_ref.double()).norm() / c_ref.double().norm().clamp_min(1e-300))
            row[precision] = {"ms": round(native_ms, 4), "tflops": round(flops / native_ms / 1e9, 1),
                              "torch_mm_ms": round(torch_ms, 4), "vs_torch_mm": round(torch_ms / native_ms, 3),
                              "path": info["path"] + ("+3xtf32" if info.get("split_3xtf32") else ""),
                              "rel_diff_vs_torch_mm": float(f"{diff:.2e}")}
            totals[precision][0] += flops
            totals[precision][1] += native_ms
            totals[precision][2] += torch_ms
        torch.backends.cuda.matmul.allow_tf32 = False
        rows.append(row)
        del a, b, c, c_ref
        torch.cuda.empty_cache()
    sampler.mark(wall_begin, time.time())
    clocks = sampler.stop()
    check_device_errors(0)
    summary = {p: {"tflops": round(f / t / 1e9, 1), "sweep_ms": round(t, 3), "torch_mm_tflops": round(f / r / 1e9, 1),
                   "vs_torch_mm": round(r / t, 3),
                   "native_wins": sum(1 for row in rows if row[p]["vs_torch_mm"] > 1.0)}
               for p, (f, t, r) in totals.items()}
    print(json.dumps({
        "metric": "masked single GEMM TFLOP/s over the {127,1000,4095,8191}^3 sweep, fp32", "unit": "TFLOP/s",
        "value": summary["ieee"]["tflops"], "value_precision": "ieee (full fp32 products)", "n_gpus": 1,
        "higher_is_better": True, "dtype": "fp32", "data": "synthetic (A ~ N(0,1), B ~ N(0, 1/sqrt(K)), seeded)",
        "config": {"workload": "BASELINE configs[4]: launch_matmul over every M, K, N in {127,1000,4095,8191}, "
                               "fp32 with input_precision tf32 and ieee",
                   "timing": "per shape: 10 calls of each side captured in a CUDA graph (as the reference's "
                             "time_cuda does), the two graphs replayed alternately 5 times, median replay / 10; "
                             "sweep time = sum over shapes"},
        "summary": summary, "shapes": len(rows), "per_shape": rows, "clocks": clocks,
    }), flush=True)


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    set_model(args.model, args.parallel_size)
    rank, world, local_rank = dist_env()
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return 0
    if args.impl == "reference-gpu":
        reference_gpu_arm(args, rank, world)
        return 0
    if args.masked_sweep:
        if rank == 0:
            masked_sweep_bench(args)
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        # NCCL's communicator lines (rank, nRanks, transport) on stderr, so a
        # run's log shows how many ranks the verification gather spans.  NCCL
        # logs through C stdio to the process's stdout, so file descriptor 1
        # points at stderr while the communicator is created (eagerly, with
        # device_id) and is restored before anything else is printed: stdout
        # keeps only the JSON line.
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"  # an image default such as VERSION or WARN hides the INIT lines
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
            dist.barrier()
        finally:
            sys.stdout.flush()
            try:
                import ctypes

                ctypes.CDLL(None).fflush(None)  # C stdio buffers (NCCL's log lines) go out on stderr too
            except (OSError, AttributeError):
                pass
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    if world > PARALLEL:
        raise SystemExit(f"{world} ranks for a P = {PARALLEL} layout: use --parallel-size >= --gpus")
    if args.moe_layer:
        moe_layer_bench(args, rank, world, local_rank, device)
        if world > 1:
            stdout_to_stderr_for_good()
            dist.destroy_process_group()
        return 0
    m_values = m_values_of(args)
    peaks, peak_source = load_peaks()

    from kernels import check_device_errors
    from moe_parallel import gemm_flops

    projections = selected_projections(args)
    cold = cold_projections(args, projections)
    parallel = tuple(p for p in ("EP", "TP") if p in args.parallel.split(","))

    def build(proj: str, seed: int) -> RankStep:
        if args.fp8:
            return build_rank_fp8(rank, m_values, device, parallel, args.expert_limit)
        if args.layout == "aggregate":
            return build_rank_aggregate(rank, m_values, device, parallel, args.expert_limit,
                                        swiglu=args.fused_swiglu)
        if proj == "W1":
            return build_rank(rank, m_values, device, parallel, args.expert_limit, swiglu=args.fused_swiglu)
        return build_rank_w2(rank, m_values, device, parallel, args.expert_limit, seed=seed)

    progress(f"building rank tensors: {projections}, rotating-cold {cold}")
    sets = {proj: [build(proj, 0)] + ([build(proj, 1)] if proj in cold else []) for proj in projections}
    first = {proj: sets[proj][0] for proj in projections}
    n_rings = 2 if cold else 1
    rings = [[(proj, par, m, ws) for proj in projections for par, m, ws in sets[proj][i % len(sets[proj])].workspaces]
             for i in range(n_rings)]
    rank_flops = sum(gemm_flops(*ws.shapes[0]) * ws.problem_count for _, _, _, ws in rings[0])

    progress("first launch of each workspace (tile policy, untimed)")
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for proj in projections:
            for rank_step in sets[proj]:
                for par, m, ws in rank_step.workspaces:
                    launch(ws)
                    progress(f"  {proj} {par} M_e={m} -> {ws.launch_info}")
    stream.synchronize()
    check_device_errors(local_rank)

    progress("capturing step graphs")
    with torch.cuda.stream(stream):
        # Keep every graph's events alive as long as the graph: the graph
        # records into them on each replay.
        warm_graph, warm_events = graph_of_steps(rings, n_rings, stream)
        graphs, order, events = step_graphs(rings, args.steps, stream)
        for _ in range(args.warmup):
            warm_graph.replay()
        for g in graphs:
            g.replay()  # warms each timed graph's instantiation
    stream.synchronize()

    progress("timed region")
    sampler = ClockSampler(local_rank)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall_begin = time.time()
    with torch.cuda.stream(stream):
        start.record(stream)
        for index in order:
            graphs[index].replay()
        end.record(stream)
    torch.cuda.synchronize(device)
    sampler.mark(wall_begin, time.time())
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    elapsed_t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed_t, op=dist.ReduceOp.MAX)
    max_ms = float(elapsed_t.item())
    check_device_errors(local_rank)
    tc_peak, tc_source = tensor_peak(peaks, clocks)

    # Per-launch device times from the last replay of the timed graphs.
    per_launch: dict[tuple[str, str, int], list[float]] = {}
    for proj, par, m, s_ev, e_ev in events:
        per_launch.setdefault((proj, par, m), []).append(s_ev.elapsed_time(e_ev))
    shapes = {(proj, par, m): (ws.shapes[0], ws.problem_count) for proj, par, m, ws in rings[0]}
    out_cols = (lambda n: n // 2) if args.fused_swiglu else (lambda n: None)
    sm_mhz = (clocks or {}).get("sm_mhz")
    per_shape = []
    for (proj, par, m), times in per_launch.items():
        (mm, k, n), count = shapes[(proj, par, m)]
        ms = statistics.median(times)
        roof, bound = roofline_ms(mm, k, n, count, peaks, tc_peak, out_cols=out_cols(n), fp8=args.fp8)
        row = {"projection": PROJECTION_NAME[proj], "parallel": par, "M_e": m, "experts": count,
               "ms": round(ms, 4), "tflops": round(gemm_flops(mm, k, n) * count / ms / 1e9, 1),
               "roofline_frac": round(roof / ms, 3), "bound": bound}
        if sm_mhz:
            row["kcycles"] = round(ms * sm_mhz, 1)  # ms x MHz = thousands of SM cycles at the region's median
        per_shape.append(row)
    total_ms = sum(statistics.median(t) for t in per_launch.values())
    dominant = max(per_shape, key=lambda r: r["ms"])
    dkey = (next(p for p in projections if PROJECTION_NAME[p] == dominant["projection"]), dominant["parallel"],
            dominant["M_e"])
    (dm, dk, dn), dcount = shapes[dkey]
    d_flops = gemm_flops(dm, dk, dn) * dcount
    if args.fp8:
        d_bytes = fp8_launch_bytes(dm, dk, dn) * dcount
    else:
        d_bytes = 2 * (dm * dk + dk * dn + dm * (dn // 2 if args.fused_swiglu else dn)) * dcount
    if dominant["bound"] == "tensor":
        scale = 2 if args.fp8 else 1
        achieved = d_flops / (dominant["ms"] * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tc_peak * scale, 1),
                    "unit": "TFLOP/s", "frac": round(achieved / (tc_peak * scale), 3),
                    "frac_vs_burst": round(achieved / (peaks["bf16_tflops"] * scale), 3),
                    "frac_vs_sustained": round(achieved / (peaks["bf16_tflops_sustained"] * scale), 3),
                    "peak_source": f"{peak_source} {tc_source}"}
    else:
        achieved = d_bytes / (dominant["ms"] * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": round(achieved / peaks["hbm_gbs"], 3), "peak_source": f"{peak_source} copy bandwidth"}
    roofline.update({"kernel": f"{dominant['projection']} {dominant['parallel']} M_e={dominant['M_e']}",
                     "algorithmic_bytes": d_bytes, "flops": d_flops,
                     "time_share": round(dominant["ms"] / total_ms, 3),
                     "traffic": None if (args.fused_swiglu or args.fp8 or args.layout != "tables")
                     else traffic_from_profiles(dominant)})
    step_roof_ms = sum(roofline_ms(*shapes[key][0], shapes[key][1], peaks, tc_peak,
                                   out_cols=out_cols(shapes[key][0][2]), fp8=args.fp8)[0] for key in shapes)

    # End to end through the public API with host buffers: per step, the
    # step's activations go host -> device from pinned memory, every launch
    # runs, and every output comes back device -> host.
    progress("end-to-end pass")
    e2e_steps = max(1, args.e2e_steps)
    act_lists = {(proj, m): (a if isinstance(a, list) else [a])
                 for proj in projections for m, a in first[proj].activations.items()}
    outs = {(proj, m): c for proj in projections for m, c in first[proj].outputs.items()}
    h2d = sum(t.numel() * t.element_size() for ts in act_lists.values() for t in ts)
    d2h = sum(t.numel() * t.element_size() for c in outs.values() for t in c)
    # Every result comes back into one pinned buffer the size of the largest
    # output (the copies run one after another on the copy stream, and each
    # overwrites the previous result, as a consumer that reads each result
    # before the next arrives would see): the ranks of one box share its host
    # memory (196 GB on the B200 boxes here), and separate buffers for every
    # output would pin ~17.5 GB per rank.
    largest = max(t.numel() * t.element_size() for c in outs.values() for t in c)
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    pinned_need = (h2d + largest) * local_world
    try:
        import psutil

        host_available = psutil.virtual_memory().available
    except ImportError:
        host_available = None
    e2e_skip = None
    if host_available is not None and pinned_need > 0.75 * host_available:
        e2e_skip = (f"{pinned_need / 1e9:.1f} GB of pinned host buffers for {local_world} rank(s) exceed 75% of the "
                    f"{host_available / 1e9:.1f} GB of host memory available")
        act_lists = {}
    host_a = {key: [torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t) for t in ts]
              for key, ts in act_lists.items()}
    result_buf = torch.empty(largest if e2e_skip is None else 0, dtype=torch.uint8, pin_memory=True)
    host_c = {key: tuple(result_buf[:t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t in c)
              for key, c in outs.items()} if e2e_skip is None else {}
    by_key = {}
    for proj in projections:
        for par, m, ws in first[proj].workspaces:
            if e2e_skip is None:
                by_key.setdefault((proj, m), []).append(ws)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Three streams, so both PCIe directions stay busy (the link is full
    # duplex): inputs go host -> device on their own stream and run ahead of
    # the launches, which wait only for their own group's inputs; outputs come
    # back on a third stream as each group finishes.  A group's device inputs
    # are overwritten only after the previous step's launches read them, and
    # its device outputs only after the previous step's copy read them.  W13
    # and W2 groups alternate, so the big W13 inputs travel while W2 outputs
    # come back.
    h2d_stream, d2h_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
    order = sorted(by_key, key=lambda key: (key[1], key[0]))
    computed: dict[tuple[str, int], object] = {}
    copied: dict[tuple[str, int], object] = {}
    with torch.cuda.stream(stream):
        e_start.record(stream)
        h2d_stream.wait_event(e_start)
        d2h_stream.wait_event(e_start)
        for _ in range(e2e_steps):
            for key in order:
                in_ready = torch.cuda.Event()
                with torch.cuda.stream(h2d_stream):
                    if key in computed:
                        h2d_stream.wait_event(computed[key])
                    for dev_t, host_t in zip(act_lists[key], host_a[key]):
                        dev_t.copy_(host_t, non_blocking=True)
                    in_ready.record(h2d_stream)
                stream.wait_event(in_ready)
                if key in copied:
                    stream.wait_event(copied[key])
                for ws in by_key[key]:
                    launch(ws)
                computed[key] = torch.cuda.Event()
                computed[key].record(stream)
                with torch.cuda.stream(d2h_stream):
                    d2h_stream.wait_event(computed[key])
                    for host_t, dev_t in zip(host_c[key], outs[key]):
                        host_t.copy_(dev_t, non_blocking=True)
                    copied[key] = torch.cuda.Event()
                    copied[key].record(d2h_stream)
        stream.wait_stream(h2d_stream)
        stream.wait_stream(d2h_stream)
        e_end.record(stream)
    torch.cuda.synchronize(device)
    e2e_t = torch.tensor([e_start.elapsed_time(e_end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_t.item())
    del host_a, host_c, result_buf
    check_device_errors(local_rank)

    progress("verification")
    checks = {}
    for proj in projections:
        for index, rank_step in enumerate(sets[proj]):
            name = PROJECTION_NAME[proj] + (f" set {index}" if len(sets[proj]) > 1 else "")
            if args.fp8:
                checks[name] = verify_fp8_outputs(world, rank_step.workspaces, m_values, device)
            elif parallel != ("EP", "TP") or args.expert_limit:
                checks[name] = {"skipped": "partial workload (--parallel / --expert-limit)"}
            elif proj == "W2":
                checks[name] = verify_w2_outputs(rank, world, rank_step.ep, rank_step.tp, rank_step.outputs,
                                                 device, m_values, seed=index)
            else:
                checks[name] = verify_rank_outputs(rank, world, rank_step.ep, rank_step.tp, rank_step.activations,
                                                   rank_step.outputs, device, m_values, swiglu=args.fused_swiglu)
    ran = [c for c in checks.values() if "passed" in c]
    verification = {"passed": all(c["passed"] for c in ran) if ran else None,
                    "max_rel_frobenius": max((c["max_rel_frobenius"] for c in ran), default=None),
                    "tolerance": 1e-2, "by_projection": checks}

    side, side_clocks = {}, None
    if not args.skip_grouped_mm and not args.fp8 and not args.fused_swiglu and args.layout == "tables":
        progress("per-shape side-by-side with torch grouped_mm")
        side_clock = ClockSampler(local_rank)
        side_clock.start()
        with torch.cuda.stream(stream):
            side = grouped_mm_side_by_side(first, device, {proj: sets[proj][1] for proj in cold})
        side_clocks = side_clock.stop()
        check_device_errors(local_rank)
    for row in per_shape:
        proj = next(p for p in projections if PROJECTION_NAME[p] == row["projection"])
        row.update(side.get((proj, row["parallel"], row["M_e"]), {}))

    # A tensor-core grouped launch is two kernels (tensor-map builder + GEMM);
    # a single-problem or generic-path launch is one.
    kernels_per_step = sum(2 if ws.launch_info["path"].startswith("tcgen05") and ws.problem_count > 1 else 1
                           for _, _, _, ws in rings[0])
    launches = torch.tensor([kernels_per_step * args.steps], device=device, dtype=torch.int64)
    if world > 1:
        dist.all_reduce(launches)
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        progress("cpu baseline")
        cpu = time_cpu(m_values, experts_per_launch=4, passes=10, budget_s=25.0, projections=projections)

    if rank == 0:
        total_flops = rank_flops * world
        value = total_flops * args.steps / (max_ms * 1e-3) / 1e12
        modes = []
        if args.fused_swiglu:
            modes.append("fused SwiGLU epilogue: C = silu(gate) * up, [M_e, F_local]")
        if args.layout == "aggregate":
            modes.append("expert-sorted aggregate layout (launch_grouped_mm, int32 offsets)")
        if args.fp8:
            modes.append("e4m3 experts with DeepSeek-V3 block scales (128x128 weight, 1x128 token), bf16 output; "
                         "tensor peak = 2x the bf16 one")
        compared = [r for r in per_shape if "vs_grouped_mm" in r]
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3" if args.fp8 else "bf16", "data": "synthetic",
            "config": {"workload": "; ".join([workload_text(projections, cold, m_values)] + modes),
                       "model": MODEL, "parallel_size": PARALLEL,
                       "parallelism": f"GPU r runs rank r of P={PARALLEL} (EP and TP), {world} rank(s)",
                       "cache": ("inputs larger than L2 (0.94-1.88 GB of weights per launch group), no flush"
                                 + ("; rotating-cold: " + ", ".join(PROJECTION_NAME[p] for p in cold)
                                    + " alternate two resident workspace sets step by step" if cold else "")),
                       "timing": "CUDA events around graph replays of whole steps, max over ranks"},
            "roofline": roofline,
            "roofline_step_frac": round(step_roof_ms / total_ms, 3),
            "per_shape": sorted(per_shape, key=lambda r: (r["projection"] != "W13", r["M_e"], r["parallel"])),
            "grouped_mm": None if not compared else {
                "native_wins": sum(1 for r in compared if r["vs_grouped_mm"] > 1.0), "shapes": len(compared),
                "step_ms_native_alone": round(sum(r["alone_ms"] for r in compared), 4),
                "step_ms_grouped_mm": round(sum(r["grouped_mm_ms"] for r in compared), 4),
                "clocks": side_clocks,
                "note": "each launch alone, hot, alternating with grouped_mm call by call, median of 15 "
                        "CUDA-event-timed calls each; grouped_mm = torch.nn.functional.grouped_mm on the same "
                        "operands (the reference's torch provider); alone_cold_ms: the rotating-cold launches "
                        "alone with their two workspace sets taking turns; clocks: NVML over the whole pass"},
            "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind",
                                                                              "sample")},
            "e2e": {"value": round(rank_flops * world * e2e_steps / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "launch_grouped per workspace with activations copied in from pinned host memory and "
                            "every output copied back every step (inputs, launches and outputs on three streams, "
                            "so both PCIe directions overlap; outputs into one reused pinned result buffer); "
                            "weights resident"}
            if e2e_skip is None else {"value": None, "skipped": e2e_skip},
            "gpu_launches": int(launches.item()),
            "clocks": clocks,
            "verification": verification,
            "peaks": {**peaks, "source": peak_source, "tensor_peak_used": round(tc_peak, 1),
                      "tensor_peak_source": tc_source},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        stdout_to_stderr_for_good()
        dist.barrier()
        dist.destroy_process_group()
    del graphs, warm_graph, events, warm_events
    return 0


def stdout_to_stderr_for_good() -> None:
    """Points file descriptor 1 at stderr for the rest of the process.

    NCCL logs through C stdio to stdout, also when a communicator is torn down
    and when its plugins close at exit; called once the JSON line is out, this
    keeps that line the only thing the run prints on stdout."""
    sys.stdout.flush()
    try:
        import ctypes

        ctypes.CDLL(None).fflush(None)
    except (OSError, AttributeError):
        pass
    os.dup2(2, 1)


def traffic_from_profiles(dominant: dict):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "dram_traffic.json"
    if not path.exists():
        return None
    data = json.loads(path.read_text())
    entry = data.get(f"{dominant['projection']}_{dominant['parallel']}_M{dominant['M_e']}")
    return None if entry is None else entry.get("bytes_per_launch")


if __name__ == "__main__":
    raise SystemExit(main())
