"""Timed CPU baseline -- test / benchmark infrastructure only.

The reference's own host-side computation of this path is per-expert
``torch.matmul`` on the expert tensors (benchmark_moe.py:259-266).  Here it
runs on host tensors with every host thread torch may use, which is the CPU
baseline of the benchmark.  It is timed, never shipped.
"""

from __future__ import annotations

import os
import statistics
import time
from collections.abc import Sequence


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def make_host_problems(shapes: Sequence[tuple[int, int, int]], dtype_name: str, seed: int = 0):
    """Seeded host inputs: A ~ N(0, 1), B ~ N(0, 1/sqrt(K)) (the metric runs' distribution)."""
    import torch

    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[dtype_name]
    gen = torch.Generator().manual_seed(seed)
    a_list, b_list = [], []
    for m, k, n in shapes:
        a_list.append(torch.randn((m, k), generator=gen).to(dtype))
        b_list.append((torch.randn((k, n), generator=gen) / k**0.5).to(dtype))
    return a_list, b_list


def per_expert_mm(a_list, b_list) -> list:
    """The reference's per-expert host computation (benchmark_moe.py:265-266)."""
    import torch

    return [torch.matmul(a, b) for a, b in zip(a_list, b_list)]


def time_per_expert_mm(a_list, b_list, repeats: int = 5, threads: int | None = None) -> dict:
    """Median wall time of per-expert host matmuls after one warm-up pass."""
    import torch

    threads = threads or host_threads()
    previous = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        per_expert_mm(a_list, b_list)
        samples = []
        for _ in range(max(1, repeats)):
            start = time.perf_counter()
            per_expert_mm(a_list, b_list)
            samples.append(time.perf_counter() - start)
    finally:
        torch.set_num_threads(previous)
    flops = sum(2 * a.shape[0] * a.shape[1] * b.shape[1] for a, b in zip(a_list, b_list))
    median = statistics.median(samples)
    return {"seconds": median, "flops": flops, "tflops": flops / median / 1e12, "threads": threads,
            "samples": len(samples)}
