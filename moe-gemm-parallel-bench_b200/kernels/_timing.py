"""Device-only timing for the launch autotuner.

Follows the reference's measurement method (utils/benchmark.py:123-198,
hot_autotune_bench :249-258): the calls are recorded into one CUDA graph with
an event pair around every call, so host dispatch never lands inside a
sample; the graph is replayed once to warm it and once to sample.
"""

from __future__ import annotations

import statistics
from collections.abc import Callable


def graph_median_ms(function: Callable[[], None], samples: int = 9, warmup: int = 2) -> float:
    import torch

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(max(1, warmup)):
            function()
    stream.synchronize()
    events = [
        (torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
        for _ in range(max(3, samples))
    ]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for start, end in events:
            start.record()
            function()
            end.record()
    with torch.cuda.stream(stream):
        graph.replay()  # warm the instantiated graph
    stream.synchronize()
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()
    values = [start.elapsed_time(end) for start, end in events]
    del graph
    return statistics.median(values)


def capturing() -> bool:
    import torch

    return bool(torch.cuda.is_current_stream_capturing())
