"""Device timing of short launches without host launch overhead.

A Python-level call into the library costs several microseconds of host
time (argument checks, ctypes, tensor-map encoding).  A decode step runs its
kernels from CUDA graphs, so the kernel time that matters is the one seen
there: `graph_time_us` captures `calls` (a list of zero-argument callables,
one launch sequence each) into one CUDA graph, `rounds` times over, and times
one replay with CUDA events on the capturing stream.
"""

from __future__ import annotations

import torch


def graph_time_us(calls, rounds: int = 4, warmup_replays: int = 2) -> float:
    """Average microseconds per call over `rounds * len(calls)` captured calls."""
    for fn in calls:  # eager warm-up: workspaces, tensor maps, lazy state
        fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in calls:
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(rounds):
            for fn in calls:
                fn()
    for _ in range(warmup_replays):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (rounds * len(calls))
    del g
    return us
