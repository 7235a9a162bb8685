"""CUDA-graph capture of a whole step (the B200 build's replacement for per-op host dispatch).

A small step -- the config-2 CNN's 58 launches, a 512^3 matmul's four -- spends most of its time in
host-side dispatch (Python, ctypes, the CUDA runtime). GraphedStep runs the step eagerly a few
times (so every per-device set-up, kernel attribute and memory-pool growth has happened), then
captures one run into a CUDA graph and replays it. Everything the step enqueues is captured: the
library's kernels, its stream-ordered scratch allocations (graph memory nodes, same addresses on
every replay) and the torch buffers it allocates (a private graph pool).

Rules for a captured step: its inputs must live in fixed buffers that are refilled before each
replay; it must not read device values on the host; host-side state that changes per step (an
optimizer's step count) is frozen at capture, so training steps with AdamW are not captured here.
"""
from __future__ import annotations

import torch

from . import lib


class GraphedStep:
    def __init__(self, fn, warmup: int = 3):
        self.fn = fn
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        lib().nnb_trace_enable(0)          # no event records inside the graph
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.out = fn()
        torch.cuda.synchronize()

    def __call__(self):
        self.graph.replay()
        return self.out
