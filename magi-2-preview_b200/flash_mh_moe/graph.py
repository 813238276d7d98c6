"""CUDA-graph replay of a fixed-shape MoE forward (launch-bound small batches).

At a few hundred tokens a layer's GPU work is ~0.1 ms while the host side of ~12 launches
(ctypes calls, tensor allocations, tensor-map encoding) costs about as much; capturing the
forward once and replaying it removes that.  The single-GPU layer is capturable: every
library call launches on the current stream, allocates through torch, and synchronises
nothing.  The expert-parallel layer is not (its exchange counts layer calls on the host).
"""
from __future__ import annotations

from typing import Callable

import torch


class CapturedForward:
    """``fn(x) -> y`` captured for one input shape; call it with a same-shape tensor.

    ``warmup`` eager calls on a side stream run first (they also perform the one-time set-up
    of the library: weight packing, kernel attributes).  The output tensor is the graph's
    static output and is overwritten by the next call.
    """

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], example: torch.Tensor, warmup: int = 3):
        self.fn = fn
        side = torch.cuda.Stream(device=example.device)
        side.wait_stream(torch.cuda.current_stream(example.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                fn(example)
        torch.cuda.current_stream(example.device).wait_stream(side)
        self.static_in = example.clone()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_out = fn(self.static_in)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape != self.static_in.shape or x.dtype != self.static_in.dtype:
            raise ValueError(f"captured for {tuple(self.static_in.shape)} {self.static_in.dtype}, "
                             f"got {tuple(x.shape)} {x.dtype}")
        if x.data_ptr() != self.static_in.data_ptr():
            self.static_in.copy_(x)
        self.graph.replay()
        return self.static_out
