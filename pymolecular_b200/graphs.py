"""Whole-training-step CUDA graphs.

A training step of this package (embedding, E_GCL layers, loss, backward,
optimizer update, and under data parallelism the gradient all-reduce) is a
fixed sequence of kernel launches on one stream: every op of the library
takes torch's current stream, allocates its workspace through torch's
allocator and never synchronizes with the host.  Such a step can be captured
once and replayed, which removes the per-launch host cost (Python autograd,
ctypes, launch latency) from every step after the first.

The graph reads its inputs from the tensors the captured step used: to
train on new data of the same shapes, copy it into those tensors (or into
the CSR's index arrays) before `replay()`.
"""
from __future__ import annotations

from typing import Callable

import torch


class GraphedStep:
    """Capture `step` (a callable returning the loss tensor, detached so that
    no autograd graph outlives the capture) as a CUDA graph.

    `warmup` eager calls run first on a side stream (they perform the
    library's one-time per-device set-up and let the allocator settle), then
    one call is captured.  Gradients that are None when the capture starts
    are allocated inside the graph's memory pool and keep their storage
    across replays.  `replay()` runs the captured step and returns the
    (static) loss tensor it writes.
    """

    def __init__(self, step: Callable[[], torch.Tensor], warmup: int = 3):
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                step()
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(self.graph):
            self.loss = step()

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.loss

    __call__ = replay

    def release(self) -> None:
        """Free the graph (do this before destroying a process group whose
        collectives the graph captured)."""
        self.graph.reset()


__all__ = ["GraphedStep"]
