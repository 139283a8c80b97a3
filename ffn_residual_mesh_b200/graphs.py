"""CUDA-graph replay of a sequence of library calls.

Decode steps are launch-bound at small batches (three kernels per layer, tens of
layers); capturing a whole step once and replaying it removes the per-call host
cost. Every entry point of the library is capturable: kernels run on the caller's
stream, and the host-streamed call forks its copy stream from that stream inside a
capture. Host buffers passed to captured host-streamed calls are baked into the
graph: refill them in place between replays.
"""
from __future__ import annotations


class StepGraph:
    """Capture ``fn()`` (a sequence of library calls) once; ``replay()`` re-issues it."""

    def __init__(self, fn, warmup: int = 1):
        import torch
        self.fn = fn
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            fn()
        torch.cuda.synchronize()

    def replay(self) -> None:
        self.graph.replay()

    def close(self) -> None:
        self.graph.reset()
