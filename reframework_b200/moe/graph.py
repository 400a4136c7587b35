"""CUDA-graph capture of a resident MoE layer forward.

A resident ``FusedMoE.forward`` has no host synchronisation: the tile table of
the grouped GEMMs is built on the device from the permute's counts, and every
buffer comes from torch's caching allocator.  Its launches can therefore be
captured once per input shape and replayed, which removes the per-call host
cost (argument checks, allocations, ~7 launches) that dominates small-batch
decode steps.  Offloaded layers and expert-parallel layers synchronise on the
host (expert residency, all-to-all split sizes) and cannot be captured.
"""

from __future__ import annotations

from typing import Optional

import torch

__all__ = ["GraphedForward", "capture_forward"]


class GraphedForward:
    """Replays a captured ``module(x)`` for inputs of one fixed shape and dtype.

    ``__call__(x)`` copies ``x`` into the captured input buffer, replays the
    graph on the current stream and returns the captured output buffer (it is
    overwritten by the next call; clone it to keep it).
    """

    def __init__(self, module, example: torch.Tensor, warmup: int = 2,
                 pool: Optional[object] = None) -> None:
        if getattr(module, "uses_offload", False):
            raise RuntimeError("offloaded layers synchronise on the host and cannot be captured")
        self.module = module
        self.static_in = example.detach().clone()
        stream = torch.cuda.Stream(device=example.device)
        stream.wait_stream(torch.cuda.current_stream(example.device))
        with torch.cuda.stream(stream), torch.no_grad():
            for _ in range(warmup):  # settle lazy set-up (kernel attributes, tensor-map entry points)
                module(self.static_in)
        torch.cuda.current_stream(example.device).wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool), torch.no_grad():
            self.static_out = module(self.static_in)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape != self.static_in.shape or x.dtype != self.static_in.dtype:
            raise ValueError(f"captured for {tuple(self.static_in.shape)} {self.static_in.dtype}, "
                             f"got {tuple(x.shape)} {x.dtype}")
        self.static_in.copy_(x)
        self.graph.replay()
        return self.static_out


def capture_forward(module, example: torch.Tensor, warmup: int = 2) -> GraphedForward:
    """Capture ``module(example)`` into a CUDA graph (see :class:`GraphedForward`)."""
    return GraphedForward(module, example, warmup=warmup)
