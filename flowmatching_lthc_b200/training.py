"""A training step replayed from CUDA graphs (BASELINE config 4's step: forward,
backward and a fused AdamW update of LTHC-B/4 under bf16 autocast).

The eager step launches about 2300 kernels; on one B200 at 32 images the GPU is
busy for about 81 % of it and the rest is launch gaps.  ``GraphedTrainStep``
captures the forward and backward (with the gradient buffer zeroed first) as one
graph and the optimizer update as another, so that a step is two replays plus
whatever runs between them.  The data-parallel gradient exchange stays eager, so
no collective lives inside a graph and no graph has to be released before the
process group is destroyed.

Requirements of the capture, as for any whole-network CUDA graph:
- the inputs are static tensors; new data is copied into them;
- gradients live in persistent buffers (``dist.FlatGradients`` views) and are
  zeroed inside the graph;
- the optimizer is capturable (``torch.optim.AdamW(..., fused=True, capturable=True)``);
- autocast runs with its weight cache off (a cached cast would be reused across
  replays).
"""
from __future__ import annotations

from typing import Callable

import torch


class GraphedTrainStep:
    """``fwd_bwd()`` computes the loss and calls ``backward()`` (it should zero the
    gradients first); ``opt_step()`` applies the update.  Both are run ``warmup``
    times eagerly on a side stream (these are real updates), then captured.
    Calling the object replays forward + backward, runs ``exchange`` (if given)
    eagerly, and replays the update."""

    def __init__(self, fwd_bwd: Callable[[], None], opt_step: Callable[[], None], warmup: int = 3) -> None:
        if warmup < 1:
            raise ValueError("warm-up of at least one eager step is needed before capture")
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fwd_bwd()
                opt_step()
        torch.cuda.current_stream().wait_stream(side)
        self.fwd_bwd_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.fwd_bwd_graph):
            fwd_bwd()
        self.opt_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.opt_graph):
            opt_step()

    def __call__(self, exchange: Callable[[], None] | None = None) -> None:
        self.fwd_bwd_graph.replay()
        if exchange is not None:
            exchange()
        self.opt_graph.replay()


def flow_matching_step(model: torch.nn.Module, zero_grad: Callable[[], None], zt: torch.Tensor, t: torch.Tensor,
                       y: torch.Tensor, v: torch.Tensor, loss_out: torch.Tensor | None = None,
                       dtype: torch.dtype | None = torch.bfloat16) -> Callable[[], None]:
    """The velocity-target loss of a flow-matching step on static tensors: zero the
    gradients, ``mean((v - model(zt, t, y))^2)`` under autocast (weight cache off),
    backward.  ``loss_out`` (a 0-d fp32 tensor) receives the loss if given."""

    def fwd_bwd() -> None:
        zero_grad()
        if dtype is None:
            loss = (v - model(zt, t, y)).float().square().mean()
        else:
            with torch.autocast("cuda", dtype=dtype, cache_enabled=False):
                loss = (v - model(zt, t, y)).float().square().mean()
        loss.backward()
        if loss_out is not None:
            loss_out.copy_(loss.detach())

    return fwd_bwd
