"""CUDA-graph capture of the forward and the training step, for callers whose shapes repeat.

At small shapes (serving, short sequences) one call of the path is a few microseconds of GPU work
per kernel and tens of microseconds of host work (argument checks, tensor-map encoding, launches).
A captured graph replays the same launches with one host call. The tensors given at capture time
are the graph's static inputs: copy new data into them, call the returned function, and read the
static outputs (valid until the next replay).

Every libfrx entry point is capture-safe: no allocation outside the graph pool, no host
synchronisation, work only on the capturing stream and on side streams forked from it.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
from torch import Tensor

from . import gemm_kernel as gk


def _capture(fn: Callable[[], Tuple[Tensor, ...]], warmup: int):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(1, warmup)):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = fn()
    return graph, outs


def graphed_forward(hidden: Tensor, weight: Tensor, target: Tensor, bias: Optional[Tensor] = None,
                    chunk_size: int = 4096, warmup: int = 2) -> Callable[[], Tuple[Tensor, Tensor, Tensor]]:
    """Captures gemm_fused_ce_entropy on these (device) tensors; returns run() -> (ce, entropy,
    log_probs), replaying the graph on the current stream."""
    graph, outs = _capture(lambda: gk.gemm_fused_ce_entropy(hidden, weight, target, bias=bias,
                                                            chunk_size=chunk_size), warmup)

    def run():
        graph.replay()
        return outs

    return run


def graphed_training_step(hidden: Tensor, weight: Tensor, target: Tensor, bias: Optional[Tensor] = None,
                          chunk_size: int = 4096, ce_weight: float = 1.0, ent_weight: float = -1.0,
                          warmup: int = 2) -> Callable[[], Tuple[Tensor, Tensor, Tensor]]:
    """Captures gemm_megakernel_fast + loss.backward() on these leaf tensors (requires_grad set);
    returns run() -> (loss, ce, entropy). After each replay hidden.grad / weight.grad (and bias.grad)
    hold that step's gradients (the same storage every time)."""
    leaves = [t for t in (hidden, weight, bias) if t is not None]

    def step():
        for t in leaves:
            t.grad = None
        loss, ce, ent = gk.gemm_megakernel_fast(hidden, weight, target, bias=bias, chunk_size=chunk_size,
                                                ce_weight=ce_weight, ent_weight=ent_weight)
        loss.backward()
        return loss.detach(), ce, ent

    graph, outs = _capture(step, warmup)

    def run():
        graph.replay()
        return outs

    return run
