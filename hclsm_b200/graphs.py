"""A whole training step (forward + backward) captured as one CUDA graph.

The training paths of this library (the slot-attention iteration, the
SimplifiedSSMBlock, the scan) launch a few hundred small kernels per step
through ctypes and autograd; at config-2 shapes the host needs longer to
launch them than the GPU needs to run them.  ``GraphedStep`` records the step
once and replays it with one launch, so the GPU runs the same kernels
back to back.  Nothing in those paths reads device memory on the host, which
is what capture requires.

Rules (those of CUDA graph capture):

* ``step()`` runs the forward and the backward on fixed input tensors; to
  train on new data, copy it into those tensors before ``replay()``;
* ``params`` are the tensors whose ``.grad`` the step produces.  Their
  gradients are set to None before the warm-up calls and the capture, so the
  captured backward allocates them from the graph's memory pool; every replay
  overwrites them (it does not accumulate);
* the first calls run eagerly on a side stream (warm-up: library handles,
  cached weight casts and workspaces are created there, not inside the graph);
* under autocast, pass ``cache_enabled=False`` to ``torch.autocast`` inside
  ``step`` (autocast's cast cache does not survive capture).
"""
from __future__ import annotations

from typing import Callable, Iterable

import torch

__all__ = ["GraphedStep"]


class GraphedStep:
    """``GraphedStep(step, params)``: capture ``step`` (a callable running a
    forward and backward) as one CUDA graph; ``replay()`` (or calling the
    object) runs it on the current stream."""

    def __init__(self, step: Callable[[], object], params: Iterable[torch.Tensor] = (), warmup: int = 3):
        if not torch.cuda.is_available():
            raise RuntimeError("hclsm_b200.GraphedStep needs a CUDA device")
        self.params = list(params)
        self.step = step
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(int(warmup), 1)):
                self._clear()
                step()
        torch.cuda.current_stream().wait_stream(side)
        self._clear()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            step()

    def _clear(self):
        for p in self.params:
            p.grad = None

    def replay(self) -> None:
        self.graph.replay()

    __call__ = replay
