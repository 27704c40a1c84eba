"""A training step of the Naylis decoder replayed as one CUDA graph.

The config-3 step issues ~1,340 kernels; launched one by one from Python the GPU
spends a few microseconds between each pair (launch latency and the drain of
the previous kernel), ~4 ms per step, although the host stays well ahead of the
device. `GraphedTrainStep` captures zero_grad + forward + loss + backward once
and replays it: the kernels, their arguments and every buffer (activations,
the routing plans, the gradient buckets) are fixed at capture, so a replay is
one launch of the whole step.

What the capture relies on:

* gradients live in a `GradAllReduce`'s buckets: `zero_grad()` clears them to
  None before the capture, so the weight-gradient GEMMs write into the bucket
  slots and the other gradients are copied in by its hooks inside the graph;
  after `step()` every `.grad` is its slot view, as in eager mode. With more
  than one process the exchange cannot be captured from the hooks: pass a
  `GradAllReduce(..., overlap=False)`, whose `finish()` (run by `step()` after
  the replay) all-reduces every bucket;
* the optimizer runs outside the graph, after `step()` (its step count changes
  every step); the package's `AdamW` rewrites the bf16 weight and bank copies
  the captured projections read, so nothing else may change the weights
  in place between replays without a new capture;
* the Gumbel draws come from torch's CUDA generator, which advances per replay;
* the token ids (and labels) are copied into static buffers by `step()`.
"""
from __future__ import annotations

import torch

from . import _lib


class GraphedTrainStep:
    def __init__(self, model, dp, ids, labels=None, warmup: int = 3, dtype=torch.bfloat16):
        if not ids.is_cuda:
            raise RuntimeError("GraphedTrainStep: token ids must be on the model's CUDA device")
        if dp.world > 1 and dp.overlap:
            raise RuntimeError("GraphedTrainStep on more than one process needs GradAllReduce(..., "
                               "overlap=False): the buckets are exchanged by finish() after each replay")
        self.model, self.dp, self.dtype = model, dp, dtype
        self.ids = ids.clone()
        self.labels = self.ids if labels is None else labels.clone()
        dev = ids.device
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        lib = _lib.load()
        n0 = lib.mom_kernel_launches()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = self._body()
        # this library's kernels in one replay (the launch counter only sees launches
        # made from the host, i.e. the capture)
        self.kernels_per_replay = int(lib.mom_kernel_launches() - n0)
        self.dp.finish()

    def _body(self):
        self.dp.zero_grad()
        with torch.autocast("cuda", dtype=self.dtype):
            loss = self.model(self.ids, labels=self.labels)
        loss.backward()
        return loss.detach()

    def step(self, ids=None, labels=None):
        """Replay the step (on new token ids / labels when given, copied into the
        static buffers) and exchange the gradients; returns the loss tensor (a
        static buffer, overwritten by the next replay)."""
        if ids is not None:
            self.ids.copy_(ids, non_blocking=True)
        if labels is not None and self.labels is not self.ids:
            self.labels.copy_(labels, non_blocking=True)
        self.graph.replay()
        self.dp.finish()
        return self.loss


__all__ = ["GraphedTrainStep"]
