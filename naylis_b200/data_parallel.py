"""Explicit data-parallel gradient exchange for MoM training over NCCL.

Replaces the reference's implicit DDP (HF Trainer under torchrun,
pretrain.py:792-817 with ddp_find_unused_parameters=False,
run_biggpu.sh:16-42): one process per GPU, the batch sharded by sequence
(every sequence whole on one rank, so the causal router needs no exchange),
and every gradient — the shared bank ``M_blocks`` (summed over all layers
first), the router and the q/k/v/o projections — averaged across ranks.

Design: each parameter owns a slot in a flat fp32 bucket, and after the
backward its ``.grad`` is a view of that slot, so the all-reduce runs on the
gradients in place. ``zero_grad()`` clears the gradients to None instead of
zeroing the buckets: the decoder's bf16 projections (``trunk.linear_f32grad``)
write their weight-gradient GEMM's fp32 output straight into the slots, which
autograd adopts as ``.grad`` (no fill, no add); any other gradient is copied
into its slot by the post-accumulate hook, which then marks the parameter
ready. Parameters that one GEMM produces gradients for together (``groups``,
or the module's ``grad_groups()``: the fused q/k/v and gate/up projections)
sit next to each other in one bucket, in the GEMM's row order. Buckets are
launched as asynchronous all-reduces strictly in bucket order (identical on
every rank, as NCCL requires) as soon as all their parameters are ready, so
the exchange overlaps the rest of the backward. ``finish()`` zero-fills the
slots of parameters that got no gradient, launches whatever is left and
waits; the average is NCCL's own (``ReduceOp.AVG``), or a division by the
world size on backends without it.

Gradient accumulation (the reference's ``[train] grad_accum``, pretrain.py:795
under DDP): run every micro-batch but the last inside ``no_sync()``, which
keeps the hooks from launching, then the last backward and ``finish()`` once.
A second backward before ``finish()`` outside ``no_sync()`` would add into
buckets already on the wire, so it raises instead.

``comm_dtype=torch.bfloat16`` sends each bucket as bf16 (half the bytes on
NVLink): the fp32 bucket is rounded into a bf16 twin on the compute stream
before its all-reduce, and the averaged result is written back into the fp32
bucket by ``finish()``.
"""
from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist

from . import trunk


class GradAllReduce:
    def __init__(self, module: torch.nn.Module, process_group=None, bucket_mb: float = 32.0,
                 average: bool = True, overlap: bool = True, comm_dtype=None, groups=None):
        self.group = process_group
        # overlap=False: no collective from the backward's hooks; finish()
        # exchanges every bucket. For a backward captured in a CUDA graph,
        # whose replay then runs no collective, with finish() after replay.
        self.overlap = overlap
        self._sync = True
        if comm_dtype not in (None, torch.float32, torch.bfloat16):
            raise ValueError(f"GradAllReduce: comm_dtype must be fp32 or bf16, got {comm_dtype}")
        self.comm_dtype = None if comm_dtype in (None, torch.float32) else comm_dtype
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.average = average
        # NCCL averages inside the reduction (no extra pass over the buckets);
        # other backends (gloo) sum, and finish() divides
        self._op = dist.ReduceOp.SUM
        self._divide = average and self.world > 1
        if self._divide and dist.get_backend(process_group) == "nccl":
            self._op = dist.ReduceOp.AVG
            self._divide = False
        params = [p for p in module.parameters() if p.requires_grad]
        for p in params:
            if p.dtype != torch.float32:
                raise RuntimeError("GradAllReduce keeps fp32 master gradients; got "
                                   f"a {p.dtype} parameter")
        if groups is None:
            groups = module.grad_groups() if hasattr(module, "grad_groups") else []
        members = {id(p) for p in params}
        group_of = {}
        for g in groups:
            g = tuple(g)
            if all(id(p) in members for p in g) and not any(id(p) in group_of for p in g):
                for p in g:
                    group_of[id(p)] = g
        # gradients arrive roughly in reverse registration order; a group is placed,
        # in its own order, where its first member appears
        units, placed = [], set()
        for p in reversed(params):
            g = group_of.get(id(p), (p,))
            if id(g[0]) not in placed:
                units.append(g)
                placed.update(id(q) for q in g)
        # every unit (a parameter, or a group) starts on a 16-byte boundary: a GEMM
        # writing into a slot needs it (a 1-element mom_scale would otherwise shift
        # every later slot), and the zero padding rides along in the all-reduce
        pad = lambda n: (n + 3) // 4 * 4
        cap = int(bucket_mb * (1 << 20) // 4)
        self.buckets = []
        cur = []
        size = 0
        for g in units:
            n = pad(sum(p.numel() for p in g))
            if cur and size + n > cap:
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(g)
            size += n
        if cur:
            self.buckets.append(cur)
        self.params = [p for units_ in self.buckets for g in units_ for p in g]
        self.flat = []
        self._bucket_of = {}
        self._slot = {}
        for i, units_ in enumerate(self.buckets):
            n = sum(pad(sum(p.numel() for p in g)) for g in units_)
            buf = torch.zeros(n, dtype=torch.float32, device=units_[0][0].device)
            off = 0
            for g in units_:
                start = off
                for p in g:
                    view = buf[off:off + p.numel()].view_as(p)
                    p.grad = view
                    self._slot[p] = view
                    trunk.register_grad_slot(p, buf, off)
                    off += p.numel()
                    self._bucket_of[p] = i
                off = start + pad(off - start)
            self.flat.append(buf)
        self.buckets = [[p for g in units_ for p in g] for units_ in self.buckets]
        self.wire = [torch.empty(b.numel(), dtype=self.comm_dtype, device=b.device) for b in self.flat] \
            if self.comm_dtype is not None and self.world > 1 else None
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_ready) for p in params]
        self._reset_state()

    def _reset_state(self):
        self._pending = [len(ps) for ps in self.buckets]
        self._next = 0
        self._works = []

    def zero_grad(self):
        """Clear every gradient to None (no device work): the next backward writes
        or copies each gradient into its slot, and ``finish()`` zero-fills the slots
        of parameters that got none."""
        for p in self.params:
            p.grad = None
        trunk.release_grad_slots(self.params)
        self._reset_state()

    def _place(self, p):
        """Make p.grad the view of its slot, copying the gradient in if autograd
        left it elsewhere (or zero-filling the slot when there is none)."""
        slot = self._slot[p]
        g = p.grad
        if g is None:
            slot.zero_()
        elif g.data_ptr() != slot.data_ptr() or g.stride() != slot.stride():
            slot.copy_(g)
        else:
            return
        p.grad = slot

    @contextlib.contextmanager
    def no_sync(self):
        """Backwards inside this context only accumulate into the buckets; the
        exchange happens after the next backward outside it, at ``finish()``."""
        prev = self._sync
        self._sync = False
        try:
            yield
        finally:
            self._sync = prev

    def _launch_ready(self, force: bool = False):
        while self._next < len(self.buckets) and (force or self._pending[self._next] == 0):
            for p in self.buckets[self._next]:
                if p.grad is None:
                    self._place(p)
            buf = self.flat[self._next]
            if self.world > 1:
                if self.wire is not None:
                    self.wire[self._next].copy_(buf)
                    buf = self.wire[self._next]
                self._works.append(dist.all_reduce(buf, op=self._op, group=self.group, async_op=True))
            self._next += 1

    def _on_ready(self, p):
        self._place(p)
        if not self._sync:
            return
        i = self._bucket_of[p]
        if i < self._next or self._pending[i] <= 0:
            raise RuntimeError(
                "GradAllReduce: a gradient arrived for a bucket that has already been exchanged or "
                "counted in this step (a second backward before finish()). Run the accumulation "
                "micro-batches inside no_sync() and call finish() after the last backward.")
        self._pending[i] -= 1
        if self.overlap:
            self._launch_ready()

    def finish(self):
        """Launch the remaining buckets, wait for all, average."""
        self._launch_ready(force=True)
        for w in self._works:
            w.wait()
        if self.wire is not None:
            for buf, w in zip(self.flat, self.wire):
                buf.copy_(w)
        if self._divide:
            for buf in self.flat:
                buf.div_(self.world)
        self._reset_state()

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
        trunk.unregister_grad_slots(self.params)
