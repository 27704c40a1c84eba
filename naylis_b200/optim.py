"""AdamW for fp32 CUDA parameters in one kernel launch (csrc/optim.cu).

The reference optimises with torch's AdamW (pretrain.py's HF Trainer, optim
"adamw_torch": decoupled weight decay). This class has the same update rule,
hyper-parameters and per-parameter state names (``step``, ``exp_avg``,
``exp_avg_sq``), so its state dict reads like torch's. Two differences in how it
runs:

* every parameter of a group is updated by one launch over a device table of
  (param, grad, exp_avg, exp_avg_sq) pointers, cached while the pointers stay
  the same;
* a parameter that the decoder's bf16 projections registered a bf16 copy for
  (``trunk.linear_f32grad``) gets that copy rewritten in the same pass, and is
  marked fresh, so the next forward reads it instead of casting the fp32 weight
  again.

Parameters without a gradient are skipped, as torch does. Only fp32,
contiguous CUDA parameters and gradients are taken; anything else raises. The
parameters updated together (those of a group with a gradient) share one step
count, kept with the group's launch plan while training and written to every
parameter's ``step`` state when the state dict is taken; a parameter that joins
later with another step count raises.
"""
from __future__ import annotations

import struct

import torch

from . import _lib, trunk

_CHUNK = 65536          # elements per CTA (kOptChunk in csrc/launch.h); a table entry is 48 bytes


def _pack_entries(entries) -> bytes:
    """The device table's bytes: per tensor {p, g, m, v, p16} as 64-bit addresses
    (0 for no bf16 copy) and the element count (int64), little-endian, 48 bytes."""
    return b"".join(struct.pack("<5Qq", p, g, m, v, p16, n) for p, g, m, v, p16, n in entries)


class _Plan:
    """One group's launch: its parameters, the device tables and the step count."""

    def __init__(self, sig, gen, params, shadowed, table, clist, nchunks, step):
        self.sig, self.gen, self.params, self.shadowed = sig, gen, params, shadowed
        self.table, self.clist, self.nchunks, self.step = table, clist, nchunks, step


class AdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2):
        if lr < 0 or eps < 0 or weight_decay < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError("AdamW: invalid hyper-parameters")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self._plans = {}

    def _plan(self, gi, params, sig):
        """Build (or rebuild, when pointers, bf16 rows or membership changed) the
        group's tables. Every parameter of a plan steps together: their states
        must share one step count."""
        steps = set()
        for p in params:
            if not (p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()):
                raise RuntimeError("naylis_b200.optim.AdamW takes contiguous fp32 CUDA parameters")
            g = p.grad
            if not (g.dtype == torch.float32 and g.is_contiguous() and g.device == p.device):
                raise RuntimeError("naylis_b200.optim.AdamW takes contiguous fp32 gradients")
            st = self.state[p]
            if not st:
                st["step"] = torch.tensor(0.0)
                st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            steps.add(int(st["step"].item()))
        if len(steps) != 1:
            raise RuntimeError("naylis_b200.optim.AdamW: the parameters of a group must share one step count")
        entries, shadowed = [], []
        for p in params:
            st = self.state[p]
            shadow = trunk.bf16_copy(p)
            p16 = shadow.data_ptr() if shadow is not None and shadow.numel() == p.numel() else 0
            if p16:
                shadowed.append(p)
            entries.append((p.data_ptr(), p.grad.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(),
                            p16, p.numel()))
        chunks = [(ti, ci) for ti, e in enumerate(entries) for ci in range((e[5] + _CHUNK - 1) // _CHUNK)]
        dev = params[0].device
        table = torch.frombuffer(bytearray(_pack_entries(entries)), dtype=torch.uint8).to(dev)
        clist = torch.tensor(chunks, dtype=torch.int32).reshape(-1).to(dev)
        plan = _Plan(sig, trunk.bf16_generation(), params, shadowed, table, clist, len(chunks), steps.pop())
        self._plans[gi] = plan
        return plan

    def state_dict(self):
        self._sync_steps()
        return super().state_dict()

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        self._plans = {}

    def _sync_steps(self):
        for plan in self._plans.values():
            for p in plan.params:
                self.state[p]["step"].fill_(float(plan.step))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for gi, group in enumerate(self.param_groups):
            b1, b2 = group["betas"]
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            sig = [(p.data_ptr(), p.grad.data_ptr()) for p in params]
            plan = self._plans.get(gi)
            if plan is None or plan.sig != sig or plan.gen != trunk.bf16_generation():
                if plan is not None:
                    self._sync_steps()
                plan = self._plan(gi, params, sig)
            plan.step += 1
            dev = params[0].device
            _lib.call("mom_adamw_step", plan.table.data_ptr(), len(params), plan.clist.data_ptr(), plan.nchunks,
                      float(group["lr"]), float(b1), float(b2), float(group["eps"]), float(group["weight_decay"]),
                      plan.step, torch.cuda.current_stream(dev).cuda_stream)
            # the kernel wrote the parameters in place: tell autograd, and mark the bf16 copies fresh
            torch.autograd.graph.increment_version(params)
            for p in plan.shadowed:
                trunk.mark_bf16_fresh(p)
        return loss


__all__ = ["AdamW"]
