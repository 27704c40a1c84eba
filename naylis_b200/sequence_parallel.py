"""Sequence-sharded router forward for long-context prefill.

A sequence split across the ranks of a process group (rank j holds rows
[t_base_j, t_base_j + S_j) of every batch row, in rank order) is routed exactly
as the whole sequence on one GPU: ``route_sequence_sharded`` returns the same
router_probs, top_idx and top_gates bit for bit as ``mom_kernels.mom_route`` on
the concatenated input. The reference routes one whole sequence per call
(model.py:169-220) and has no sequence split; this is the exchange its causal
prefix mean needs once the sequence no longer fits one GPU's step.

The exchange (scan_mode "fp64", the default):

1. every rank reduces its shard to per-(b, column) totals: the sum, an upper
   bound of the sum of |x| and the smallest ulp exponent (``mom_route_shard_stats``);
2. one all-gather of those totals (3 x B x d fp64 per rank);
3. each rank forms its carry: the sum of the earlier shards' totals, and the
   whole sequence's exactness certificate per column (``mom_route_shard_carry``).
   A certified column's partial sums are exact in any order, so every rank
   scans its shard at once from that carry;
4. columns whose certificate fails (tiny or huge dynamic range) need the
   sequential fp64 sum of everything before: the ranks then run in rank order,
   each sending its end-of-shard state to the next (point-to-point). All ranks
   see the same count of such columns, so all take the same branch.

scan_mode "fp32" (the sequential fp32 scan of torch's CUDA cumsum) has no
exact form, so its shards always run in rank order, passing the fp32 state.

The per-shard compute is behind ``ShardOps`` so that the exchange itself can be
exercised with gloo ranks on the CPU; ``CudaShardOps`` is the product path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .mom_kernels import _compute_dtype, _dt_code, _ptr, _stream


class ShardOps:
    """Per-shard compute of the exchange (see the module docstring)."""

    def stats(self, x):                                  # -> (3, B, d) fp64
        raise NotImplementedError

    def carry(self, stats_all, world, rank):             # -> ((2, B, d) fp64, int uncertified)
        raise NotImplementedError

    def zero_carry(self, x, scan_mode):                  # rank 0's state in the sequential chain
        raise NotImplementedError

    def route(self, x, t_base, carry_in, want_carry_out, scan_mode):
        """-> (probs, top_idx, gates, carry_out or None)"""
        raise NotImplementedError


class CudaShardOps(ShardOps):
    """The C ABI (``mom_route_shard_stats`` / ``_carry`` / ``mom_route_fwd_shard``)."""

    def __init__(self, w_down, w_up, top_blocks, noise=None, compute_dtype=None):
        self.cd = compute_dtype or _compute_dtype(w_down)
        self.wd = w_down.detach().to(self.cd).contiguous()
        self.wu = w_up.detach().to(self.cd).contiguous()
        self.top = int(top_blocks)
        self.noise = None if noise is None else noise.to(torch.float32).contiguous()

    def stats(self, x):
        B, S, d = x.shape
        out = torch.empty((3, B, d), dtype=torch.float64, device=x.device)
        _lib.call("mom_route_shard_stats", x.data_ptr(), _dt_code(x.dtype), B, S, d, out.data_ptr(),
                  _stream(x.device))
        return out

    def carry(self, stats_all, world, rank):
        _, _, B, d = stats_all.shape
        carry = torch.empty((2, B, d), dtype=torch.float64, device=stats_all.device)
        unc = torch.empty(1, dtype=torch.int32, device=stats_all.device)
        _lib.call("mom_route_shard_carry", stats_all.data_ptr(), world, rank, B, d, carry.data_ptr(),
                  unc.data_ptr(), _stream(stats_all.device))
        return carry, int(unc.item())

    def zero_carry(self, x, scan_mode):
        B, _, d = x.shape
        if scan_mode == "fp32":
            return torch.zeros((B, d), dtype=torch.float32, device=x.device)
        raise RuntimeError("the fp64 chain starts from mom_route_shard_carry's carry")

    def route(self, x, t_base, carry_in, want_carry_out, scan_mode):
        B, S, d = x.shape
        r, nb = self.wd.shape[0], self.wu.shape[0]
        dev = x.device
        probs = torch.empty((B, S, nb), dtype=torch.float32, device=dev)
        top_idx = torch.empty((B, S, self.top), dtype=torch.int64, device=dev)
        gates = torch.empty((B, S, self.top), dtype=torch.float32, device=dev)
        carry_out = torch.empty_like(carry_in) if want_carry_out else None
        ws = torch.empty(_lib.load().mom_route_workspace_size(B, S, d, r, nb, _dt_code(self.cd)),
                         dtype=torch.uint8, device=dev)
        _lib.call("mom_route_fwd_shard", x.data_ptr(), _dt_code(x.dtype), B, S, d, self.wd.data_ptr(),
                  self.wu.data_ptr(), _dt_code(self.cd), r, nb, self.top, _ptr(self.noise),
                  _lib.SCAN_MODES[scan_mode], int(t_base), carry_in.data_ptr(), _ptr(carry_out),
                  probs.data_ptr(), top_idx.data_ptr(), _lib.I64, gates.data_ptr(), None, None,
                  ws.data_ptr(), ws.numel(), _stream(dev))
        return probs, top_idx, gates, carry_out


def _chain(ops, x, t_base, carry, scan_mode, group, rank, world):
    """Shards in rank order: rank j waits for rank j-1's end state, routes its
    shard from it and hands its own end state to rank j+1."""
    if rank > 0:
        dist.recv(carry, src=dist.get_global_rank(group, rank - 1) if group is not None else rank - 1,
                  group=group)
    probs, idx, gates, carry_out = ops.route(x, t_base, carry, rank < world - 1, scan_mode)
    if rank < world - 1:
        dist.send(carry_out, dst=dist.get_global_rank(group, rank + 1) if group is not None else rank + 1,
                  group=group)
    return probs, idx, gates


def route_sequence_sharded(x, w_down=None, w_up=None, top_blocks=None, noise=None, *, group=None,
                           t_base=None, compute_dtype=None, scan_mode: str = "fp64", ops: ShardOps = None):
    """Forward router over a sequence sharded by rows across ``group``.

    x (B, S_local, d): this rank's rows of every sequence; ranks hold
    consecutive row ranges in rank order. t_base: this shard's first global row
    (default rank * S_local: equal shards). noise: this shard's Gumbel noise or
    None. Returns (router_probs, top_idx, top_gates) for the local rows, equal
    bit for bit to ``mom_route`` over the whole sequence. Forward only (the
    prefill the split serves); no autograd.
    """
    if scan_mode not in _lib.SCAN_MODES:
        raise RuntimeError(f"route_sequence_sharded: scan_mode must be one of {sorted(_lib.SCAN_MODES)}")
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    B, S, d = x.shape
    if t_base is None:
        t_base = rank * S
    if ops is None:
        if not x.is_cuda:
            raise RuntimeError("route_sequence_sharded: x must be on a CUDA device")
        ops = CudaShardOps(w_down, w_up, top_blocks, noise, compute_dtype)
    x = x.contiguous()
    if scan_mode == "fp32":
        return _chain(ops, x, t_base, ops.zero_carry(x, scan_mode), scan_mode, group, rank, world)
    stats = ops.stats(x)
    gathered = [torch.empty_like(stats) for _ in range(world)]
    dist.all_gather(gathered, stats, group=group)
    carry, uncertified = ops.carry(torch.stack(gathered), world, rank)
    if uncertified == 0:
        probs, idx, gates, _ = ops.route(x, t_base, carry, False, scan_mode)
        return probs, idx, gates
    return _chain(ops, x, t_base, carry, scan_mode, group, rank, world)
