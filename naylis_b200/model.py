"""MoMLayer of the sm100 backend: the reference's constructor, attributes and
state-dict keys (model.py:71-158 of the reference), running the fused router
and the bucketed read through the ``"sm100"`` door.

The module exists so that a reference checkpoint loads as is and the trunk
in ``naylis_b200.decoder`` can call the kernels directly. It has no eager
path: the reference's own ``model.MoMLayer`` with ``use_kernel=False`` is that
path. Building this layer with ``use_kernel=False`` raises.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import mom_kernels, trunk


class MoMLayer(nn.Module):
    """Mixture-of-Memory read over a shared bank with the causal router (one
    routing decision per token from the prefix mean of x).

    Same arguments as the reference. ``scan_mode`` picks which torch cumsum
    the router's exact prefix scan reproduces bit for bit: ``"fp32"`` (the
    default) is torch's CUDA cumsum, i.e. what the reference's eager layer
    computes on the same GPU; ``"fp64"`` is torch's CPU cumsum.
    """

    def __init__(self, d_model: int, n_heads: int, mem_size: int, block_size: int,
                 top_blocks: int, router_rank: int, use_kernel: bool = True,
                 mom_grad_ckpt: bool = False, scan_mode: str = "fp32"):
        super().__init__()
        if d_model % n_heads != 0:
            raise ValueError(f"d_model ({d_model}) must be divisible by n_heads ({n_heads})")
        if mem_size % block_size != 0:
            raise ValueError(f"mem_size ({mem_size}) must be a multiple of block_size ({block_size})")
        if top_blocks > mem_size // block_size:
            raise ValueError(
                f"top_blocks ({top_blocks}) exceeds the number of memory blocks "
                f"({mem_size // block_size} = mem_size {mem_size} // block_size {block_size})")
        if not use_kernel:
            raise ValueError(
                "naylis_b200.model.MoMLayer runs the sm100 kernels only; the eager SDPA path "
                "(use_kernel=False) is the reference's own model.MoMLayer")
        self.num_blocks = mem_size // block_size
        self.block_size = block_size
        self.top_blocks = top_blocks
        self.mem_slots = mem_size
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.router_down = nn.Linear(d_model, router_rank, bias=False)
        self.router_up = nn.Linear(router_rank, self.num_blocks, bias=False)
        self.q_proj = nn.Linear(d_model, d_model, bias=False)
        self.k_proj = nn.Linear(d_model, d_model, bias=False)
        self.v_proj = nn.Linear(d_model, d_model, bias=False)
        self.o_proj = nn.Linear(d_model, d_model, bias=False)
        self.mom_scale = nn.Parameter(torch.zeros(1))
        # routing statistics for the load-balancing aux loss (training only)
        self.last_router_probs = None
        self.last_top_idx = None
        self.last_entropy = None
        self.last_dead_frac = None
        self.noise_scale = 1.0
        self.use_kernel = True
        self.mom_grad_ckpt = mom_grad_ckpt
        self.scan_mode = scan_mode
        self._kernel_mode = None

    def _resolve(self, x):
        if self._kernel_mode is None:
            self._kernel_mode = mom_kernels.resolve_mode(x.device, x.dtype, head_dim=self.head_dim)
            mom_kernels.announce(self._kernel_mode)
        return self._kernel_mode

    def forward(self, x, M_blocks):
        """x (B, S, d_model), M_blocks (num_blocks, block_size * d_model) ->
        mom_scale * o_proj(read) (B, S, d_model), fp32 when mom_scale is."""
        out = self.forward_unscaled(x, M_blocks)
        if torch.result_type(self.mom_scale, out) == torch.float32:
            return mom_kernels.mom_scale(out, self.mom_scale)
        return self.mom_scale * out

    def forward_unscaled(self, x, M_blocks, x_lowp=None):
        """o_proj(read) before the mom_scale factor, for a caller that folds the
        factor into the residual add that follows (the decoder's fused add +
        RMSNorm). x feeds the router (its prefix scan sees x's own values);
        x_lowp, when given, is the same activations already rounded to bf16
        (to nearest even), for the q projection and the router's backward."""
        mode = self._resolve(x)
        B, S, _ = x.shape
        noise = None
        if self.training and self.noise_scale > 0:
            noise = mom_kernels.gumbel_noise((B, S, self.num_blocks), x.device, self.noise_scale)
        # probs, top_idx, gates and log(max(gates, 1e-9)) from the router kernel; the read
        # takes the log-gates, whose gradient goes straight back into the router kernel
        probs, top_idx, _, log_gates = mom_kernels.mom_route_log_gates(
            x, self.router_down.weight, self.router_up.weight, self.top_blocks, noise,
            scan_mode=self.scan_mode, x_lowp=x_lowp)
        if self.training:
            self.last_router_probs = probs.reshape(-1, self.num_blocks)
            self.last_top_idx = top_idx.reshape(-1, self.top_blocks)
        xq = x if x_lowp is None else x_lowp
        if self.mom_grad_ckpt and self.training and torch.is_grad_enabled():
            # the read holds no RNG draw, so its recompute is exact
            return torch.utils.checkpoint.checkpoint(
                self._read, xq, top_idx, log_gates, M_blocks, mode,
                use_reentrant=False, preserve_rng_state=False)
        return self._read(xq, top_idx, log_gates, M_blocks, mode)

    def grad_groups(self):
        """The bank's k and v weights, whose gradients one GEMM produces (k rows first)."""
        return [(self.k_proj.weight, self.v_proj.weight)]

    @staticmethod
    def _proj(lin, x):
        """lin(x); under CUDA bf16 autocast the bf16 GEMM with fp32 weight
        gradients (trunk.linear_f32grad) instead of autocast's cast + linear."""
        if x.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
            return trunk.linear_f32grad(x, lin.weight)
        return lin(x)

    def _read(self, x, top_idx, log_gates, M_blocks, mode):
        B, S, D = x.shape
        q_sh = self._proj(self.q_proj, x).view(B, S, self.n_heads, self.head_dim)
        if M_blocks.is_cuda and torch.is_autocast_enabled("cuda") and \
                torch.get_autocast_dtype("cuda") == torch.bfloat16 and M_blocks.dtype == torch.float32:
            # both bank projections in one GEMM over the bank's bf16 copy
            k_shared, v_shared = trunk.bank_kv(M_blocks, self.k_proj.weight, self.v_proj.weight, self.mem_slots)
        else:
            slots = M_blocks.view(self.mem_slots, D)
            k_shared = self._proj(self.k_proj, slots)
            v_shared = self._proj(self.v_proj, slots)
        out = mom_kernels.mom_read_log_gates(q_sh, k_shared, v_shared, top_idx, log_gates,
                                             num_blocks=self.num_blocks, block_size=self.block_size,
                                             mode=mode)
        return self._proj(self.o_proj, out.reshape(B, S, D))
