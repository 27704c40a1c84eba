"""MoMLayer with the reference's constructor, attributes and state-dict keys
(model.py:71-276 of the reference), wired to the sm100 kernels.

``use_kernel=True`` resolves the ``"sm100"`` mode once (fail-loud) and runs
the fused router (``mom_route``) and the bucketed read (``mom_read``).
``use_kernel=False`` is the reference's own default, its eager dense-bias SDPA
path, kept so that a module built with the reference's arguments behaves the
same; it is selected only by that flag, never as a fallback.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import mom_kernels


def _prefix_mean_eager(x):
    cs = torch.cumsum(x.float(), dim=1)
    denom = torch.arange(1, x.shape[1] + 1, device=x.device, dtype=cs.dtype)
    return cs / denom.view(1, -1, 1)


def _gate_bias_eager(top_idx, top_gates, num_blocks, block_size, mask_dtype):
    log_gates = top_gates.clamp_min(1e-9).log().float()
    onehot = F.one_hot(top_idx, num_blocks)
    sel = onehot.any(dim=2)
    bias = torch.einsum("bsk,bske->bse", log_gates, onehot.to(log_gates.dtype))
    bias = bias.masked_fill(~sel, float(torch.finfo(mask_dtype).min))
    return bias.repeat_interleave(block_size, dim=-1)


class MoMLayer(nn.Module):
    """Mixture-of-Memory read over a shared bank, causal router (one routing
    decision per token from the prefix mean of x).

    Same arguments as the reference; ``scan_mode`` picks which torch cumsum the
    router's exact prefix scan reproduces ("fp64": CPU, "fp32": CUDA).
    """

    def __init__(self, d_model: int, n_heads: int, mem_size: int, block_size: int,
                 top_blocks: int, router_rank: int, use_kernel: bool = False,
                 mom_grad_ckpt: bool = False, scan_mode: str = "fp64"):
        super().__init__()
        if d_model % n_heads != 0:
            raise ValueError(f"d_model ({d_model}) must be divisible by n_heads ({n_heads})")
        if mem_size % block_size != 0:
            raise ValueError(f"mem_size ({mem_size}) must be a multiple of block_size ({block_size})")
        if top_blocks > mem_size // block_size:
            raise ValueError(
                f"top_blocks ({top_blocks}) exceeds the number of memory blocks "
                f"({mem_size // block_size} = mem_size {mem_size} // block_size {block_size})")
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
        self.last_router_probs = None
        self.last_top_idx = None
        self.last_entropy = None
        self.last_dead_frac = None
        self.noise_scale = 1.0
        self.use_kernel = use_kernel
        self.mom_grad_ckpt = mom_grad_ckpt
        self.scan_mode = scan_mode
        self._kernel_mode = None

    def _resolve_kernel(self, x):
        mode = mom_kernels.resolve_mode(x.device, torch.bfloat16 if torch.is_autocast_enabled("cuda")
                                        else x.dtype, head_dim=self.head_dim)
        mom_kernels.announce(mode)
        return mode

    # ------------------------------------------------------------- router
    def _route_eager(self, x):
        h = _prefix_mean_eager(x).to(self.router_down.weight.dtype)
        logits = self.router_up(torch.tanh(self.router_down(h))).float()
        if self.training and self.noise_scale > 0:
            gumbel = -torch.log(-torch.log(torch.rand_like(logits) + 1e-9) + 1e-9)
            noisy = logits + self.noise_scale * gumbel
        else:
            noisy = logits
        probs = F.softmax(logits, dim=-1)
        top_values, top_idx = noisy.topk(self.top_blocks, dim=-1)
        return probs, top_idx, F.softmax(top_values, dim=-1)

    def _route_kernel(self, x):
        B, S, _ = x.shape
        noise = None
        if self.training and self.noise_scale > 0:
            noise = mom_kernels.gumbel_noise((B, S, self.num_blocks), x.device, self.noise_scale)
        # probs, top_idx, top_gates and log(max(top_gates, 1e-9)) from the router kernel:
        # the read takes the log-gates (the gradient flows back into the router kernel
        # without torch's clamp / log ops)
        return mom_kernels.mom_route_log_gates(x, self.router_down.weight, self.router_up.weight,
                                               self.top_blocks, noise, scan_mode=self.scan_mode)

    def forward(self, x, M_blocks):
        if self.use_kernel:
            if self._kernel_mode is None:
                self._kernel_mode = self._resolve_kernel(x)
            mode = self._kernel_mode
        else:
            mode = None
        if mode is not None:
            router_probs, top_idx, _, gate_in = self._route_kernel(x)
        else:
            router_probs, top_idx, gate_in = self._route_eager(x)
        if self.training:
            self.last_router_probs = router_probs.reshape(-1, self.num_blocks)
            self.last_top_idx = top_idx.reshape(-1, self.top_blocks)
        if self.mom_grad_ckpt and self.training and torch.is_grad_enabled():
            out = torch.utils.checkpoint.checkpoint(
                self._read, x, top_idx, gate_in, M_blocks, mode,
                use_reentrant=False, preserve_rng_state=False)
        else:
            out = self._read(x, top_idx, gate_in, M_blocks, mode)
        if mode is not None and torch.result_type(self.mom_scale, out) == torch.float32:
            return mom_kernels.mom_scale(out, self.mom_scale)
        return self.mom_scale * out

    def _read(self, x, top_idx, gate_in, M_blocks, mode=None):
        """gate_in: the log-gates on the kernel path (mode set), the gates on the
        reference's eager path."""
        B, S, D = x.shape
        q_sh = self.q_proj(x).view(B, S, self.n_heads, self.head_dim)
        L = self.mem_slots
        slots = M_blocks.view(L, D)
        k_shared = self.k_proj(slots)
        v_shared = self.v_proj(slots)
        if mode is not None:
            out = mom_kernels.mom_read_log_gates(q_sh, k_shared, v_shared, top_idx, gate_in,
                                                 num_blocks=self.num_blocks, block_size=self.block_size,
                                                 mode=mode)
        else:
            bias = _gate_bias_eager(top_idx, gate_in, self.num_blocks, self.block_size, q_sh.dtype)
            q = q_sh.transpose(1, 2)
            k = k_shared.view(1, L, self.n_heads, self.head_dim).transpose(1, 2).expand(B, -1, -1, -1)
            v = v_shared.view(1, L, self.n_heads, self.head_dim).transpose(1, 2).expand(B, -1, -1, -1)
            out = F.scaled_dot_product_attention(q, k, v, attn_mask=bias.unsqueeze(1).to(q.dtype),
                                                 is_causal=False)
            out = out.transpose(1, 2)
        return self.o_proj(out.reshape(B, S, D))
