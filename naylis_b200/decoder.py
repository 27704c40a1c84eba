"""The Naylis decoder (a Llama trunk with a Mixture-of-Memory read in every
layer) driving the sm100 MoM kernels: BASELINE config 3's training step.

It is the caller of the hot path that the reference trains
(``NaylisLlamaForCausalLM``, model.py:350-560 of the reference, built by
pretrain.py:184-207): per layer

    x = x + attn(input_layernorm(x))          causal self-attention with RoPE
    x = x + mom(mom_norm(x), M_blocks)        the memory read (sm100 kernels)
    x = x + mlp(post_attention_layernorm(x))  SwiGLU

with one bank ``M_blocks`` shared by all layers, a final RMSNorm, an LM head
tied to the token embedding, the shifted cross-entropy summed in fp32 over the
valid labels, and the MoM load-balancing aux loss (model.py:476-517) added with
weight ``mom_aux_weight`` in training.

Parameter names and shapes are the reference's (``model.embed_tokens``,
``model.layers.{i}.self_attn.{q,k,v,o}_proj``, ``...mlp.{gate,up,down}_proj``,
``...input_layernorm`` / ``post_attention_layernorm`` / ``mom_norm``,
``...mom.*``, ``model.M_blocks``, ``model.norm``, ``lm_head`` tied), so a
reference checkpoint loads with ``load_state_dict``.

The trunk runs on torch's CUDA kernels (cuBLAS GEMMs, the flash attention
backend of scaled_dot_product_attention); the MoM router and read run on this
package's sm_100a kernels. Layout choices that differ from a module-by-module
port: q/k/v and gate/up each run as ONE GEMM over their concatenated weights
(wider N per tensor-core launch; the weights stay separate parameters); in bf16
the rotary embedding, the SwiGLU gate and every residual add with the RMSNorm
after it are fused kernels (csrc/trunk.cu) with the reference's rounding
points: the rotation writes q/k/v straight into the token-major layout
attention reads, the add + norm writes the fp32 residual stream and the bf16
input of the next projection in one pass, and the layer's mom_scale factor
rides on the add that follows the memory read. The rotary tables are built
once per forward for all layers. The loss reads the LM head's bf16 logits once
(csrc/trunk.cu, cross-entropy): the fp32 copy of the logits and torch's fp32
log-softmax are never formed.
"""
from __future__ import annotations

import dataclasses
import math

import torch
import torch.nn as nn
import torch.nn.functional as F
import torch.utils.checkpoint

from . import mom_kernels as mk
from . import trunk
from .model import MoMLayer


@dataclasses.dataclass
class NaylisConfig:
    """The architecture keys of the reference's LlamaConfig + [naylis] table
    (pretrain.py:184-207; configs/naylisMoM.toml). Defaults: BASELINE config 3."""
    vocab_size: int = 32000
    hidden_size: int = 1024
    intermediate_size: int = 2816
    num_hidden_layers: int = 20
    num_attention_heads: int = 16
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    initializer_range: float = 0.02
    mem_size: int = 1024
    mom_block_size: int = 128
    mom_top_blocks: int = 2
    mom_router_rank: int = 32
    mom_aux_weight: float = 0.01
    mom_grad_ckpt: bool = False
    grad_ckpt: bool = False
    scan_mode: str = "fp32"

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


class RMSNorm(nn.Module):
    """Llama RMSNorm: weight * (x / sqrt(mean(x^2) + eps)) in fp32, returned in
    x's dtype scaled by the (fp32) weight."""

    def __init__(self, d: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        with torch.autocast("cuda", enabled=False):
            y = F.rms_norm(x.float(), (x.shape[-1],), eps=self.eps).to(x.dtype)
            return self.weight * y


def rope_tables(seq_len: int, head_dim: int, theta: float, device):
    """cos / sin (S, head_dim) fp32 of the rotary embedding, the two halves of
    the head dimension sharing one frequency (Llama's rotate-half layout)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(seq_len, device=device, dtype=torch.float32)
    freqs = torch.outer(pos, inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(t, cos, sin):
    """t (B, H, S, hd): t * cos + rotate_half(t) * sin, in fp32."""
    t = t.float()
    half = t.shape[-1] // 2
    rot = torch.cat((-t[..., half:], t[..., :half]), dim=-1)
    return t * cos + rot * sin


def _bf16_path(x) -> bool:
    """The decoder's bf16 kernel path: CUDA activations in bf16 under CUDA bf16
    autocast (the residual stream's RMSNorm kernels hand bf16 to every projection)."""
    return x.is_cuda and x.dtype == torch.bfloat16 and torch.is_autocast_enabled("cuda")


class SelfAttention(nn.Module):
    def __init__(self, cfg: NaylisConfig):
        super().__init__()
        d = cfg.hidden_size
        self.n_heads = cfg.num_attention_heads
        self.head_dim = cfg.head_dim
        self.q_proj = nn.Linear(d, d, bias=False)
        self.k_proj = nn.Linear(d, d, bias=False)
        self.v_proj = nn.Linear(d, d, bias=False)
        self.o_proj = nn.Linear(d, d, bias=False)

    def forward(self, x, cos, sin):
        B, S, d = x.shape
        if _bf16_path(x):
            qkv = trunk.linear_f32grad(x, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
            # fused rotary embedding into attention's layout (csrc/trunk.cu)
            q, k, v = trunk.rope_qkv(qkv, cos, sin, self.n_heads)
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            return trunk.linear_f32grad(o.transpose(1, 2).reshape(B, S, d), self.o_proj.weight)
        w = torch.cat((self.q_proj.weight, self.k_proj.weight, self.v_proj.weight), dim=0)
        qkv = F.linear(x, w)
        if qkv.is_cuda and qkv.dtype == torch.bfloat16:
            q, k, v = trunk.rope_qkv(qkv, cos, sin, self.n_heads)
        else:
            qkv = qkv.view(B, S, 3, self.n_heads, self.head_dim)
            q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
            q = apply_rope(q, cos, sin)
            k = apply_rope(k, cos, sin)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.o_proj(o.transpose(1, 2).reshape(B, S, d))


class SwiGLU(nn.Module):
    def __init__(self, cfg: NaylisConfig):
        super().__init__()
        d, f = cfg.hidden_size, cfg.intermediate_size
        self.gate_proj = nn.Linear(d, f, bias=False)
        self.up_proj = nn.Linear(d, f, bias=False)
        self.down_proj = nn.Linear(f, d, bias=False)

    def forward(self, x):
        if _bf16_path(x):
            gu = trunk.linear_f32grad(x, self.gate_proj.weight, self.up_proj.weight)
            return trunk.linear_f32grad(trunk.swiglu(gu), self.down_proj.weight)   # fused (csrc/trunk.cu)
        gu = F.linear(x, torch.cat((self.gate_proj.weight, self.up_proj.weight), dim=0))
        if gu.is_cuda and gu.dtype == torch.bfloat16:
            return self.down_proj(trunk.swiglu(gu))      # fused (csrc/trunk.cu)
        g, u = gu.chunk(2, dim=-1)
        return self.down_proj(F.silu(g) * u)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: NaylisConfig):
        super().__init__()
        d = cfg.hidden_size
        self.self_attn = SelfAttention(cfg)
        self.mlp = SwiGLU(cfg)
        self.input_layernorm = RMSNorm(d, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(d, cfg.rms_norm_eps)
        self.mom_norm = RMSNorm(d, cfg.rms_norm_eps)
        self.mom = MoMLayer(d, cfg.num_attention_heads, cfg.mem_size, cfg.mom_block_size, cfg.mom_top_blocks,
                            cfg.mom_router_rank, mom_grad_ckpt=cfg.mom_grad_ckpt, scan_mode=cfg.scan_mode)
        self.grad_ckpt = cfg.grad_ckpt

    def _ckpt(self, fn, *args):
        if self.grad_ckpt and self.training and torch.is_grad_enabled():
            return torch.utils.checkpoint.checkpoint(fn, *args, use_reentrant=False, preserve_rng_state=False)
        return fn(*args)

    def forward(self, x, M_blocks, cos, sin):
        x = x + self._ckpt(lambda h: self.self_attn(self.input_layernorm(h), cos, sin), x)
        x = x + self.mom(self.mom_norm(x), M_blocks)
        return x + self._ckpt(lambda h: self.mlp(self.post_attention_layernorm(h)), x)

    def grad_groups(self):
        """Weights whose gradients one GEMM produces, in that GEMM's row order."""
        a, m = self.self_attn, self.mlp
        return [(a.q_proj.weight, a.k_proj.weight, a.v_proj.weight), (m.gate_proj.weight, m.up_proj.weight),
                *self.mom.grad_groups()]

    def forward_fused(self, x, pending, pending_scale, M_blocks, cos, sin):
        """bf16 path: each residual add runs inside the RMSNorm that follows it
        (csrc/trunk.cu add_rmsnorm). x is the residual stream before `pending`,
        the previous sublayer's output (times pending_scale), is added; returns
        the stream and this layer's MLP output, still to be added."""
        eps = self.input_layernorm.eps
        x, y = trunk.add_rmsnorm(x, pending, self.input_layernorm.weight, eps, scale=pending_scale)
        a = self.self_attn(y, cos, sin)
        x, y16, y32 = trunk.add_rmsnorm(x, a, self.mom_norm.weight, eps, want_f32=True)
        o = self.mom.forward_unscaled(y32, M_blocks, x_lowp=y16)
        # mom_scale * o_proj(read) folded into the add (model.py:239 of the reference)
        x, y = trunk.add_rmsnorm(x, o, self.post_attention_layernorm.weight, eps, scale=self.mom.mom_scale)
        return x, self.mlp(y)


class NaylisModel(nn.Module):
    def __init__(self, cfg: NaylisConfig):
        super().__init__()
        nb = cfg.mem_size // cfg.mom_block_size
        # registered first: its gradient, summed over every layer, is complete
        # only at the end of the backward, so its bucket is the last exchanged
        self.M_blocks = nn.Parameter(torch.randn(nb, cfg.mom_block_size * cfg.hidden_size) * 0.02)
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.cfg = cfg

    def grad_groups(self):
        return [g for layer in self.layers for g in layer.grad_groups()]

    def forward(self, input_ids):
        x = self.embed_tokens(input_ids)
        cos, sin = rope_tables(input_ids.shape[1], self.cfg.head_dim, self.cfg.rope_theta, x.device)
        fused = (x.is_cuda and x.dtype == torch.float32 and torch.is_autocast_enabled("cuda")
                 and torch.get_autocast_dtype("cuda") == torch.bfloat16 and not self.cfg.grad_ckpt
                 and self.cfg.hidden_size in (128, 256, 512, 1024, 2048))
        if fused:
            pending = None
            for layer in self.layers:
                x, pending = layer.forward_fused(x, pending, None, self.M_blocks, cos, sin)
            _, y = trunk.add_rmsnorm(x, pending, self.norm.weight, self.norm.eps)
            return y
        for layer in self.layers:
            x = layer(x, self.M_blocks, cos, sin)
        return self.norm(x)


class NaylisForCausalLM(nn.Module):
    """Causal LM: tied LM head, fp32 cross-entropy, MoM aux loss in training."""

    def __init__(self, cfg: NaylisConfig):
        super().__init__()
        self.config = cfg
        self.model = NaylisModel(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.model.embed_tokens.weight
        self.mom_aux_weight = cfg.mom_aux_weight
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        """The reference's initialisation: Linear and Embedding weights
        N(0, initializer_range), norms 1, bank N(0, 0.02), mom_scale 0."""
        std = self.config.initializer_range
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                m.weight.normal_(0.0, std)
            elif isinstance(m, RMSNorm):
                m.weight.fill_(1.0)
            elif isinstance(m, MoMLayer):
                m.mom_scale.zero_()
        self.model.M_blocks.normal_(0.0, 0.02)

    def grad_groups(self):
        """Parameter groups a gradient bucketing wrapper keeps contiguous and in
        order (data_parallel.GradAllReduce), so the fused q/k/v and gate/up
        weight-gradient GEMMs can write into the buckets directly."""
        return self.model.grad_groups()

    def mom_layers(self):
        return [layer.mom for layer in self.model.layers]

    def mom_aux_loss(self, device):
        """num_blocks * sum_b(frac_selected_b * mean_prob_b), averaged over the
        MoM layers (model.py:476-517); also records each layer's router entropy
        and dead-block fraction, then clears the stashed routing."""
        aux = torch.zeros((), device=device, dtype=torch.float32)
        count = 0
        for m in self.mom_layers():
            if m.last_router_probs is None or m.last_top_idx is None:
                continue
            if m.last_router_probs.is_cuda:
                # one fused kernel per layer (csrc/route.cu, router_aux)
                st = mk.router_aux(m.last_router_probs, m.last_top_idx, m.num_blocks)
                aux = aux + st[0]
                m.last_entropy = st[1].detach()
                m.last_dead_frac = st[2].detach()
                m.last_router_probs = None
                m.last_top_idx = None
                count += 1
                continue
            probs = m.last_router_probs.float()
            blocks = torch.arange(m.num_blocks, device=probs.device)
            sel = (m.last_top_idx.unsqueeze(2) == blocks.view(1, 1, -1)).any(1)
            frac = sel.to(probs.dtype).mean(dim=0)
            aux = aux + m.num_blocks * (frac * probs.mean(dim=0)).sum()
            with torch.no_grad():
                m.last_entropy = -(probs * probs.clamp_min(1e-9).log()).sum(-1).mean()
                m.last_dead_frac = (~sel.any(0)).to(probs.dtype).mean()
            m.last_router_probs = None
            m.last_top_idx = None
            count += 1
        return aux / count if count else aux

    def forward(self, input_ids, labels=None):
        """labels given: the scalar training loss (LM loss + aux weight x aux in
        training). Otherwise the logits (B, S, vocab)."""
        h = self.model(input_ids)
        if labels is None:
            return self.lm_head(h)
        if _bf16_path(h):
            # every position through the head, the last of each sequence with an ignored
            # label: the same loss as the reference's h[:, :-1] / labels[:, 1:] shift, without
            # the copy of the sliced activations and the scatter of its gradient
            shift_labels = torch.full_like(labels, -100)
            shift_labels[:, :-1] = labels[:, 1:]
            shift_labels = shift_labels.reshape(-1)
            logits = trunk.linear_f32grad(h.reshape(-1, h.shape[-1]), self.lm_head.weight)
        else:
            shift_labels = labels[:, 1:].reshape(-1)
            logits = self.lm_head(h[:, :-1].reshape(-1, h.shape[-1]))
        if logits.is_cuda and logits.dtype == torch.bfloat16:
            # fused (csrc/trunk.cu): the same fp32 math on the bf16 logits, no fp32 copy
            loss = trunk.cross_entropy_sum(logits, shift_labels)
        else:
            loss = F.cross_entropy(logits.float(), shift_labels, reduction="sum")
        loss = loss / (shift_labels != -100).sum().clamp_min(1)
        if self.training:
            loss = loss + self.mom_aux_weight * self.mom_aux_loss(h.device)
        return loss


def flops_per_token(cfg: NaylisConfig, seq_len: int, tokens_per_step: int) -> float:
    """Forward FLOPs per token of the decoder: per layer the q/k/v/o GEMMs
    (8 d^2), causal attention (2 S d: half of the S x S scores and their PV),
    the SwiGLU (6 d f), the MoM q/o GEMMs (4 d^2), the read over the active
    slots (4 La d), the router (2 (d r + r nb)) and the bank's k/v projections
    (4 L d^2 once per step, spread over the step's tokens on this GPU); plus
    the LM head (2 d V). A training step is 3x this (backward = 2x forward)."""
    d, f, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    nb = cfg.mem_size // cfg.mom_block_size
    La = cfg.mom_top_blocks * cfg.mom_block_size
    r = cfg.mom_router_rank
    L = cfg.mem_size
    per_layer = (8 * d * d + 2 * seq_len * d + 6 * d * f + 4 * d * d + 4 * La * d + 2 * (d * r + r * nb)
                 + 4 * L * d * d / tokens_per_step)
    return cfg.num_hidden_layers * per_layer + 2 * d * V


def param_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


__all__ = ["NaylisConfig", "NaylisForCausalLM", "flops_per_token", "param_count", "rope_tables", "apply_rope",
           "RMSNorm"]
