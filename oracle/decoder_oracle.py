"""CPU restatement of the reference's Naylis decoder training step — TEST
INFRASTRUCTURE ONLY (the checker and the timed CPU baseline; nothing in the
product imports it).

It restates, in plain torch on the host, what the reference's
``NaylisLlamaForCausalLM`` (model.py:350-560, on transformers' Llama modules)
computes for a training forward:

* token embedding; per layer RMSNorm -> causal self-attention with rotary
  embeddings (rotate-half layout, theta from the config) -> residual;
  RMSNorm -> MoM read (model.py:189-276) -> residual; RMSNorm -> SwiGLU ->
  residual; final RMSNorm; LM head tied to the embedding;
* the MoM read as the reference's eager path: prefix mean by torch.cumsum over
  fp32 divided by t+1 (model.py:169-176), router W_up tanh(W_down h)
  (model.py:178-187), softmax probabilities, top-k of the logits, softmax
  gates (model.py:209-220), the dense per-token bias log(max(g, 1e-9)) on the
  selected blocks and the dtype's lowest value elsewhere
  (mom_kernels/reference.py:14-29), attention of q over all bank slots with
  that bias (model.py:262-275), o_proj, times mom_scale (model.py:239);
* the loss: cross-entropy of the shifted logits summed in fp32 over the valid
  labels and divided by their count (model.py:539-551), plus
  aux_weight x the load-balancing aux loss averaged over the layers
  (model.py:476-517).

Parameters are a dict in the reference's names (``model.layers.{i}.mom.q_proj.weight``
...). It is pinned to the reference itself by tests/test_oracle_golden.py
against tests/golden/decoder_small_f32.npz, which the reference's own model
produced (tests/golden/make_golden.py).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x, w, eps):
    xf = x.float()
    return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def rope(t, cos, sin):
    half = t.shape[-1] // 2
    return t * cos + torch.cat((-t[..., half:], t[..., :half]), dim=-1) * sin


def rope_cos_sin(S, hd, theta):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))
    ang = torch.arange(S, dtype=torch.float32)[:, None] * inv[None, :]
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos(), ang.sin()


def attention(x, p, pre, H, cos, sin):
    B, S, d = x.shape
    hd = d // H
    q = F.linear(x, p[pre + "q_proj.weight"]).view(B, S, H, hd).transpose(1, 2)
    k = F.linear(x, p[pre + "k_proj.weight"]).view(B, S, H, hd).transpose(1, 2)
    v = F.linear(x, p[pre + "v_proj.weight"]).view(B, S, H, hd).transpose(1, 2)
    q, k = rope(q, cos, sin), rope(k, cos, sin)
    sc = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
    causal = torch.ones(S, S, dtype=torch.bool).triu(1)
    sc = sc.masked_fill(causal, float("-inf"))
    o = torch.softmax(sc.float(), dim=-1).to(v.dtype) @ v
    return F.linear(o.transpose(1, 2).reshape(B, S, d), p[pre + "o_proj.weight"])


def swiglu(x, p, pre):
    return F.linear(F.silu(F.linear(x, p[pre + "gate_proj.weight"])) * F.linear(x, p[pre + "up_proj.weight"]),
                    p[pre + "down_proj.weight"])


def mom_read(x, M, p, pre, geo, stats):
    """One MoM layer; appends (probs, top_idx) to ``stats`` for the aux loss."""
    B, S, d = x.shape
    H, nb, bs, top = geo["H"], geo["nb"], geo["bs"], geo["top"]
    hd = d // H
    L = nb * bs
    h = torch.cumsum(x.float(), dim=1) / torch.arange(1, S + 1, dtype=torch.float32).view(1, -1, 1)
    h = h.to(p[pre + "router_down.weight"].dtype)
    logits = F.linear(torch.tanh(F.linear(h, p[pre + "router_down.weight"])), p[pre + "router_up.weight"]).float()
    probs = torch.softmax(logits, dim=-1)
    vals, idx = logits.topk(top, dim=-1)
    gates = torch.softmax(vals, dim=-1)
    stats.append((probs.reshape(-1, nb), idx.reshape(-1, top)))
    q = F.linear(x, p[pre + "q_proj.weight"]).view(B, S, H, hd).transpose(1, 2)
    slots = M.view(L, d)
    k = F.linear(slots, p[pre + "k_proj.weight"]).view(L, H, hd).transpose(0, 1)
    v = F.linear(slots, p[pre + "v_proj.weight"]).view(L, H, hd).transpose(0, 1)
    # dense bias over all slots: sum of the log-gates of the token's picks of a
    # block (a block picked twice sums), the lowest value of q's dtype elsewhere
    onehot = F.one_hot(idx, nb).to(torch.float32)                       # (B,S,top,nb)
    blk = torch.einsum("bst,bstn->bsn", gates.clamp_min(1e-9).log(), onehot)
    blk = blk.masked_fill(onehot.sum(2) == 0, torch.finfo(q.dtype).min)
    bias = blk.repeat_interleave(bs, dim=-1).to(q.dtype)               # (B,S,L)
    sc = (q @ k.transpose(-1, -2).unsqueeze(0)) / math.sqrt(hd) + bias.unsqueeze(1)
    o = torch.softmax(sc.float(), dim=-1).to(v.dtype) @ v.unsqueeze(0)
    out = F.linear(o.transpose(1, 2).reshape(B, S, d), p[pre + "o_proj.weight"])
    return p[pre + "mom_scale"] * out


def aux_loss(stats, nb):
    aux = torch.zeros((), dtype=torch.float32)
    for probs, idx in stats:
        sel = (idx.unsqueeze(2) == torch.arange(nb).view(1, 1, -1)).any(1).float()
        aux = aux + nb * (sel.mean(0) * probs.float().mean(0)).sum()
    return aux / max(len(stats), 1)


def forward(ids, p, geo, labels=None):
    """The training forward: the loss with labels, the logits without."""
    x = F.embedding(ids, p["model.embed_tokens.weight"])
    B, S = ids.shape
    cos, sin = rope_cos_sin(S, geo["d"] // geo["H"], geo["rope_theta"])
    stats = []
    for i in range(geo["layers"]):
        pre = f"model.layers.{i}."
        x = x + attention(rms_norm(x, p[pre + "input_layernorm.weight"], geo["eps"]), p, pre + "self_attn.",
                          geo["H"], cos, sin)
        x = x + mom_read(rms_norm(x, p[pre + "mom_norm.weight"], geo["eps"]), p["model.M_blocks"], p,
                         pre + "mom.", geo, stats)
        x = x + swiglu(rms_norm(x, p[pre + "post_attention_layernorm.weight"], geo["eps"]), p, pre + "mlp.")
    hN = rms_norm(x, p["model.norm.weight"], geo["eps"])
    if labels is None:
        return F.linear(hN, p["model.embed_tokens.weight"]), stats
    logits = F.linear(hN[:, :-1].reshape(-1, hN.shape[-1]), p["model.embed_tokens.weight"])
    lab = labels[:, 1:].reshape(-1)
    loss = F.cross_entropy(logits.float(), lab, reduction="sum") / (lab != -100).sum().clamp_min(1)
    return loss + geo["aux"] * aux_loss(stats, geo["nb"]), stats


def init_params(geo, seed=0):
    """The reference's initialisation at ``geo``: Linear / Embedding weights
    N(0, 0.02), norm weights 1, bank N(0, 0.02), mom_scale 0."""
    g = torch.Generator().manual_seed(seed)
    d, f, r, nb, bs = geo["d"], geo["ffn"], geo["r"], geo["nb"], geo["bs"]
    p = {"model.M_blocks": 0.02 * torch.randn(nb, bs * d, generator=g),
         "model.embed_tokens.weight": 0.02 * torch.randn(geo["vocab"], d, generator=g)}
    for i in range(geo["layers"]):
        pre = f"model.layers.{i}."
        for n in ("q", "k", "v", "o"):
            p[pre + f"self_attn.{n}_proj.weight"] = 0.02 * torch.randn(d, d, generator=g)
            p[pre + f"mom.{n}_proj.weight"] = 0.02 * torch.randn(d, d, generator=g)
        p[pre + "mlp.gate_proj.weight"] = 0.02 * torch.randn(f, d, generator=g)
        p[pre + "mlp.up_proj.weight"] = 0.02 * torch.randn(f, d, generator=g)
        p[pre + "mlp.down_proj.weight"] = 0.02 * torch.randn(d, f, generator=g)
        for n in ("input_layernorm", "post_attention_layernorm", "mom_norm"):
            p[pre + n + ".weight"] = torch.ones(d)
        p[pre + "mom.router_down.weight"] = 0.02 * torch.randn(r, d, generator=g)
        p[pre + "mom.router_up.weight"] = 0.02 * torch.randn(nb, r, generator=g)
        p[pre + "mom.mom_scale"] = torch.zeros(1)
    p["model.norm.weight"] = torch.ones(d)
    return p


# BASELINE config 3's architecture in the keys above
CONFIG3 = dict(vocab=32000, d=1024, ffn=2816, layers=20, H=16, nb=8, bs=128, top=2, r=32,
               rope_theta=500000.0, eps=1e-5, aux=0.01)


def train_step_timer(geo, B, S, threads=None, seed=0):
    """A callable running one fp32 training step (forward, backward, AdamW) of
    the decoder on a fixed (B, S) batch of token ids on the host cores."""
    if threads:
        torch.set_num_threads(threads)
    p = {k: v.requires_grad_(True) for k, v in init_params(geo, seed).items()}
    opt = torch.optim.AdamW(list(p.values()), lr=3e-4, weight_decay=0.1)
    ids = torch.randint(0, geo["vocab"], (B, S), generator=torch.Generator().manual_seed(seed + 1))

    def step():
        opt.zero_grad(set_to_none=True)
        loss, _ = forward(ids, p, geo, labels=ids)
        loss.backward()
        opt.step()
        return float(loss.detach())

    return step
