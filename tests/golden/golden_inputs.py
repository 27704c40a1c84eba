"""Seeded input generators shared by the golden-vector script and the tests.

Everything here draws from torch's CPU generator, which is bit-reproducible on
any machine with the same torch build, so the golden files store only input
digests, never the inputs. The layer helpers fill any module that has the
MoMLayer attribute names (``router_down``, ``router_up``, ``q_proj``,
``k_proj``, ``v_proj``, ``o_proj``, ``mom_scale``) — the reference's
``model.MoMLayer`` when generating goldens, this package's mirror in the tests.

Canonical draw order after ``torch.manual_seed(seed)``: x, M_blocks,
router_down, router_up, q_proj, k_proj, v_proj, o_proj.
"""
import hashlib

import numpy as np

# fp32 layer forward.
CFG1 = dict(B=1, S=256, d=1024, H=16, nb=8, bs=128, top=2, r=32,
            seed=0, x_std=1.0, m_std=0.02, w_std=0.02, mom_scale=1.0)
# The reference test-suite geometry (tests/test_parity.py:74-77), fp32.
SMALL_F32 = dict(B=2, S=64, d=32, H=2, nb=4, bs=16, top=2, r=8,
                 seed=7, x_std=1.0, m_std=1.0, w_std=0.18, mom_scale=0.5)
# A head_dim-64 geometry with a ragged sequence length, bf16 autocast.
SMALL_BF16 = dict(B=2, S=96, d=128, H=2, nb=4, bs=64, top=2, r=8,
                  seed=21, x_std=1.0, m_std=1.0, w_std=0.09, mom_scale=0.5)
# BASELINE config 2 at full size (B=8 x S=2048): the benchmarked layer.
CFG2 = dict(B=8, S=2048, d=1024, H=16, nb=8, bs=128, top=2, r=32,
            seed=2, x_std=1.0, m_std=0.02, w_std=0.02, mom_scale=1.0)
# Read-only cases (q, k, v, routing given directly).
READ = dict(B=2, S=80, H=2, hd=64, nb=4, bs=64, top=2, seed=5)


def _torch():
    import torch
    return torch


def layer_inputs(geo: dict, layer=None) -> dict:
    """x, M_blocks and (when ``layer`` is given) its weights, drawn in order."""
    torch = _torch()
    torch.manual_seed(geo["seed"])
    B, S, d, nb, bs = geo["B"], geo["S"], geo["d"], geo["nb"], geo["bs"]
    x = torch.randn(B, S, d) * geo["x_std"]
    M = torch.empty(nb, bs * d).normal_(0.0, geo["m_std"])
    w = {}
    shapes = dict(router_down=(geo["r"], d), router_up=(nb, geo["r"]),
                  q_proj=(d, d), k_proj=(d, d), v_proj=(d, d), o_proj=(d, d))
    for name, shp in shapes.items():
        w[name] = torch.empty(*shp).normal_(0.0, geo["w_std"])
    if layer is not None:
        with torch.no_grad():
            for name, t in w.items():
                getattr(layer, name).weight.copy_(t)
            layer.mom_scale.fill_(geo["mom_scale"])
    return dict(x=x, M=M, w=w)


def upstream_grad(geo: dict):
    torch = _torch()
    g = torch.Generator().manual_seed(geo["seed"] + 1000)
    return torch.randn(geo["B"], geo["S"], geo["d"], generator=g)


def oracle_params(inp: dict, geo: dict) -> dict:
    """The numpy parameter dict the oracle's layer functions take."""
    w = {k: v.numpy() for k, v in inp["w"].items()}
    return dict(w_down=w["router_down"], w_up=w["router_up"], wq=w["q_proj"],
                wk=w["k_proj"], wv=w["v_proj"], wo=w["o_proj"],
                mom_scale=np.float32(geo["mom_scale"]), M_blocks=inp["M"].numpy())


def input_digest(inp: dict) -> str:
    h = hashlib.sha256()
    for t in [inp["x"], inp["M"]] + [inp["w"][k] for k in sorted(inp["w"])]:
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def read_inputs(geo: dict, dtype_name: str):
    """q (B,S,H,hd), shared k/v (L, H*hd), top_idx, gates (fp32), upstream grad."""
    torch = _torch()
    torch.manual_seed(geo["seed"])
    B, S, H, hd, nb, bs, top = (geo[k] for k in ("B", "S", "H", "hd", "nb", "bs", "top"))
    L, D = nb * bs, H * hd
    q = torch.randn(B, S, H, hd) * 0.7
    k = torch.randn(L, D) * 0.4
    v = torch.randn(L, D) * 0.4
    g = torch.softmax(torch.randn(B, S, top), -1)
    # distinct blocks per token, as topk produces
    top_idx = torch.argsort(torch.rand(B, S, nb), dim=-1)[..., :top]
    dout = torch.randn(B, S, H, hd)
    if dtype_name == "bf16":
        q, k, v, dout = (t.to(torch.bfloat16) for t in (q, k, v, dout))
    return q, k, v, top_idx, g, dout


def scan_input(dtype_name: str):
    torch = _torch()
    torch.manual_seed(99)
    x = torch.randn(2, 1024, 64)
    if dtype_name == "bf16":
        x = x.to(torch.bfloat16)
    return x


# A small Naylis decoder (BASELINE config 3's architecture at reduced size):
# 2 layers, d=256, 4 heads of 64, SwiGLU 512, vocab 512, bank 8 x 128 slots,
# router rank 32, top-2, RoPE theta 5e5, RMSNorm eps 1e-5, tied LM head.
DECODER = dict(B=2, S=256, vocab=512, d=256, ffn=512, layers=2, H=4, nb=8, bs=128, top=2, r=32,
               rope_theta=500000.0, eps=1e-5, aux=0.01, seed=31)


def decoder_param_shapes(geo: dict) -> list:
    """(name, shape) of every parameter of the reference's NaylisLlamaForCausalLM
    (model.py:350-470 with transformers' Llama modules), lm_head tied."""
    d, f, r, nb, bs = geo["d"], geo["ffn"], geo["r"], geo["nb"], geo["bs"]
    out = [("model.M_blocks", (nb, bs * d)), ("model.embed_tokens.weight", (geo["vocab"], d))]
    for i in range(geo["layers"]):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj.weight", (d, d)), (p + "self_attn.k_proj.weight", (d, d)),
                (p + "self_attn.v_proj.weight", (d, d)), (p + "self_attn.o_proj.weight", (d, d)),
                (p + "mlp.gate_proj.weight", (f, d)), (p + "mlp.up_proj.weight", (f, d)),
                (p + "mlp.down_proj.weight", (d, f)), (p + "input_layernorm.weight", (d,)),
                (p + "post_attention_layernorm.weight", (d,)), (p + "mom_norm.weight", (d,)),
                (p + "mom.mom_scale", (1,)), (p + "mom.router_down.weight", (r, d)),
                (p + "mom.router_up.weight", (nb, r)), (p + "mom.q_proj.weight", (d, d)),
                (p + "mom.k_proj.weight", (d, d)), (p + "mom.v_proj.weight", (d, d)),
                (p + "mom.o_proj.weight", (d, d))]
    return out + [("model.norm.weight", (d,))]


def decoder_state(geo: dict) -> dict:
    """A deterministic parameter set for the decoder, in the reference's names:
    matrices and the bank N(0, 0.02), norm weights 1 + N(0, 0.1), mom_scale 1
    (so the memory read reaches the output), plus lm_head.weight tied to the
    embedding. Drawn in decoder_param_shapes order from one CPU generator."""
    torch = _torch()
    g = torch.Generator().manual_seed(geo["seed"])
    sd = {}
    for name, shape in decoder_param_shapes(geo):
        if name.endswith("mom_scale"):
            sd[name] = torch.ones(shape)
        elif len(shape) == 1:
            sd[name] = 1.0 + 0.1 * torch.randn(shape, generator=g)
        else:
            sd[name] = 0.02 * torch.randn(shape, generator=g)
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


def decoder_tokens(geo: dict):
    torch = _torch()
    g = torch.Generator().manual_seed(geo["seed"] + 1)
    return torch.randint(0, geo["vocab"], (geo["B"], geo["S"]), generator=g)


def state_digest(sd: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].contiguous().numpy().tobytes())
    return h.hexdigest()
