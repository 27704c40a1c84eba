#!/usr/bin/env python3
"""Generate the golden vectors that pin the oracle (and the CUDA path) to the
reference implementation of the Naylis MoM hot path.

Run HERE, where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

It imports the reference's own ``model.MoMLayer`` and ``mom_kernels.reference``
(no code is copied) and runs them on seeded inputs. Inputs are NOT stored:
``golden_inputs.py`` regenerates them bit-identically from torch's CPU RNG, and
their SHA-256 digests are stored so a drift in the generator is detected.
Outputs are stored in full where small, and as SHA-256 + a seeded subsample
where large (config 1).

Cases:
  cfg1_fwd        BASELINE config 1: fp32 layer forward, B=1 S=256 d=1024,
                  16x64 heads, bank 8x128, rank 32, top-2, mom_scale=1, eval.
  small_f32       layer forward+backward, fp32, the reference test-suite
                  geometry (tests/test_parity.py:74-77), upstream grad N(0,1).
  small_bf16      layer forward+backward under CPU bf16 autocast.
  read_f32/bf16   read only (build_gate_bias + mom_attention_reference), with
                  gradients w.r.t. q, k, v and the gates.
  scan            prefix mean h at (2, 1024, 64), fp32 and bf16 input: SHA-256.
  decoder_small   the reference's NaylisLlamaForCausalLM (2 layers, d=256,
                  4x64 heads, SwiGLU 512, vocab 512, bank 8x128, top-2) under
                  CPU bf16 autocast in training mode, Gumbel off: loss,
                  gradient subsamples, logits subsample, every layer's routing.
  decoder_small_f32  the same in fp32 (no autocast): pins oracle/decoder_oracle.py.
  cfg2_layer      BASELINE config 2 at full size (B=8, S=2048): layer
                  forward+backward under CPU bf16 autocast, Gumbel off. Stored:
                  every token's top-2 ids, every token's logit margin between
                  its 2nd and 3rd block, the tokens with equal values among
                  their top 3 logits with those logits, and seeded
                  subsamples of the output and of every gradient.
"""
import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import golden_inputs as gi  # noqa: E402


def sha(t) -> str:
    import torch
    a = t.detach().contiguous()
    if a.dtype == torch.bfloat16:
        a = a.float()
    return hashlib.sha256(a.cpu().numpy().tobytes()).hexdigest()


def to_np(t):
    import torch
    t = t.detach()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.cpu().numpy()


def build_layer(model_mod, geo):
    return model_mod.MoMLayer(
        d_model=geo["d"], n_heads=geo["H"], mem_size=geo["nb"] * geo["bs"],
        block_size=geo["bs"], top_blocks=geo["top"], router_rank=geo["r"])


def run_cfg1(model_mod, reference):
    import torch
    geo = gi.CFG1
    layer = build_layer(model_mod, geo)
    inp = gi.layer_inputs(geo, layer)
    layer.eval()
    with torch.no_grad():
        out, probs, top_idx, gates = reference.mom_full_reference(inp["x"], layer, inp["M"])
        out_layer = layer(inp["x"], inp["M"])
        logits = layer._router_logits(inp["x"])
        h = reference.prefix_mean_reference(inp["x"])
    assert torch.equal(out, out_layer)
    rng = np.random.default_rng(1234)
    sub = rng.choice(out.numel(), size=4096, replace=False)
    return dict(
        input_sha=np.array(gi.input_digest(inp)),
        out_sha=np.array(sha(out)), h_sha=np.array(sha(h)),
        out_sub_idx=sub.astype(np.int64), out_sub=to_np(out).reshape(-1)[sub],
        h_sub=to_np(h).reshape(-1)[sub],
        probs=to_np(probs).reshape(geo["B"], geo["S"], -1),
        top_idx=to_np(top_idx).astype(np.int64),
        gates=to_np(gates), logits=to_np(logits),
    )


def run_layer_small(model_mod, autocast: bool):
    import torch
    geo = gi.SMALL_BF16 if autocast else gi.SMALL_F32
    layer = build_layer(model_mod, geo)
    inp = gi.layer_inputs(geo, layer)
    layer.train()
    layer.noise_scale = 0.0          # deterministic routing, no Gumbel draw
    x = inp["x"].clone().requires_grad_(True)
    M = inp["M"].clone().requires_grad_(True)
    dout = gi.upstream_grad(geo)
    with torch.autocast("cpu", dtype=torch.bfloat16, enabled=autocast):
        out = layer(x, M)
    out.backward(dout)
    res = dict(input_sha=np.array(gi.input_digest(inp)), out=to_np(out),
               probs=to_np(layer.last_router_probs).reshape(geo["B"], geo["S"], -1),
               top_idx=to_np(layer.last_top_idx).reshape(geo["B"], geo["S"], -1).astype(np.int64),
               dx=to_np(x.grad), dM_blocks=to_np(M.grad))
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16, enabled=autocast):
        res["logits"] = to_np(layer._router_logits(inp["x"]))
    for name, p in layer.named_parameters():
        res["d_" + name.replace(".weight", "")] = to_np(p.grad)
    return res


def run_cfg2(model_mod):
    import torch
    geo = gi.CFG2
    layer = build_layer(model_mod, geo)
    inp = gi.layer_inputs(geo, layer)
    layer.train()
    layer.noise_scale = 0.0
    x = inp["x"].clone().requires_grad_(True)
    M = inp["M"].clone().requires_grad_(True)
    dout = gi.upstream_grad(geo)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        out = layer(x, M)
    out.backward(dout)
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        logits = layer._router_logits(inp["x"])
    top_idx = layer.last_top_idx.reshape(geo["B"], geo["S"], -1)
    srt = torch.sort(logits, dim=-1, descending=True).values
    margin = (srt[..., geo["top"] - 1] - srt[..., geo["top"]]).reshape(-1)
    rng = np.random.default_rng(4321)
    res = dict(input_sha=np.array(gi.input_digest(inp)),
               top_idx=to_np(top_idx).astype(np.uint8), margin=to_np(margin))
    # tokens with two equal values anywhere among their top (k + 1) logits
    top3 = srt[..., :geo["top"] + 1].reshape(-1, geo["top"] + 1)
    ties = torch.nonzero((top3[:, 1:] == top3[:, :-1]).any(-1)).reshape(-1)
    res["tie_tokens"] = to_np(ties).astype(np.int64)
    res["tie_logits"] = to_np(logits.reshape(-1, geo["nb"])[ties])
    tensors = dict(out=out, dx=x.grad, dM_blocks=M.grad)
    for name, p in layer.named_parameters():
        tensors["d_" + name.replace(".weight", "")] = p.grad
    for name, t in tensors.items():
        flat = to_np(t).reshape(-1)
        sub = np.sort(rng.choice(flat.size, size=min(flat.size, 8192), replace=False))
        res[name + "_idx"] = sub.astype(np.int64)
        res[name] = flat[sub]
        res[name + "_absmax"] = np.array(np.abs(flat).max())
    return res


def run_decoder(model_mod, autocast=True):
    """The reference's NaylisLlamaForCausalLM (transformers Llama trunk, MoM
    layers, tied head, aux loss) at golden_inputs.DECODER under CPU bf16
    autocast, training mode without Gumbel noise: the loss and its gradient,
    the logits, and every layer's routing."""
    import torch
    from transformers import LlamaConfig
    geo = gi.DECODER
    cfg = LlamaConfig(vocab_size=geo["vocab"], hidden_size=geo["d"], intermediate_size=geo["ffn"],
                      num_hidden_layers=geo["layers"], num_attention_heads=geo["H"],
                      num_key_value_heads=geo["H"], max_position_embeddings=geo["S"],
                      rms_norm_eps=geo["eps"], rope_theta=geo["rope_theta"], attention_bias=False,
                      tie_word_embeddings=True, attn_implementation="sdpa", use_cache=False)
    model = model_mod.NaylisLlamaForCausalLM(cfg, mem_size=geo["nb"] * geo["bs"], mom_block_size=geo["bs"],
                                             mom_top_blocks=geo["top"], mom_router_rank=geo["r"],
                                             mom_aux_weight=geo["aux"])
    sd = gi.decoder_state(geo)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
    moms = [m for m in model.modules() if isinstance(m, model_mod.MoMLayer)]
    for m in moms:
        m.noise_scale = 0.0
    model.train()
    ids = gi.decoder_tokens(geo)
    with torch.autocast("cpu", dtype=torch.bfloat16, enabled=autocast):
        out = model(input_ids=ids, labels=ids)
    routing = np.stack([to_np(m.last_top_idx) for m in moms]).astype(np.int64) if moms[0].last_top_idx \
        is not None else None
    out.loss.backward()
    res = dict(state_sha=np.array(gi.state_digest(sd)), loss=np.array(float(out.loss)))
    rng = np.random.default_rng(77)
    for name, p in model.named_parameters():
        flat = to_np(p.grad).reshape(-1)
        sub = np.sort(rng.choice(flat.size, size=min(flat.size, 2048), replace=False))
        res["g_" + name + "_idx"] = sub.astype(np.int64)
        res["g_" + name] = flat[sub]
        res["g_" + name + "_absmax"] = np.array(np.abs(flat).max())
    model.zero_grad(set_to_none=True)
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16, enabled=autocast):
        logits = model(input_ids=ids).logits
    res["routing"] = np.stack([to_np(m.last_top_idx) for m in moms]).astype(np.int8)
    flat = to_np(logits).reshape(-1)
    sub = np.sort(rng.choice(flat.size, size=8192, replace=False))
    res["logits_idx"] = sub.astype(np.int64)
    res["logits"] = flat[sub]
    res["logits_absmax"] = np.array(np.abs(flat).max())
    if routing is not None:
        assert np.array_equal(routing, res["routing"])
    return res


def run_read(reference, dtype_name: str):
    import torch
    geo = gi.READ
    q, k, v, top, g, dout = gi.read_inputs(geo, dtype_name)
    for t in (q, k, v, g):
        t.requires_grad_(True)
    bias = reference.build_gate_bias(top, g, geo["nb"], geo["bs"], q.dtype)
    out = reference.mom_attention_reference(q, k, v, bias)
    out.backward(dout)
    return dict(out=to_np(out), dq=to_np(q.grad), dk=to_np(k.grad), dv=to_np(v.grad),
                dgates=to_np(g.grad), top_idx=to_np(top).astype(np.int64))


def run_scan(reference):
    import torch
    res = {}
    for name in ("f32", "bf16"):
        x = gi.scan_input(name)
        h = reference.prefix_mean_reference(x)
        res[f"h_sha_{name}"] = np.array(sha(h))
        res[f"x_sha_{name}"] = np.array(sha(x))
        res[f"h_first_row_{name}"] = to_np(h[:, :4])
        assert h.dtype == torch.float32
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--cases", default="", help="comma-separated subset of the cases (default: all)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    import model as model_mod
    from mom_kernels import reference

    cases = {
        "cfg1_fwd": lambda: run_cfg1(model_mod, reference),
        "small_f32": lambda: run_layer_small(model_mod, autocast=False),
        "small_bf16": lambda: run_layer_small(model_mod, autocast=True),
        "read_f32": lambda: run_read(reference, "f32"),
        "read_bf16": lambda: run_read(reference, "bf16"),
        "scan": lambda: run_scan(reference),
        "cfg2_layer": lambda: run_cfg2(model_mod),
        "decoder_small": lambda: run_decoder(model_mod),
        "decoder_small_f32": lambda: run_decoder(model_mod, autocast=False),
    }
    ap_cases = [c for c in args.cases.split(",") if c] if args.cases else list(cases)
    for name, fn in ((n, cases[n]) for n in ap_cases):
        res = fn()
        path = os.path.join(args.out, f"{name}.npz")
        np.savez_compressed(path, **res)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


if __name__ == "__main__":
    main()
