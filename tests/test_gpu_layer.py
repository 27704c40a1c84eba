"""GPU parity of the whole MoM layer (router + projections + read, forward and
backward) with ``use_kernel=True`` (mode "sm100"), under bf16 autocast as the
reference trains, against the reference's golden vectors and the oracle.
"""
import os

import numpy as np
import pytest
import torch

import golden_inputs as gi
import mom_oracle as O
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _layer(geo, scan_mode="fp64"):
    """The layer under test. scan_mode "fp64" (torch's CPU cumsum) for the
    comparisons with the reference's CPU goldens and the oracle."""
    from naylis_b200.model import MoMLayer
    layer = MoMLayer(d_model=geo["d"], n_heads=geo["H"], mem_size=geo["nb"] * geo["bs"],
                     block_size=geo["bs"], top_blocks=geo["top"], router_rank=geo["r"],
                     scan_mode=scan_mode)
    inp = gi.layer_inputs(geo, layer)
    return layer, inp


def _run(layer, inp, dout, train=True):
    dev = torch.device("cuda")
    layer = layer.to(dev)
    layer.train(train)
    layer.noise_scale = 0.0
    x = inp["x"].to(dev).requires_grad_(True)
    M = inp["M"].to(dev).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = layer(x, M)
    out.backward(dout.to(dev))
    torch.cuda.synchronize()
    res = {"out": out.detach().float().cpu().numpy(), "dx": x.grad.float().cpu().numpy(),
           "dM_blocks": M.grad.float().cpu().numpy(),
           "top_idx": layer.last_top_idx.cpu().numpy()}
    for name, p in layer.named_parameters():
        res["d_" + name.replace(".weight", "")] = p.grad.float().cpu().numpy()
    return res


def test_layer_matches_reference_golden_bf16():
    geo = gi.SMALL_BF16
    g = np.load(os.path.join(GOLDEN, "small_bf16.npz"))
    layer, inp = _layer(geo)
    assert gi.input_digest(inp) == str(g["input_sha"])
    got = _run(layer, inp, gi.upstream_grad(geo))
    assert np.array_equal(got["top_idx"].reshape(g["top_idx"].shape), g["top_idx"])
    keys = ["out", "dx", "dM_blocks", "d_router_down", "d_router_up", "d_q_proj", "d_k_proj",
            "d_v_proj", "d_o_proj"]
    errs = {k: O.scaled_err(got[k], g[k]) for k in keys}
    assert all(e < TOL for e in errs.values()), errs
    assert abs(got["d_mom_scale"][0] - g["d_mom_scale"][0]) <= TOL * abs(g["d_mom_scale"][0])


def test_layer_matches_reference_golden_fp32():
    """The whole layer in fp32 (no autocast): fp32 router head, the fp32 read,
    fp32 projections (TF32 off), against the reference's fp32 layer: output
    and every gradient within 1e-5 of the largest magnitude (the reference's
    fp32 bar), routing bitwise."""
    geo = gi.SMALL_F32
    g = np.load(os.path.join(GOLDEN, "small_f32.npz"))
    layer, inp = _layer(geo)
    assert gi.input_digest(inp) == str(g["input_sha"])
    dev = torch.device("cuda")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        layer = layer.to(dev).train()
        layer.noise_scale = 0.0
        x = inp["x"].to(dev).requires_grad_(True)
        M = inp["M"].to(dev).requires_grad_(True)
        out = layer(x, M)
        out.backward(gi.upstream_grad(geo).to(dev))
        torch.cuda.synchronize()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert out.dtype == torch.float32
    assert np.array_equal(layer.last_top_idx.cpu().numpy().reshape(g["top_idx"].shape), g["top_idx"])
    got = {"out": out.detach().cpu().numpy(), "dx": x.grad.cpu().numpy(), "dM_blocks": M.grad.cpu().numpy()}
    for name, p in layer.named_parameters():
        got["d_" + name.replace(".weight", "")] = p.grad.cpu().numpy()
    keys = ["out", "dx", "dM_blocks", "d_router_down", "d_router_up", "d_q_proj", "d_k_proj", "d_v_proj",
            "d_o_proj"]
    errs = {k: O.scaled_err(got[k], g[k]) for k in keys}
    assert all(e < 1e-5 for e in errs.values()), errs
    assert abs(got["d_mom_scale"][0] - g["d_mom_scale"][0]) <= 1e-5 * abs(g["d_mom_scale"][0])


def test_layer_config2_full_size_matches_reference_golden(monkeypatch):
    """BASELINE config 2 at the benchmarked size (B=8 x S=2048, d=1024, 16x64
    heads, bank 8x128, rank 32, top-2) against what the reference's own
    MoMLayer computed under CPU bf16 autocast (tests/golden/cfg2_layer.npz).

    Routing: bitwise on every token whose top three bf16 logits are distinct.
    On the ~1 % of tokens with two equal values among them, torch.topk's
    choice is implementation-defined (the CPU picks or lists the higher block
    id first about a quarter of the time); there the kernel must follow its
    documented rule, torch's CUDA order, on the golden logits.

    Output and gradients: to compare them on the same routing, the layer is run
    again with the reference's choice at the tied tokens imposed through the
    router's noise input (the one Gumbel noise uses): +8 bf16 ulps of the tied
    value on the reference's first block and +4 on its second, at the tied
    tokens only (more than the 1-ulp differences that the kernel's and the
    CPU's accumulation orders leave in the bf16 logits; the gates move by
    ~1e-4). Then every token routes as the reference did, and seeded
    subsamples of the output and of every gradient are within 2e-2 of the full
    tensor's largest magnitude."""
    from naylis_b200 import mom_kernels as mk
    geo = gi.CFG2
    g = np.load(os.path.join(GOLDEN, "cfg2_layer.npz"))
    layer, inp = _layer(geo)
    assert gi.input_digest(inp) == str(g["input_sha"])
    dev = torch.device("cuda")
    layer = layer.to(dev)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        _, idx, _ = mk.mom_route(inp["x"].to(dev), layer.router_down.weight, layer.router_up.weight,
                                 geo["top"], None, scan_mode="fp64")
    ours = idx.reshape(-1, geo["top"]).cpu().numpy()
    ref = g["top_idx"].reshape(-1, geo["top"]).astype(np.int64)
    tie = np.zeros(ours.shape[0], dtype=bool)
    tie[g["tie_tokens"]] = True
    differ = np.any(ours != ref, axis=-1)
    assert not (differ & ~tie).any(), \
        f"{int((differ & ~tie).sum())} non-tied tokens route differently; margins " \
        f"{g['margin'][differ & ~tie][:8]}"
    cuda_rule = O.topk_cuda_order(g["tie_logits"], geo["top"])[0]
    assert np.array_equal(ours[g["tie_tokens"]], cuda_rule)

    nudge = torch.zeros(geo["B"] * geo["S"], geo["nb"])
    rows = torch.from_numpy(g["tie_tokens"])
    golden_idx = torch.from_numpy(ref[g["tie_tokens"]])
    # 8 and 4 bf16 ulps of the tied value: more than the 1-ulp differences that
    # the kernel's and the CPU's accumulation orders leave in the bf16 logits
    kth = torch.from_numpy(np.abs(np.sort(g["tie_logits"], axis=1)[:, -geo["top"]]).astype(np.float32))
    nudge[rows, golden_idx[:, 0]] = kth * 2.0 ** -5
    nudge[rows, golden_idx[:, 1]] = kth * 2.0 ** -6
    nudge = nudge.view(geo["B"], geo["S"], geo["nb"]).to(dev)
    monkeypatch.setattr(mk, "gumbel_noise", lambda shape, device, scale: nudge)
    layer.noise_scale = 1.0
    layer.train()
    x = inp["x"].to(dev).requires_grad_(True)
    M = inp["M"].to(dev).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = layer(x, M)
    out.backward(gi.upstream_grad(geo).to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(layer.last_top_idx.cpu().numpy(), ref)
    got = {"out": out.detach(), "dx": x.grad, "dM_blocks": M.grad}
    for name, p in layer.named_parameters():
        got["d_" + name.replace(".weight", "")] = p.grad
    flat = {k: v.float().reshape(-1).cpu().numpy() for k, v in got.items()}
    errs = {}
    for k in ("out", "dx", "dM_blocks", "d_router_down", "d_router_up", "d_q_proj", "d_k_proj",
              "d_v_proj", "d_o_proj"):
        errs[k] = float(np.abs(flat[k][g[k + "_idx"]] - g[k]).max() / g[k + "_absmax"])
    assert all(e < TOL for e in errs.values()), errs
    assert abs(flat["d_mom_scale"][0] - g["d_mom_scale"][0]) <= TOL * abs(g["d_mom_scale"][0])


def test_layer_config2_geometry_matches_oracle():
    # config-2 geometry (d=1024, 16x64 heads, bank 8x128, rank 32, top-2) on
    # one 2048-token sequence, so that the fp64 oracle stays within seconds
    geo = dict(B=1, S=2048, d=1024, H=16, nb=8, bs=128, top=2, r=32, seed=0, x_std=1.0,
               m_std=0.02, w_std=0.02, mom_scale=1.0)
    layer, inp = _layer(geo)
    dout = gi.upstream_grad(geo)
    got = _run(layer, inp, dout)
    P = gi.oracle_params(inp, geo)
    f = O.layer_forward(inp["x"].numpy(), P, geo["H"], geo["nb"], geo["bs"], geo["top"], "bf16")
    mism = np.any(got["top_idx"].reshape(f["router"]["top_idx"].shape) != f["router"]["top_idx"], -1)
    assert not mism.any(), f"{int(mism.sum())} routing mismatches"
    b = O.layer_backward(f, inp["x"].numpy(), P, dout.numpy(), geo["H"], geo["nb"], geo["bs"])
    pairs = [("out", f["out"]), ("dx", b["dx"]), ("dM_blocks", b["dM_blocks"]),
             ("d_router_down", b["dw_down"]), ("d_router_up", b["dw_up"]), ("d_q_proj", b["dwq"]),
             ("d_k_proj", b["dwk"]), ("d_v_proj", b["dwv"]), ("d_o_proj", b["dwo"])]
    errs = {k: O.scaled_err(got[k], ref) for k, ref in pairs}
    assert all(e < TOL for e in errs.values()), errs


def test_layer_top4_of_32_geometry_matches_oracle():
    # d=2048, 16x128 heads, bank 32x128, rank 64, top-4: 35,960 block sets, so
    # the read takes the block-split path; one 512-token sequence for the oracle
    geo = dict(B=1, S=512, d=2048, H=16, nb=32, bs=128, top=4, r=64, seed=3, x_std=1.0,
               m_std=0.02, w_std=0.02, mom_scale=1.0)
    layer, inp = _layer(geo)
    dout = gi.upstream_grad(geo)
    got = _run(layer, inp, dout)
    P = gi.oracle_params(inp, geo)
    f = O.layer_forward(inp["x"].numpy(), P, geo["H"], geo["nb"], geo["bs"], geo["top"], "bf16")
    mism = np.any(got["top_idx"].reshape(f["router"]["top_idx"].shape) != f["router"]["top_idx"], -1)
    assert not mism.any(), f"{int(mism.sum())} routing mismatches"
    b = O.layer_backward(f, inp["x"].numpy(), P, dout.numpy(), geo["H"], geo["nb"], geo["bs"])
    pairs = [("out", f["out"]), ("dx", b["dx"]), ("dM_blocks", b["dM_blocks"]),
             ("d_router_down", b["dw_down"]), ("d_router_up", b["dw_up"]), ("d_q_proj", b["dwq"]),
             ("d_k_proj", b["dwk"]), ("d_v_proj", b["dwv"]), ("d_o_proj", b["dwo"])]
    errs = {k: O.scaled_err(got[k], ref) for k, ref in pairs}
    assert all(e < TOL for e in errs.values()), errs


def test_layer_kernel_path_is_causal():
    geo = dict(B=2, S=512, d=256, H=4, nb=8, bs=64, top=2, r=32, seed=3, x_std=1.0,
               m_std=1.0, w_std=0.06, mom_scale=1.0)
    layer, inp = _layer(geo)
    dev = torch.device("cuda")
    layer = layer.to(dev).eval()
    x = inp["x"].to(dev)
    M = inp["M"].to(dev)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        a = layer(x, M)
        x2 = x.clone()
        x2[:, 301:] += 1.0
        b = layer(x2, M)
    assert torch.equal(a[:, :301], b[:, :301])


def test_resolve_mode_contract_on_gpu():
    from naylis_b200 import mom_kernels as mk
    assert mk.resolve_mode("cuda", torch.bfloat16, head_dim=64) == "sm100"
    assert mk.resolve_mode(torch.device("cuda", 0), torch.bfloat16, head_dim=128) == "sm100"
    assert mk.resolve_mode("cuda", torch.float32, head_dim=64) == "sm100"   # the fp32 read
    with pytest.raises(RuntimeError):
        mk.resolve_mode("cuda", torch.float16, head_dim=64)
    # the reference resolves with x.dtype (model.py:164-165): fp32 inside a bf16
    # autocast region, where the q projection, and so the read, runs in bf16
    with torch.autocast("cuda", dtype=torch.bfloat16):
        assert mk.resolve_mode("cuda", torch.float32, head_dim=64) == "sm100"
    with pytest.raises(RuntimeError):
        mk.resolve_mode("cuda", torch.bfloat16, head_dim=96)
    assert mk.preflight("cuda") is None


@pytest.mark.parametrize("g_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("offset", [0, 1])
def test_fused_output_scale_matches_torch(g_dtype, offset):
    """mom_scale (model.py:239 fused): fp32 y = s * o from bf16 o; backward
    d_o = s * g in bf16 and d_s = sum(g * o), against torch's own mul. offset 1
    starts o and g one element into their storage (not vector-aligned: the
    kernels' scalar path)."""
    from naylis_b200 import mom_kernels as mk
    torch.manual_seed(0)
    dev = torch.device("cuda")
    n = 3 * 257 * 64
    o = torch.randn(n + offset, device=dev).to(torch.bfloat16)[offset:].view(3, 257, 64).requires_grad_(True)
    s = torch.tensor([0.37], device=dev, requires_grad=True)
    g = torch.randn(n + offset, device=dev).to(g_dtype)[offset:].view(3, 257, 64)
    y = mk.mom_scale(o, s)
    y.backward(g)
    o2 = o.detach().clone().requires_grad_(True)
    s2 = s.detach().clone().requires_grad_(True)
    y2 = s2 * o2
    y2.backward(g.float())
    assert y.dtype == torch.float32 and torch.equal(y, y2)
    assert torch.equal(o.grad, o2.grad)
    assert abs(float(s.grad) - float(s2.grad)) <= 1e-5 * abs(float(s2.grad))


def test_layer_grad_checkpoint_recompute_matches():
    """mom_grad_ckpt (model.py:233-238): the read runs under
    torch.utils.checkpoint, so its forward kernels run a second time during the
    backward. The forward kernels are deterministic: output and routing equal
    the run without checkpointing bitwise; the gradients, which sum fp32
    partials by atomics in an order that varies between runs, agree to a
    scaled 1e-4. Config-2 geometry at 2 x 512 tokens, so the tensor-core read
    kernels are the ones recomputed."""
    geo = dict(gi.SMALL_BF16)
    geo.update(B=2, S=512, d=1024, H=16, nb=8, bs=128, top=2, r=32, seed=77)
    res = []
    for ckpt in (False, True):
        layer, inp = _layer(geo)
        layer.mom_grad_ckpt = ckpt
        res.append(_run(layer, inp, gi.upstream_grad(geo)))
    for key in ("out", "top_idx"):
        assert np.array_equal(res[0][key], res[1][key]), key
    errs = {k: O.scaled_err(res[1][k], res[0][k]) for k in res[0] if k not in ("out", "top_idx")}
    assert all(e < 1e-4 for e in errs.values()), errs

