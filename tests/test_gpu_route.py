"""GPU parity of the fused causal router through the C ABI.

* prefix mean: bitwise against the reference's golden digests (fp64 mode,
  torch CPU cumsum semantics) and against torch.cumsum on CUDA (fp32 mode);
* top-k indices: bitwise against the oracle and the reference golden vectors
  (a token may differ only where the oracle's k-th / (k+1)-th logit gap is
  within a rounding of zero — reported, and required to be absent here);
* probabilities and gates: scaled error < 1e-5 (fp32) / 2e-2 (bf16);
* backward: dx, dW_down, dW_up against the oracle's fp64 adjoint.
"""
import hashlib
import os

import numpy as np
import pytest
import torch

import golden_inputs as gi
import mom_oracle as O
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _prefix_mean_gpu(x, mode, out_dtype=torch.float32):
    from naylis_b200 import _lib
    xd = x.cuda().contiguous()
    B, S, d = xd.shape
    out = torch.empty(B, S, d, dtype=out_dtype, device="cuda")
    code = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}
    _lib.call("mom_prefix_mean", xd.data_ptr(), code[xd.dtype], B, S, d, out.data_ptr(),
              code[out_dtype], _lib.SCAN_MODES[mode], torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("name", ["f32", "bf16"])
def test_prefix_mean_fp64_mode_bitwise_vs_reference(name):
    g = np.load(os.path.join(GOLDEN, "scan.npz"))
    x = gi.scan_input(name)
    h = _prefix_mean_gpu(x, "fp64")
    assert hashlib.sha256(h.numpy().tobytes()).hexdigest() == str(g[f"h_sha_{name}"])


@pytest.mark.parametrize("shape", [(2, 2048, 1024), (3, 1000, 104), (1, 1, 40), (1, 65, 24), (2, 4097, 64)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prefix_mean_fp32_mode_bitwise_vs_torch_cuda(dtype, shape):
    """fp32 mode = torch's CUDA cumsum divided by t+1, bit for bit; ragged
    shapes cover partial column groups and partial row stages."""
    torch.manual_seed(0)
    x = (torch.randn(*shape) * torch.exp(torch.randn(*shape) * 3)).to(dtype)
    h = _prefix_mean_gpu(x, "fp32")
    xc = x.cuda()
    ref = torch.cumsum(xc.float(), dim=1) / torch.arange(1, shape[1] + 1, device="cuda",
                                                          dtype=torch.float32).view(1, -1, 1)
    assert torch.equal(h, ref.cpu())
    hb = _prefix_mean_gpu(x, "fp32", torch.bfloat16)
    assert torch.equal(hb, ref.cpu().to(torch.bfloat16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prefix_mean_fp64_mode_dynamic_range_fallback(dtype):
    """Columns whose dynamic range defeats the exactness certificate of the
    parallel scan (a 1e-30 next to O(1) values, or 1e30 values) must still be
    bit-identical to the sequential fp64 cumsum (they take the sequential walk)."""
    torch.manual_seed(2)
    x = torch.randn(2, 3000, 96)
    x[0, 17, 5] = 1e-30
    x[1, 2999, 40] = -3e-38
    x[1, :, 77] *= 1e30
    x = x.to(dtype)
    h = _prefix_mean_gpu(x, "fp64")
    ref = O.prefix_mean(x.float().numpy(), "fp64")
    assert np.array_equal(h.numpy(), ref)


def test_prefix_mean_fp64_mode_bf16_special_values():
    """bf16 inputs enter the fp64 sums through their bit patterns: zeros (both
    signs), subnormals (below 2^-126, converted), the smallest and largest
    normals around them and sparse columns must give the sequential fp64 cumsum
    bit for bit, whichever path (parallel or fallback) a column takes."""
    torch.manual_seed(5)
    x = torch.randn(2, 700, 64)
    x[:, ::3, 0] = 0.0
    x[:, 1::3, 1] = -0.0
    x[:, :, 2] = 0.0
    x[0, 10, 3] = 2.0 ** -130            # bf16 subnormal
    x[1, 20:40, 4] = -(2.0 ** -133)      # the smallest bf16 subnormal
    x[0, :, 5] = 2.0 ** -126             # smallest normal, all rows
    x[1, :, 6] = torch.randn(700) * 1e-20
    x[0, 300:, 7] = 0.0                  # a column that turns to zeros
    x[:, :50, 8] = -0.0                  # a prefix of negative zeros (torch's CPU cumsum gives +0.0)
    x[1, :, 9] = -0.0
    x = x.to(torch.bfloat16)
    h = _prefix_mean_gpu(x, "fp64")
    ref = O.prefix_mean(x.float().numpy(), "fp64")
    assert np.array_equal(h.numpy().view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_prefix_mean_causality_and_bf16_output():
    torch.manual_seed(1)
    x = torch.randn(3, 700, 64)
    h = _prefix_mean_gpu(x, "fp64")
    x2 = x.clone()
    x2[:, 400:] += 3.0
    h2 = _prefix_mean_gpu(x2, "fp64")
    assert torch.equal(h[:, :400], h2[:, :400])
    hb = _prefix_mean_gpu(x, "fp64", torch.bfloat16)
    assert torch.equal(hb, h.to(torch.bfloat16))


def _route_gpu(x, w_down, w_up, top, compute_dtype, noise=None, scan_mode="fp64", grad=None):
    from naylis_b200 import mom_kernels as mk
    xd = x.cuda().requires_grad_(grad is not None)
    wd = w_down.cuda().requires_grad_(grad is not None)
    wu = w_up.cuda().requires_grad_(grad is not None)
    nz = None if noise is None else noise.cuda()
    probs, idx, gates = mk.mom_route(xd, wd, wu, top, nz, compute_dtype=compute_dtype,
                                     scan_mode=scan_mode)
    res = {"probs": probs.detach().cpu().numpy(), "top_idx": idx.cpu().numpy(),
           "gates": gates.detach().cpu().numpy()}
    if grad is not None:
        dgates, dprobs = (t.cuda() for t in grad)
        torch.autograd.backward([gates, probs], [dgates, dprobs])
        res.update(dx=xd.grad.float().cpu().numpy(), dw_down=wd.grad.cpu().numpy(),
                   dw_up=wu.grad.cpu().numpy())
    return res


def _assert_indices(got_idx, rt, top, tag):
    mism = np.any(got_idx != rt["top_idx"], axis=-1)
    if mism.any():
        margin = O.topk_margin(rt["noisy"], top)[mism]
        raise AssertionError(f"{tag}: {int(mism.sum())} tokens differ; oracle top-k margins there: "
                             f"{margin[:10]}")


def test_router_cfg1_matches_reference_golden():
    geo = gi.CFG1
    g = np.load(os.path.join(GOLDEN, "cfg1_fwd.npz"))
    inp = gi.layer_inputs(geo)
    h = _prefix_mean_gpu(inp["x"], "fp64")
    assert hashlib.sha256(h.numpy().tobytes()).hexdigest() == str(g["h_sha"])
    got = _route_gpu(inp["x"], inp["w"]["router_down"], inp["w"]["router_up"], geo["top"],
                     torch.float32)
    assert np.array_equal(got["top_idx"], g["top_idx"])
    assert O.scaled_err(got["probs"], g["probs"]) < 1e-5
    assert O.scaled_err(got["gates"], g["gates"]) < 1e-5


@pytest.mark.parametrize("compute,x_dtype,B,S,d,r,nb,top", [
    ("bf16", torch.bfloat16, 2, 2048, 1024, 32, 8, 2),   # config-2 router geometry
    ("bf16", torch.bfloat16, 1, 1000, 2048, 64, 32, 4),  # config-4 router geometry, ragged S
    ("f32", torch.float32, 2, 300, 256, 16, 8, 2),       # SIMT head, odd rank
    ("bf16", torch.float32, 1, 513, 512, 32, 8, 2),      # fp32 residual stream under autocast
])
def test_router_matches_oracle(compute, x_dtype, B, S, d, r, nb, top):
    torch.manual_seed(B * 1000 + S)
    x = torch.randn(B, S, d).to(x_dtype)
    w_down = torch.randn(r, d) * 0.02
    w_up = torch.randn(nb, r) * 0.02 * 8
    cd = torch.bfloat16 if compute == "bf16" else torch.float32
    got = _route_gpu(x, w_down, w_up, top, cd)
    rt = O.router_forward(x.float().numpy(), w_down.numpy(), w_up.numpy(), top, compute)
    _assert_indices(got["top_idx"], rt, top, "router")
    tol = 1e-5 if compute == "f32" else 2e-2
    assert O.scaled_err(got["probs"], rt["probs"]) < tol
    assert O.scaled_err(got["gates"], rt["gates"]) < tol


def test_router_prefix_certificate_fallback_inside_the_head():
    """The router's prefix mean runs exact fp64 chunk carries; columns whose
    dynamic range fails the certificate (a 1e-30 next to O(1) values, a column
    scaled by 1e30) take the sequential walk. Indices must still match the
    oracle bitwise."""
    torch.manual_seed(41)
    x = torch.randn(2, 300, 256)
    x[0, 17, 5] = 1e-30
    x[1, :, 77] *= 1e30
    x = x.to(torch.bfloat16)
    w_down = torch.randn(32, 256) * 0.02
    w_up = torch.randn(8, 32) * 0.2
    got = _route_gpu(x, w_down, w_up, 2, torch.bfloat16)
    rt = O.router_forward(x.float().numpy(), w_down.numpy(), w_up.numpy(), 2, "bf16")
    _assert_indices(got["top_idx"], rt, 2, "router with fallback columns")
    assert O.scaled_err(got["probs"], rt["probs"]) < 2e-2
    assert O.scaled_err(got["gates"], rt["gates"]) < 2e-2


def _route_shards_in_one_process(x, w_down, w_up, top, compute_dtype, sizes, scan_mode, noise=None):
    """The sequence-sharded router's exchange, its ranks emulated in rank order
    in one process (the all-gather is a stack; the chain passes carry_out on)."""
    from naylis_b200.sequence_parallel import CudaShardOps
    xd = x.cuda()
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
    shards = [xd[:, s0:s0 + n].contiguous() for s0, n in zip(starts, sizes)]
    noises = [None if noise is None else noise.cuda()[:, s0:s0 + n] for s0, n in zip(starts, sizes)]
    ops = [CudaShardOps(w_down.cuda(), w_up.cuda(), top, nz, compute_dtype) for nz in noises]
    W = len(sizes)
    outs, chained = [], False
    if scan_mode == "fp64":
        stats_all = torch.stack([o.stats(xs) for o, xs in zip(ops, shards)])
        carries = [o.carry(stats_all, W, j) for j, o in enumerate(ops)]
        assert len({u for _, u in carries}) == 1        # every rank takes the same branch
        chained = carries[0][1] > 0
        carry = carries[0][0]
        for j in range(W):
            c_in = carry if chained else carries[j][0]
            p, i, g, c_out = ops[j].route(shards[j], starts[j], c_in, chained, scan_mode)
            outs.append((p, i, g))
            carry = c_out
    else:
        chained = True
        carry = ops[0].zero_carry(shards[0], scan_mode)
        for j in range(W):
            p, i, g, carry = ops[j].route(shards[j], starts[j], carry, True, scan_mode)
            outs.append((p, i, g))
    torch.cuda.synchronize()
    cat = lambda k: torch.cat([o[k] for o in outs], 1).cpu().numpy()
    return {"probs": cat(0), "top_idx": cat(1), "gates": cat(2)}, chained


@pytest.mark.parametrize("scan_mode,extreme,x_dtype,compute", [
    ("fp64", False, torch.bfloat16, torch.bfloat16),
    ("fp64", False, torch.float32, torch.float32),
    ("fp64", True, torch.bfloat16, torch.bfloat16),
    ("fp32", False, torch.bfloat16, torch.bfloat16),
    ("fp32", False, torch.float32, torch.float32),
])
def test_router_sequence_shards_equal_the_whole_sequence_bitwise(scan_mode, extreme, x_dtype, compute):
    """Rows split over 5 shards of unequal length (one empty): every output of
    the shards, concatenated, equals the single-call router bit for bit. With
    columns that fail the exactness certificate the shards run as a chain."""
    torch.manual_seed(7)
    B, d, sizes = 2, 256, [300, 1, 0, 257, 466]
    x = torch.randn(B, sum(sizes), d)
    if extreme:
        x[0, 17, 5] = 1e-30
        x[1, :, 77] *= 1e30
    x = x.to(x_dtype)
    w_down = torch.randn(32, d) * 0.02
    w_up = torch.randn(8, 32) * 0.2
    noise = torch.randn(B, sum(sizes), 8)
    whole = _route_gpu(x, w_down, w_up, 2, compute, noise=noise, scan_mode=scan_mode)
    got, chained = _route_shards_in_one_process(x, w_down, w_up, 2, compute, sizes, scan_mode, noise)
    assert chained == (extreme or scan_mode == "fp32")
    for k in ("probs", "top_idx", "gates"):
        assert np.array_equal(got[k], whole[k]), k


def test_router_noise_goes_into_topk_only():
    torch.manual_seed(3)
    x = torch.randn(2, 256, 512, dtype=torch.bfloat16)
    w_down = torch.randn(32, 512) * 0.02
    w_up = torch.randn(8, 32) * 0.2
    noise = torch.randn(2, 256, 8) * 2.0
    got = _route_gpu(x, w_down, w_up, 2, torch.bfloat16, noise=noise)
    rt = O.router_forward(x.float().numpy(), w_down.numpy(), w_up.numpy(), 2, "bf16",
                          noise=noise.numpy())
    _assert_indices(got["top_idx"], rt, 2, "noisy router")
    assert O.scaled_err(got["probs"], rt["probs"]) < 2e-2   # probs from the clean logits
    assert O.scaled_err(got["gates"], rt["gates"]) < 2e-2   # gates from the noisy top values


@pytest.mark.parametrize("compute,tol", [("f32", 1e-5), ("bf16", 2e-2)])
@pytest.mark.parametrize("r,nb,top", [(32, 8, 2), (64, 16, 2), (16, 32, 3)])
def test_router_backward_matches_oracle(compute, tol, r, nb, top):
    # (32, 8): config 2; (64, 16): rank-64 tensor-core pass, 16-block dW_up;
    # (16, 32): rank 16 (SIMT dx / dW_down), more blocks than the register dW_up holds
    torch.manual_seed(7)
    B, S, d = 2, 384, 256
    cd = torch.bfloat16 if compute == "bf16" else torch.float32
    x = torch.randn(B, S, d).to(cd)
    w_down = torch.randn(r, d) * 0.05
    w_up = torch.randn(nb, r) * 0.3
    dgates = torch.randn(B, S, top)
    dprobs = torch.randn(B, S, nb)
    got = _route_gpu(x, w_down, w_up, top, cd, grad=(dgates, dprobs))
    rt = O.router_forward(x.float().numpy(), w_down.numpy(), w_up.numpy(), top, compute)
    _assert_indices(got["top_idx"], rt, top, "router")
    g = rt["gates"].astype(np.float64)
    dlg = dgates.numpy().astype(np.float64) * np.maximum(g, 1e-9)   # d/dlog_gates
    ref = O.router_backward(rt, x.float().numpy(), w_down.numpy(), w_up.numpy(), dlg,
                            dprobs.numpy())
    for key in ("dx", "dw_down", "dw_up"):
        err = O.scaled_err(got[key], ref[key])
        assert err < tol, f"{key}: {err:.3e}"


@pytest.mark.parametrize("compute", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nb,top", [(8, 1), (8, 2), (8, 3), (8, 4), (32, 2), (32, 4), (32, 5)])
def test_topk_tie_order_matches_torch_cuda(compute, nb, top):
    """torch.topk leaves the order of equal values to the implementation. On
    CUDA, the reference's eager router (model.py:214) runs torch's CUDA topk;
    the kernel reproduces its choice and order on ties. With W_up = 0 the
    logits are exactly 0 and the noisy logits equal the noise, which here takes
    values in {1, 2, 3} only, so nearly every token has ties at every boundary.
    Indices must equal torch.topk's on this GPU, token for token."""
    torch.manual_seed(11 + top + nb)
    B, S, d, r = 4, 512, 64, 8
    x = torch.randn(B, S, d)
    w_down = torch.randn(r, d) * 0.1
    w_up = torch.zeros(nb, r)
    noise = torch.randint(1, 4, (B, S, nb)).float()
    got = _route_gpu(x, w_down, w_up, top, compute, noise=noise, scan_mode="fp32")
    ref_v, ref_i = torch.topk(noise.cuda(), top, dim=-1)
    ref_i = ref_i.cpu().numpy()
    tied = (noise.sort(-1, descending=True).values[..., :top + 1].diff(dim=-1) == 0).any(-1)
    assert float(tied.float().mean()) > 0.5          # the case really is tie-heavy
    mism = np.any(got["top_idx"] != ref_i, axis=-1)
    assert not mism.any(), (f"{int(mism.sum())} of {mism.size} tokens differ from torch.topk on CUDA; "
                            f"first: noise {noise.reshape(-1, nb)[mism.reshape(-1)][:3].tolist()}, "
                            f"kernel {got['top_idx'].reshape(-1, top)[mism.reshape(-1)][:3].tolist()}, "
                            f"torch {ref_i.reshape(-1, top)[mism.reshape(-1)][:3].tolist()}")
    assert np.array_equal(got["top_idx"], O.topk_cuda_order(noise.numpy(), top)[0])


def _torch_cuda_router(x, w_down, w_up, top, noise=None):
    """The reference's eager router (model.py:169-220) as torch runs it on this
    GPU under bf16 autocast with fp32 master weights: CUDA cumsum (sequential
    fp32 per column), IEEE division by t+1, cuBLAS bf16 linears, tanh, fp32
    softmax, torch's CUDA topk."""
    import torch.nn.functional as F
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        cs = torch.cumsum(x.float(), dim=1)
        h = cs / torch.arange(1, x.shape[1] + 1, device=x.device, dtype=cs.dtype).view(1, -1, 1)
        logits = F.linear(torch.tanh(F.linear(h.to(w_down.dtype), w_down)), w_up).float()
    noisy = logits if noise is None else logits + noise
    probs = torch.softmax(logits, -1)
    vals, idx = noisy.topk(top, dim=-1)
    return logits, probs, idx, torch.softmax(vals, -1)


@pytest.mark.parametrize("noise_on", [False, True])
def test_router_fp32_scan_matches_torch_cuda_eager_router(noise_on):
    """The default scan mode ("fp32") against the reference's eager router
    math run by torch on this B200 at BASELINE config 2's full size (x bf16
    (8, 2048, 1024), rank 32, 8 blocks, top-2). The prefix means are bitwise
    equal (tested above); the bf16 logits can differ only where cuBLAS and the
    kernel accumulate the rank-32 / d=1024 dot products in different orders and
    the fp32 sums round to different bf16 values. So every token must route
    alike except tokens whose torch top-k margin is within one bf16 rounding of
    the logits (at most 4 ulps of the k-th logit), and those stay rare."""
    torch.manual_seed(2024)
    B, S, d, r, nb, top = 8, 2048, 1024, 32, 8, 2
    x = torch.randn(B, S, d).to(torch.bfloat16)
    w_down = torch.randn(r, d) * 0.02
    w_up = torch.randn(nb, r) * 0.02
    noise = None
    if noise_on:
        from naylis_b200 import mom_kernels as mk
        torch.manual_seed(5)
        noise = mk.gumbel_noise((B, S, nb), torch.device("cuda"), 1.0).cpu()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        got = _route_gpu(x, w_down, w_up, top, torch.bfloat16, noise=noise, scan_mode="fp32")
    xd, wd, wu = x.cuda(), w_down.cuda(), w_up.cuda()
    logits, probs, idx, gates = _torch_cuda_router(xd, wd, wu, top, None if noise is None else noise.cuda())
    ref_i = idx.cpu().numpy()
    mism = np.any(got["top_idx"] != ref_i, axis=-1).reshape(-1)
    noisy = (logits if noise is None else logits + noise.cuda()).reshape(-1, nb)
    srt = noisy.sort(-1, descending=True).values
    margin = (srt[:, top - 1] - srt[:, top]).cpu().numpy()
    # a bf16 value has 8 significant bits: 4 ulps of the k-th logit ~ 4 * |v| * 2^-7
    kth = np.abs(srt[:, top - 1].cpu().numpy())
    allowed = margin <= 4 * kth * 2.0 ** -7
    assert not (mism & ~allowed).any(), \
        f"{int((mism & ~allowed).sum())} tokens differ with torch margins {margin[mism & ~allowed][:8]}"
    assert mism.mean() < 2e-3, f"{int(mism.sum())} of {mism.size} tokens differ (all near ties)"
    assert O.scaled_err(got["probs"].reshape(-1, nb), probs.reshape(-1, nb).cpu().numpy()) < 2e-2
    ok = ~mism
    assert O.scaled_err(got["gates"].reshape(-1, top)[ok], gates.reshape(-1, top).cpu().numpy()[ok]) < 2e-2


@pytest.mark.parametrize("N,nb,top,idx_dtype", [(16384, 8, 2, torch.int64), (1000, 20, 4, torch.int32),
                                                (77, 32, 3, torch.int64)])
def test_router_aux_matches_reference_formula(N, nb, top, idx_dtype):
    """The fused aux loss / entropy / dead fraction of a layer against the
    reference's torch expressions (model.py:476-517) on the same router outputs,
    and the aux gradient w.r.t. probs against torch autograd. Block 0 is never
    selected, so the dead fraction is non-zero."""
    from naylis_b200 import mom_kernels as mk
    torch.manual_seed(7)
    dev = torch.device("cuda")
    probs = torch.softmax(torch.randn(N, nb, device=dev), -1).requires_grad_(True)
    idx = torch.argsort(torch.rand(N, nb, device=dev), -1)[:, :top]
    idx = torch.where(idx == 0, torch.full_like(idx, nb - 1), idx).to(idx_dtype)   # repeats allowed
    out = mk.router_aux(probs, idx, nb)
    pr = probs.detach().clone().requires_grad_(True)
    blocks = torch.arange(nb, device=dev)
    sel = (idx.long().unsqueeze(2) == blocks.view(1, 1, -1)).any(1)
    frac = sel.float().mean(0)
    aux = nb * (frac * pr.mean(0)).sum()
    ent = -(pr * pr.clamp_min(1e-9).log()).sum(-1).mean()
    dead = (~sel.any(0)).float().mean()
    assert torch.allclose(out[0], aux, rtol=1e-5, atol=1e-7)
    assert torch.allclose(out[1], ent, rtol=1e-5, atol=1e-6)
    assert float(out[2]) == float(dead) and float(dead) > 0
    assert torch.equal(out[3:], frac)
    (out[0] * 0.3).backward()
    (aux * 0.3).backward()
    assert torch.allclose(probs.grad, pr.grad, rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("shape,scale", [((8, 2048, 8), 1.0), ((3, 7, 5), 0.7), ((1, 1, 3), 2.5)])
def test_gumbel_noise_is_the_torch_expression_bitwise(shape, scale):
    """The router's Gumbel noise as one kernel equals the reference's torch
    expression noise_scale * -log(-log(u + 1e-9) + 1e-9) on the same draws u,
    bit for bit (105 values: the scalar tail; 131,072: the vector form)."""
    from naylis_b200 import mom_kernels as mk
    dev = torch.device("cuda")
    torch.manual_seed(9)
    got = mk.gumbel_noise(shape, dev, scale)
    torch.manual_seed(9)
    u = torch.rand(shape, device=dev, dtype=torch.float32)
    want = scale * (-torch.log(-torch.log(u + 1e-9) + 1e-9))
    assert torch.equal(got, want)


@pytest.mark.parametrize("r", [32, 64])
def test_router_backward_from_the_bf16_copy_of_x_is_identical(r):
    """The router's backward uses x only rounded to bf16 (dW_down = u^T bf16(x));
    handing it that rounding (x_lowp, as the decoder's add + RMSNorm writes it)
    instead of the fp32 x gives the same dx bit for bit (an fp32 dx) and the
    same dW_down, dW_up up to the order of their fp32 atomic sums."""
    from naylis_b200 import mom_kernels as mk
    torch.manual_seed(17)
    dev = torch.device("cuda")
    B, S, d, nb, top = 2, 700, 1024, 8, 2
    x = torch.randn(B, S, d, device=dev)
    w_down = 0.02 * torch.randn(r, d, device=dev)
    w_up = 0.02 * torch.randn(nb, r, device=dev)
    dlg = torch.randn(B, S, top, device=dev)
    dpr = torch.randn(B, S, nb, device=dev)
    out = []
    for lowp in (None, x.bfloat16()):
        xd, wd, wu = (t.clone().requires_grad_(True) for t in (x, w_down, w_up))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            probs, _, _, lg = mk.mom_route_log_gates(xd, wd, wu, top, None, x_lowp=lowp)
        torch.autograd.backward([lg, probs], [dlg, dpr])
        out.append((xd.grad, wd.grad, wu.grad))
    assert out[1][0].dtype == torch.float32
    assert torch.equal(out[0][0], out[1][0])
    for a, b in zip(out[0][1:], out[1][1:]):
        assert float((a - b).abs().max()) <= 1e-5 * float(b.abs().max())
