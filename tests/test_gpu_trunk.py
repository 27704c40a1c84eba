"""GPU parity of the decoder trunk's fused kernels (csrc/trunk.cu, through
the C ABI) with torch's own ops on the same bf16 inputs: the rotary embedding
of the fused q/k/v projection (the reference's apply_rotary_pos_emb under bf16
autocast: fp32 math on bf16 q / k with fp32 cos / sin, rounded to bf16 for
attention) and the SwiGLU gate (LlamaMLP's silu(gate) * up in bf16), forward
and backward.

RoPE is bit-exact (the same fp32 products and sums, no fused multiply-add).
Both kernels have a 16-byte vector form and an element form (head_dim not a
multiple of 16, gate width not a multiple of 8): the shapes cover both.
SwiGLU goes through expf and one division like torch's kernels; a result
may still land one bf16 rounding step apart where torch's exp differs in the
last fp32 bit, so it is held to at most one bf16 ulp, on under 0.1 % of the
elements.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rope_ref(qkv, cos, sin, H):
    from naylis_b200.decoder import apply_rope
    B, S, d3 = qkv.shape
    hd = d3 // (3 * H)
    t = qkv.view(B, S, 3, H, hd)
    q, k, v = (t[:, :, i].transpose(1, 2) for i in range(3))
    return apply_rope(q, cos, sin).bfloat16(), apply_rope(k, cos, sin).bfloat16(), v


@pytest.mark.parametrize("B,S,H,hd", [(2, 300, 4, 64), (1, 128, 2, 128), (1, 17, 3, 32), (1, 9, 2, 24)])
def test_rope_qkv_matches_torch_bitwise(B, S, H, hd):
    from naylis_b200 import trunk
    from naylis_b200.decoder import rope_tables
    torch.manual_seed(0)
    dev = torch.device("cuda")
    qkv = torch.randn(B, S, 3 * H * hd, device=dev).bfloat16().requires_grad_(True)
    cos, sin = rope_tables(S, hd, 500000.0, dev)
    q, k, v = trunk.rope_qkv(qkv, cos, sin, H)
    qkv2 = qkv.detach().clone().requires_grad_(True)
    rq, rk, rv = _rope_ref(qkv2, cos, sin, H)
    for a, b in ((q, rq), (k, rk), (v, rv)):
        assert a.shape == b.shape and torch.equal(a, b)
    g = [torch.randn(B, H, S, hd, device=dev).bfloat16() for _ in range(3)]
    torch.autograd.backward([q, k, v], g)
    torch.autograd.backward([rq, rk, rv], g)
    assert torch.equal(qkv.grad, qkv2.grad)


@pytest.mark.parametrize("N,f", [(4096, 2816), (333, 64), (50, 36)])
def test_swiglu_matches_torch(N, f):
    from naylis_b200 import trunk
    torch.manual_seed(1)
    dev = torch.device("cuda")
    gu = (torch.randn(N, 2 * f, device=dev) * 3).bfloat16().requires_grad_(True)
    h = trunk.swiglu(gu)
    gu2 = gu.detach().clone().requires_grad_(True)
    g2, u2 = gu2.chunk(2, dim=-1)
    ref = torch.nn.functional.silu(g2) * u2
    dh = torch.randn(N, f, device=dev).bfloat16()
    h.backward(dh)
    ref.backward(dh)

    def ulps_apart(a, b):
        a, b = a.float(), b.float()
        ulp = torch.clamp(b.abs(), min=2.0 ** -126) * 2.0 ** -7
        diff = (a - b).abs()
        return float((diff > 0).float().mean()), float((diff / ulp).max())

    for name, (a, b) in {"h": (h, ref), "dgu": (gu.grad, gu2.grad)}.items():
        frac, worst = ulps_apart(a, b)
        assert worst <= 1.0 and frac < 1e-3, (name, frac, worst)


@pytest.mark.parametrize("delta_dtype,scaled,want_f32,d", [
    (None, False, False, 1024), (torch.bfloat16, False, True, 1024), (torch.bfloat16, True, False, 1024),
    (torch.float32, False, False, 1024), (torch.bfloat16, True, True, 2048), (torch.float32, True, False, 256),
    (None, False, False, 128)])
def test_add_rmsnorm_matches_torch(delta_dtype, scaled, want_f32, d):
    """x_new = x + s * delta then Llama's RMSNorm (transformers' LlamaRMSNorm:
    fp32 x * rsqrt(mean(x^2) + eps), times the weight) against torch ops on the
    same inputs. x_new is the same two roundings (exact match); y differs from
    torch's only by the order of the mean's sum (bf16 output: at most one ulp);
    gradients (the residual gradient passed through plus the norm's, dw, ds)
    agree to 1e-5 of their largest magnitude. d = 1024 and 2048 take the
    backward with a warp pair per token, 128 and 256 a warp per token; 777
    tokens leave a ragged last group."""
    from naylis_b200 import trunk
    torch.manual_seed(2)
    dev = torch.device("cuda")
    N, eps = 777, 1e-5
    x = torch.randn(N, d, device=dev).requires_grad_(True)
    delta = None if delta_dtype is None else torch.randn(N, d, device=dev).to(delta_dtype).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(d, device=dev)).requires_grad_(True)
    s = torch.tensor([0.37], device=dev, requires_grad=True) if scaled else None
    outs = trunk.add_rmsnorm(x, delta, w, eps, scale=s, want_f32=want_f32)
    xr = x.detach().clone().requires_grad_(True)
    dr = None if delta is None else delta.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    sr = None if s is None else s.detach().clone().requires_grad_(True)
    xn = xr if dr is None else xr + (dr if sr is None else sr * dr)
    yr = wr * (xn * torch.rsqrt(xn.pow(2).mean(-1, keepdim=True) + eps))
    assert torch.equal(outs[0], xn)
    assert ((outs[1].float() - yr).abs() <= yr.abs() * 2.0 ** -7 + 1e-30).all()
    if want_f32:
        assert torch.allclose(outs[2], yr, rtol=1e-5, atol=1e-6)
    gx = torch.randn(N, d, device=dev)
    gy = torch.randn(N, d, device=dev).bfloat16()
    grads = [gx, gy] + ([torch.randn(N, d, device=dev)] if want_f32 else [])
    torch.autograd.backward(list(outs), grads)
    ref_out = [xn, yr.bfloat16()] + ([yr] if want_f32 else [])
    # the reference path takes the bf16 y through a cast: its gradient is gy in fp32
    torch.autograd.backward([xn, yr] + ([] if not want_f32 else []),
                            [gx, gy.float() + (grads[2] if want_f32 else 0)])

    def err(a, b):
        return float((a.float() - b.float()).abs().max() / b.float().abs().max())

    assert err(x.grad, xr.grad) < 1e-5
    assert err(w.grad, wr.grad) < 1e-5
    if delta is not None:
        tol = 1e-2 if delta_dtype == torch.bfloat16 else 1e-5     # bf16 delta gradient: one rounding
        assert err(delta.grad, dr.grad) < tol
    if scaled:
        assert abs(float(s.grad) - float(sr.grad)) <= 1e-4 * abs(float(sr.grad))


@pytest.mark.parametrize("R,V,scale", [(300, 32000, 1.0), (257, 1000, 30.0), (64, 1003, 3.0), (5, 8, 1.0)])
def test_cross_entropy_matches_torch(R, V, scale):
    """The LM head's loss (the reference's cross_entropy(logits.float(), labels,
    reduction="sum"), labels -100 ignored) from bf16 logits against torch on
    the same values: the loss within 1e-5 relative (the kernel sums e^(x - m)
    in another order and through exp2), the bf16 logit gradient within one bf16
    rounding step of torch's fp32 gradient cast to bf16. V = 1003 takes the
    element form of the kernels; scale 30 makes the running maximum move."""
    from naylis_b200 import trunk
    torch.manual_seed(3)
    dev = torch.device("cuda")
    logits = (scale * torch.randn(R, V, device=dev)).bfloat16().requires_grad_(True)
    labels = torch.randint(0, V, (R,), device=dev)
    labels[::7] = -100
    loss = trunk.cross_entropy_sum(logits, labels)
    ref_in = logits.detach().float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(ref_in, labels, reduction="sum")
    assert abs(float(loss) - float(ref)) <= 1e-5 * abs(float(ref)) + 1e-5
    g = 0.37
    (loss * g).backward()
    (ref * g).backward()
    got = logits.grad.float()
    want = ref_in.grad
    assert torch.all(got[labels == -100] == 0)
    # one bf16 step of the fp32 value, or an fp32 ulp-level absolute floor
    assert ((got - want).abs() <= want.abs() * 2.0 ** -7 + 1e-7).all()


@pytest.mark.parametrize("nb,bs,d,n", [(8, 128, 1024, 1024), (4, 32, 256, 128)])
def test_bank_kv_matches_two_linears(nb, bs, d, n):
    """The bank's k / v projections as one batched GEMM (trunk.bank_kv) against
    two bf16 linears on the bank cast to bf16: k and v within one bf16 rounding
    step (cuBLAS may sum in another order), the bank and weight gradients
    within 1e-2 of their largest magnitude (the reference rounds them through
    bf16, bank_kv keeps fp32) — also when dK / dV do not arrive side by side."""
    from naylis_b200 import trunk
    torch.manual_seed(11)
    dev = torch.device("cuda")
    L = nb * bs
    bank = torch.nn.Parameter(0.02 * torch.randn(nb, bs * d, device=dev))
    wk = torch.nn.Parameter(0.02 * torch.randn(n, d, device=dev))
    wv = torch.nn.Parameter(0.02 * torch.randn(n, d, device=dev))
    gk = torch.randn(L, n, device=dev).bfloat16()
    gv = torch.randn(L, n, device=dev).bfloat16()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        k, v = trunk.bank_kv(bank, wk, wv, L)
        kr = torch.nn.functional.linear(bank.view(L, d), wk)
        vr = torch.nn.functional.linear(bank.view(L, d), wv)
    assert k.is_contiguous() and v.is_contiguous() and k.dtype == torch.bfloat16
    for a, b in ((k, kr), (v, vr)):
        assert ((a.float() - b.float()).abs() <= b.float().abs() * 2.0 ** -7 + 1e-6).all()
    grads = torch.autograd.grad((k.float() * gk.float()).sum() + (v.float() * gv.float()).sum(), (bank, wk, wv))
    refs = torch.autograd.grad((kr.float() * gk.float()).sum() + (vr.float() * gv.float()).sum(), (bank, wk, wv))
    for a, b in zip(grads, refs):
        assert float((a - b).abs().max()) <= 1e-2 * float(b.abs().max())


@pytest.mark.parametrize("L,n", [(1024, 1024), (37, 12)])
def test_kv_pack_is_the_torch_cast_bitwise(L, n):
    """The read backward's fp32 dK / dV cast to bf16 side by side in one kernel
    (mom_kv_pack_bf16, through the C ABI) equals torch's cast of their
    concatenation bit for bit, large and small magnitudes included."""
    from naylis_b200 import _lib
    torch.manual_seed(13)
    dev = torch.device("cuda")
    dk = torch.randn(L, n, device=dev) * torch.logspace(-30, 30, L * n, device=dev).view(L, n)
    dv = torch.randn(L, n, device=dev)
    out = torch.empty(L, 2 * n, dtype=torch.bfloat16, device=dev)
    _lib.call("mom_kv_pack_bf16", dk.data_ptr(), dv.data_ptr(), L, n, out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    assert torch.equal(out.view(torch.int16), torch.cat([dk, dv], 1).bfloat16().view(torch.int16))
