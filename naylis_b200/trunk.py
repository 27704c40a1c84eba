"""Autograd wrappers of the decoder trunk's fused bf16 kernels (csrc/trunk.cu):
the rotary embedding of the fused q/k/v projection, the SwiGLU gate, the
residual add + RMSNorm and the LM head's cross-entropy.

Both reproduce the rounding points of the reference's trunk under bf16
autocast (transformers' Llama apply_rotary_pos_emb and LlamaMLP); they take
and return bf16 CUDA tensors only and raise otherwise (the decoder keeps
torch's ops for fp32 runs).
"""
from __future__ import annotations

import torch
from torch.utils.weak import WeakIdKeyDictionary

from . import _lib


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_bf16(*ts):
    for t in ts:
        if not (t.is_cuda and t.dtype == torch.bfloat16):
            raise RuntimeError(f"naylis_b200 trunk kernels take bf16 CUDA tensors, got {t.dtype} on {t.device}")


class _RopeQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin, n_heads):
        B, S, d3 = qkv.shape
        hd = d3 // (3 * n_heads)
        qkv = qkv.contiguous()
        cos = cos.float().contiguous()
        sin = sin.float().contiguous()
        q = torch.empty(B, S, n_heads, hd, dtype=torch.bfloat16, device=qkv.device)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        _lib.call("mom_rope_qkv_fwd", qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), B, S, n_heads, hd,
                  q.data_ptr(), k.data_ptr(), v.data_ptr(), _stream(qkv))
        ctx.save_for_backward(cos, sin)
        ctx.meta = (B, S, n_heads, hd)
        # attention's (B, H, S, hd) views over the token-major buffers
        return q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin = ctx.saved_tensors
        B, S, H, hd = ctx.meta
        tok = [t.to(torch.bfloat16).transpose(1, 2).contiguous() for t in (dq, dk, dv)]
        dqkv = torch.empty(B, S, 3 * H * hd, dtype=torch.bfloat16, device=cos.device)
        _lib.call("mom_rope_qkv_bwd", tok[0].data_ptr(), tok[1].data_ptr(), tok[2].data_ptr(), cos.data_ptr(),
                  sin.data_ptr(), B, S, H, hd, dqkv.data_ptr(), _stream(dqkv))
        return dqkv, None, None, None


def rope_qkv(qkv, cos, sin, n_heads: int):
    """qkv (B, S, 3*H*hd) bf16 -> q, k, v as (B, H, S, hd) bf16 views, q and k
    rotated (fp32 math with fp32 cos / sin (S, hd), rounded to bf16)."""
    _need_bf16(qkv)
    if qkv.shape[-1] % (6 * n_heads):
        raise RuntimeError("rope_qkv: last dimension must be 3 * n_heads * (even head_dim)")
    return _RopeQKV.apply(qkv, cos, sin, int(n_heads))


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        f = gu.shape[-1] // 2
        N = gu.numel() // gu.shape[-1]
        h = torch.empty(*gu.shape[:-1], f, dtype=torch.bfloat16, device=gu.device)
        _lib.call("mom_swiglu_fwd", gu.data_ptr(), N, f, h.data_ptr(), _stream(gu))
        ctx.save_for_backward(gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        f = gu.shape[-1] // 2
        N = gu.numel() // gu.shape[-1]
        dh = dh.to(torch.bfloat16).contiguous()
        dgu = torch.empty_like(gu)
        _lib.call("mom_swiglu_bwd", dh.data_ptr(), gu.data_ptr(), N, f, dgu.data_ptr(), _stream(gu))
        return dgu


def swiglu(gu):
    """gu (..., 2f) bf16 = [gate | up] -> bf16(bf16(silu(gate)) * up) (..., f)."""
    _need_bf16(gu)
    if gu.shape[-1] % 4:
        raise RuntimeError("swiglu: the gate/up width 2f must have f even")
    return _SwiGLU.apply(gu)


class _AddRMSNorm(torch.autograd.Function):
    """x_new = x + s * delta, y = RMSNorm(x_new) (bf16, and fp32 when asked)."""

    @staticmethod
    def forward(ctx, x, delta, scale, weight, eps, want_f32):
        x = x.contiguous()
        d = x.shape[-1]
        N = x.numel() // d
        x_out = torch.empty_like(x)
        y16 = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        y32 = torch.empty_like(x) if want_f32 else None
        rstd = torch.empty(N, dtype=torch.float32, device=x.device)
        dcode = _lib.F32
        if delta is not None:
            delta = delta.contiguous()
            dcode = _lib.BF16 if delta.dtype == torch.bfloat16 else _lib.F32
        sc = None if scale is None else scale.detach().float().contiguous()
        w = weight.detach().float().contiguous()
        _lib.call("mom_add_rmsnorm_fwd", x.data_ptr(), None if delta is None else delta.data_ptr(), dcode,
                  None if sc is None else sc.data_ptr(), w.data_ptr(), N, d, float(eps), x_out.data_ptr(),
                  y16.data_ptr(), None if y32 is None else y32.data_ptr(), rstd.data_ptr(), _stream(x))
        ctx.save_for_backward(x_out, rstd, w, delta, sc)
        ctx.meta = (dcode, delta is not None, scale is not None, scale.dtype if scale is not None else None,
                    weight.dtype)
        # an output nobody reads (the final norm's residual stream) reaches the backward as
        # None, so the kernel skips it instead of reading a zero-filled gradient
        ctx.set_materialize_grads(False)
        if want_f32:
            return x_out, y16, y32
        return x_out, y16

    @staticmethod
    def backward(ctx, dx_out, dy16, dy32=None):
        x_out, rstd, w, delta, sc = ctx.saved_tensors
        dcode, has_delta, has_scale, scale_dtype, w_dtype = ctx.meta
        d = x_out.shape[-1]
        N = x_out.numel() // d
        g16 = None if dy16 is None else dy16.to(torch.bfloat16).contiguous()
        g32 = None if dy32 is None else dy32.float().contiguous()
        gx = None if dx_out is None else dx_out.float().contiguous()
        dx = torch.empty_like(x_out)
        ddelta = torch.empty_like(delta) if has_delta else None
        dw = torch.empty(d, dtype=torch.float32, device=x_out.device)
        dsc = torch.empty(1, dtype=torch.float32, device=x_out.device) if has_scale else None
        if g16 is None and g32 is None:
            g32 = torch.zeros_like(x_out)
        _lib.call("mom_add_rmsnorm_bwd", x_out.data_ptr(), rstd.data_ptr(), w.data_ptr(),
                  None if delta is None else delta.data_ptr(), dcode, None if sc is None else sc.data_ptr(),
                  None if g16 is None else g16.data_ptr(), None if g32 is None else g32.data_ptr(),
                  None if gx is None else gx.data_ptr(), N, d, dx.data_ptr(),
                  None if ddelta is None else ddelta.data_ptr(), dw.data_ptr(),
                  None if dsc is None else dsc.data_ptr(), _stream(x_out))
        return (dx, ddelta, None if dsc is None else dsc.to(scale_dtype), dw.to(w_dtype), None, None)


def add_rmsnorm(x, delta, weight, eps: float, scale=None, want_f32: bool = False):
    """The residual add fused with the RMSNorm that follows it:
    x_new = x + scale * delta (delta bf16 / fp32 or None, scale a (1,) tensor or
    None), y = weight * x_new / sqrt(mean(x_new^2) + eps). Returns (x_new fp32,
    y bf16) or, with want_f32, (x_new, y bf16, y fp32)."""
    if not (x.is_cuda and x.dtype == torch.float32):
        raise RuntimeError("add_rmsnorm: x must be an fp32 CUDA tensor (the residual stream)")
    return _AddRMSNorm.apply(x, delta, scale, weight, float(eps), bool(want_f32))


# parameter -> [group buffer, its rows (a view), the parameter's _version when the
# rows were written]; weak keys, so the buffers go with the parameters and are
# not part of what a parameter pickles
_SHADOWS = WeakIdKeyDictionary()
_SHADOW_GEN = [0]   # bumped whenever rows are (re)registered, so holders of pointers can re-read them


def _bf16_weights(weights):
    """One bf16 buffer holding cat(weights) for the GEMM, kept per parameter and
    reused while every weight's `_version` matches the one its rows were written
    at. The optimizer of this package rewrites the rows in its update and marks
    them fresh (`mark_bf16_fresh`); any other in-place change of a weight makes
    the next call recast it."""
    rows = sum(w.shape[0] for w in weights)
    ent = [_SHADOWS.get(w) for w in weights]
    buf = ent[0][0] if ent[0] is not None else None
    if buf is None or any(e is None or e[0] is not buf for e in ent) or buf.shape[0] != rows or \
            buf.device != weights[0].device:
        buf = torch.empty(rows, weights[0].shape[1], dtype=torch.bfloat16, device=weights[0].device)
        o = 0
        for w in weights:
            _SHADOWS[w] = [buf, buf[o:o + w.shape[0]], -1]
            o += w.shape[0]
        _SHADOW_GEN[0] += 1
    for w in weights:
        e = _SHADOWS[w]
        if e[2] != w._version:
            e[1].copy_(w.detach())
            e[2] = w._version
    return buf


def bf16_generation() -> int:
    """A counter that changes whenever a parameter's bf16 rows are (re)registered."""
    return _SHADOW_GEN[0]


def bf16_copy(param):
    """The bf16 rows registered for `param` by the bf16 projections, or None."""
    e = _SHADOWS.get(param)
    return None if e is None else e[1]


def mark_bf16_fresh(param) -> None:
    """Record that `param`'s bf16 rows were rewritten from its current values."""
    e = _SHADOWS.get(param)
    if e is not None:
        e[2] = param._version


# parameter -> [flat fp32 gradient buffer, element offset of the parameter's slot in it,
# claimed]: registered by a gradient bucketing wrapper (data_parallel.GradAllReduce).
# While a parameter's .grad is None and its slot is unclaimed, the weight-gradient GEMM
# of linear_f32grad writes straight into the slot and hands autograd a view of it, which
# AccumulateGrad then adopts as .grad (no zero fill, no add, no copy).
_GRAD_SLOTS = WeakIdKeyDictionary()


def register_grad_slot(param, flat, offset: int) -> None:
    """Declare flat[offset : offset + param.numel()] as `param`'s gradient storage."""
    _GRAD_SLOTS[param] = [flat, int(offset), False]


def release_grad_slots(params) -> None:
    """Re-arm the slots of `params` (their gradients were cleared to None)."""
    for p in params:
        e = _GRAD_SLOTS.get(p)
        if e is not None:
            e[2] = False


def unregister_grad_slots(params) -> None:
    for p in params:
        _GRAD_SLOTS.pop(p, None)


def _claim_grad_rows(weights, cols):
    """The (sum of rows, cols) fp32 view of the slots that hold cat(weights)' gradients,
    claimed for this backward, or None: every weight needs an unclaimed slot, no
    .grad yet, fp32, and the slots must follow each other in the weights' order."""
    ents = [_GRAD_SLOTS.get(w) for w in weights]
    if any(e is None or e[2] for e in ents):
        return None
    if any(w.grad is not None or w.dtype != torch.float32 for w in weights):
        return None
    flat, start = ents[0][0], ents[0][1]
    o = start
    for w, e in zip(weights, ents):
        if e[0] is not flat or e[1] != o:
            return None
        o += w.numel()
    for e in ents:
        e[2] = True
    return flat[start:o].view(-1, cols)


class _LinearF32Grad(torch.autograd.Function):
    """y = x @ cat(weights)^T in bf16 from the weights' bf16 buffer (no fp32
    concatenation, no cast when the buffer is fresh); the backward gives dx in
    bf16 and the weights' gradients from one GEMM with fp32 output, split per
    weight — written into the weights' gradient slots when they have them."""

    @staticmethod
    def forward(ctx, x, *weights):
        rows = [w.shape[0] for w in weights]
        w16 = _bf16_weights(weights)
        x16 = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        y = torch.nn.functional.linear(x16, w16)
        ctx.save_for_backward(x16, w16)
        ctx.rows = rows
        ctx.weights = weights
        ctx.x_dtype = x.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x16, w16 = ctx.saved_tensors
        dy = dy.to(torch.bfloat16)
        dx = torch.matmul(dy, w16) if ctx.needs_input_grad[0] else None
        dy2 = dy.reshape(-1, dy.shape[-1]).t()
        x2 = x16.reshape(-1, x16.shape[-1])
        slot = _claim_grad_rows(ctx.weights, x2.shape[1])
        if slot is not None:
            dw = torch.mm(dy2, x2, out_dtype=torch.float32, out=slot)
        else:
            dw = torch.mm(dy2, x2, out_dtype=torch.float32)
        grads, o = [], 0
        for n, w in zip(ctx.rows, ctx.weights):
            grads.append(dw[o:o + n] if w.dtype == torch.float32 else dw[o:o + n].to(w.dtype))
            o += n
        return (None if dx is None else dx.to(ctx.x_dtype), *grads)


def linear_f32grad(x, *weights):
    """bf16 x @ cat(weights)^T on CUDA (fp32 master weights cast once per call)
    whose weight gradients are computed in fp32 by the GEMM itself; the
    reference's autocast linear rounds them to bf16 and casts them back."""
    if not x.is_cuda:
        raise RuntimeError("linear_f32grad: CUDA tensors only")
    return _LinearF32Grad.apply(x, *weights)


def _side_by_side(a, b):
    """(R, n) a and b as one (R, 2n) tensor: a zero-copy view when b is the right
    half of a buffer whose left half is a (how the read's backward returns its
    dK / dV), else a copy."""
    R, n = a.shape
    if (b.dtype == a.dtype and b.device == a.device and a.stride() == (2 * n, 1) and b.stride() == (2 * n, 1)
            and b.data_ptr() == a.data_ptr() + n * a.element_size()):
        return a.as_strided((R, 2 * n), (2 * n, 1))
    out = torch.empty(R, 2 * n, dtype=a.dtype, device=a.device)
    out[:, :n].copy_(a)
    out[:, n:].copy_(b)
    return out


class _BankKV(torch.autograd.Function):
    """k = slots @ Wk^T, v = slots @ Wv^T for the bank's L slots (its rows viewed
    as (L, d)) as one batched bf16 GEMM over the bank's bf16 copy; the backward
    is one GEMM for the bank's gradient ([dk | dv] @ [Wk; Wv], fp32 out) and one
    for both weights' gradients ([dk | dv]^T @ slots, fp32, into their slots
    when they have them)."""

    @staticmethod
    def forward(ctx, bank, wk, wv, L):
        d = wk.shape[1]
        m16 = _bf16_weights([bank]).view(L, d)
        w16 = _bf16_weights([wk, wv])
        n = wk.shape[0]
        kv = torch.bmm(m16.unsqueeze(0).expand(2, L, d), w16.view(2, n, d).transpose(1, 2))
        ctx.save_for_backward(m16, w16)
        ctx.weights = (wk, wv)
        ctx.bank_shape = bank.shape
        return kv[0], kv[1]

    @staticmethod
    def backward(ctx, dk, dv):
        m16, w16 = ctx.saved_tensors
        wk, wv = ctx.weights
        n = wk.shape[0]
        dkv = _side_by_side(dk.to(torch.bfloat16), dv.to(torch.bfloat16))
        dbank = torch.mm(dkv, w16, out_dtype=torch.float32) if ctx.needs_input_grad[0] else None
        slot = _claim_grad_rows(ctx.weights, m16.shape[1])
        if slot is not None:
            dw = torch.mm(dkv.t(), m16, out_dtype=torch.float32, out=slot)
        else:
            dw = torch.mm(dkv.t(), m16, out_dtype=torch.float32)
        return (None if dbank is None else dbank.view(ctx.bank_shape), dw[:n], dw[n:], None)


def bank_kv(bank, wk, wv, slots: int):
    """The k and v projections of the memory bank under bf16 autocast: bank
    (num_blocks, block_size * d) fp32 viewed as (slots, d); wk, wv (n, d) fp32.
    Returns k, v (slots, n) bf16, contiguous. The bank and the weights are cast
    to bf16 once per update (their bf16 copies, which the package's AdamW
    rewrites); the weight gradients are fp32 from the GEMM."""
    if not bank.is_cuda:
        raise RuntimeError("bank_kv: CUDA tensors only")
    if bank.numel() != slots * wk.shape[1] or wv.shape != wk.shape:
        raise RuntimeError("bank_kv: bank must hold slots x d values and wk, wv be (n, d)")
    return _BankKV.apply(bank, wk, wv, int(slots))


class _CrossEntropySum(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index):
        R, V = logits.shape
        logits = logits.contiguous()
        labels = labels.to(torch.int64).contiguous()
        row_loss = torch.empty(R, dtype=torch.float32, device=logits.device)
        lse = torch.empty(R, dtype=torch.float32, device=logits.device)
        _lib.call("mom_xent_fwd", logits.data_ptr(), labels.data_ptr(), R, V, int(ignore_index),
                  row_loss.data_ptr(), lse.data_ptr(), _stream(logits))
        ctx.save_for_backward(logits, labels, lse)
        ctx.ignore_index = int(ignore_index)
        return row_loss.sum()

    @staticmethod
    def backward(ctx, grad):
        logits, labels, lse = ctx.saved_tensors
        R, V = logits.shape
        g = grad.detach().to(torch.float32).reshape(1).contiguous()
        dlogits = torch.empty_like(logits)
        _lib.call("mom_xent_bwd", logits.data_ptr(), labels.data_ptr(), lse.data_ptr(), g.data_ptr(), R, V,
                  ctx.ignore_index, dlogits.data_ptr(), _stream(logits))
        return dlogits, None, None


def cross_entropy_sum(logits, labels, ignore_index: int = -100):
    """sum over rows of cross_entropy(logits.float(), labels) for bf16 logits
    (R, V) and int labels (R), rows with label == ignore_index counting 0: the
    reference's loss before its division by the count of valid labels, without
    the fp32 copy of the logits. Its gradient is bf16, like the LM head's."""
    _need_bf16(logits)
    if logits.dim() != 2 or labels.shape != logits.shape[:1]:
        raise RuntimeError("cross_entropy_sum: logits (R, V) and labels (R,)")
    return _CrossEntropySum.apply(logits, labels, int(ignore_index))


__all__ = ["rope_qkv", "swiglu", "add_rmsnorm", "cross_entropy_sum", "linear_f32grad", "bank_kv", "register_grad_slot",
           "release_grad_slots", "unregister_grad_slots"]
