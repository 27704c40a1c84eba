"""ORACLE — test infrastructure only.

CPU restatement (numpy + the C prefix scan in ``prefix_scan.c``) of the Naylis
Mixture-of-Memory hot path: the causal router, the gated memory read (forward
and backward) and the full MoM layer around them. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this module, and only as the checker or as the timed CPU baseline —
never as a fallback for the CUDA path.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by the reference itself (``tests/golden/make_golden.py``
imports the reference's ``model.MoMLayer`` and ``mom_kernels.reference`` and
runs them on seeded inputs).

Numerical conventions (each cited against the reference):

* Prefix mean: sequential per-column accumulation, fp64 ("fp64", torch CPU
  semantics) or fp32 ("fp32", torch CUDA outer-dim scan semantics), then one
  IEEE fp32 division — model.py:169-176, mom_kernels/reference.py:32-36.
* Router GEMMs: the inputs are rounded to the compute dtype (``"f32"`` or
  ``"bf16"``, i.e. what torch autocast feeds the linear layers), the dot
  products are accumulated in fp64 and rounded to the compute dtype once —
  model.py:178-187.
* Top-k: value descending, ties broken by the LOWER block index. torch.topk's
  tie order is implementation-defined (the CPU backend follows no index rule,
  measured), so this oracle fixes one rule and the CUDA kernel implements the
  same rule — model.py:216.
* Memory read: fp64 softmax over exactly the selected slots (the reference's
  ``finfo.min`` bias underflows to an exact zero probability elsewhere) —
  mom_kernels/reference.py:14-61, model.py:262-275.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

f32 = np.float32
f64 = np.float64

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def _scan_lib():
    """Load (building on demand) the C restatement of the prefix scan."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.path.join(_HERE, "_build", "liboracle_scan.so")
    if not os.path.exists(path):
        import subprocess
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    lib = ctypes.CDLL(path)
    for fn in (lib.oracle_prefix_mean_f32, lib.oracle_suffix_scaled_sum_f32):
        fn.restype = ctypes.c_int
    lib.oracle_prefix_mean_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int]
    lib.oracle_suffix_scaled_sum_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_int64, ctypes.c_int64,
                                                 ctypes.c_int64]
    _LIB = lib
    return lib


# --------------------------------------------------------------------- dtypes
def bf16_round(a) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returned as fp32.

    Matches torch's float->bfloat16 conversion for finite values.
    """
    a = np.ascontiguousarray(np.asarray(a, dtype=f32))
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(f32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def round_to(a, compute: str) -> np.ndarray:
    """Round to the compute dtype ("f32" or "bf16"), returned as fp32."""
    a32 = np.asarray(a).astype(f32)
    if compute == "f32":
        return a32
    if compute == "bf16":
        return bf16_round(a32)
    raise ValueError(f"unknown compute dtype {compute!r}")


def linear(x, w, compute: str) -> np.ndarray:
    """``nn.Linear`` without bias as autocast runs it: inputs rounded to the
    compute dtype, fp64 accumulation, output rounded to the compute dtype."""
    xq = round_to(x, compute).astype(f64)
    wq = round_to(w, compute).astype(f64)
    return round_to(xq @ wq.T, compute)


# ---------------------------------------------------------------- prefix mean
def prefix_mean(x, mode: str = "fp64") -> np.ndarray:
    """h[b,t,:] = cumsum_{i<=t} x[b,i,:] / (t+1) in fp32 (model.py:169-176)."""
    x32 = np.ascontiguousarray(np.asarray(x, dtype=f32))
    if x32.ndim != 3:
        raise ValueError("prefix_mean expects (B, S, d)")
    B, S, d = x32.shape
    h = np.empty_like(x32)
    m = {"fp64": 0, "fp32": 1}[mode]
    rc = _scan_lib().oracle_prefix_mean_f32(x32.ctypes.data, h.ctypes.data, B, S, d, m)
    if rc != 0:
        raise RuntimeError("oracle_prefix_mean_f32 failed")
    return h


def suffix_scaled_sum(g) -> np.ndarray:
    """u[b,t,:] = sum_{s>=t} g[b,s,:]/(s+1) (adjoint of the prefix mean)."""
    g32 = np.ascontiguousarray(np.asarray(g, dtype=f32))
    B, S, n = g32.shape
    u = np.empty_like(g32)
    rc = _scan_lib().oracle_suffix_scaled_sum_f32(g32.ctypes.data, u.ctypes.data, B, S, n)
    if rc != 0:
        raise RuntimeError("oracle_suffix_scaled_sum_f32 failed")
    return u


# --------------------------------------------------------------------- router
def softmax64(a, axis=-1) -> np.ndarray:
    a = np.asarray(a, dtype=f64)
    m = a.max(axis=axis, keepdims=True)
    e = np.exp(a - m)
    return e / e.sum(axis=axis, keepdims=True)


def _bitonic32_desc(keys):
    """Order of a list of at most 32 keys under a 32-wide Batcher bitonic
    network sorting descending whose compare-exchange also exchanges equal
    keys, unused slots last: how torch's CUDA topk sorts its gathered
    selection. Returns the permutation of positions."""
    P = 32
    key = list(keys) + [None] * (P - len(keys))
    pos_of = list(range(len(keys))) + [-1] * (P - len(keys))

    def cmpx(a, b, direction):
        va, vb = key[a] is not None, key[b] is not None
        swap = (va and vb and key[a] > key[b]) or not vb
        if swap == direction:
            key[a], key[b] = key[b], key[a]
            pos_of[a], pos_of[b] = pos_of[b], pos_of[a]

    size = 2
    while size < P:
        stride = size // 2
        while stride:
            for i in range(P // 2):
                cmpx(2 * i - (i & (stride - 1)), 2 * i - (i & (stride - 1)) + stride, (i & (size // 2)) != 0)
            stride //= 2
        size *= 2
    stride = P // 2
    while stride:
        for i in range(P // 2):
            cmpx(2 * i - (i & (stride - 1)), 2 * i - (i & (stride - 1)) + stride, False)
        stride //= 2
    return pos_of[:len(keys)]


def topk_cuda_order(values, k: int):
    """Top-k along the last axis as torch's CUDA topk returns it (the
    reference's eager router on a GPU, model.py:214): the k largest values,
    the lower indices winning among equal values at the k-th boundary. Without
    equal selected values the order is by value descending. With them, torch
    gathers (values above the k-th, index order) then (values equal to it,
    index order) and sorts that with a 32-wide bitonic network that exchanges
    equal keys; that network is run here (tests/golden/topk_cuda_ties.npz holds
    torch.topk outputs recorded on a B200 that pin this rule). torch's CPU
    topk follows no index rule on ties."""
    v = np.asarray(values).astype(f64)
    chosen = np.argsort(-v, axis=-1, kind="stable")[..., :k].astype(np.int64)
    flat_v = v.reshape(-1, v.shape[-1])
    flat_c = chosen.reshape(-1, k)
    for r in range(flat_c.shape[0]):
        sel = flat_v[r, flat_c[r]]
        if k > 1 and np.any(sel[1:] == sel[:-1]):
            kth = sel[-1]
            cols = np.sort(flat_c[r])
            gathered = [int(c) for c in cols if flat_v[r, c] > kth] + [int(c) for c in cols if flat_v[r, c] == kth]
            perm = _bitonic32_desc([flat_v[r, c] for c in gathered])
            flat_c[r] = [gathered[p] for p in perm]
    chosen = flat_c.reshape(chosen.shape)
    return chosen, np.take_along_axis(np.asarray(values), chosen, axis=-1)


def router_forward(x, w_down, w_up, top_k: int, compute: str = "f32",
                   noise=None, scan_mode: str = "fp64") -> dict:
    """Causal router, model.py:178-220 (the Gumbel draw itself stays with the
    caller: ``noise`` is the already-scaled additive noise, or None)."""
    h = prefix_mean(x, scan_mode)
    hq = round_to(h, compute)
    z = linear(hq, w_down, compute)                    # (B,S,r)
    a = round_to(np.tanh(z.astype(f64)), compute)      # tanh on the rounded z
    logits = linear(a, w_up, compute).astype(f32)      # (B,S,nb), .float()
    probs = softmax64(logits).astype(f32)
    noisy = logits if noise is None else (logits + np.asarray(noise, f32)).astype(f32)
    top_idx, top_vals = topk_cuda_order(noisy, top_k)
    gates = softmax64(top_vals).astype(f32)
    log_gates = np.log(np.maximum(gates.astype(f64), 1e-9)).astype(f32)
    return dict(h=h, hq=hq, z=z, a=a, logits=logits, noisy=noisy, probs=probs,
                top_idx=top_idx, top_vals=top_vals, gates=gates, log_gates=log_gates)


def topk_margin(noisy, k: int) -> np.ndarray:
    """Gap between the k-th and (k+1)-th largest value per row (inf if k == nb)."""
    s = -np.sort(-np.asarray(noisy, f64), axis=-1)
    if s.shape[-1] <= k:
        return np.full(s.shape[:-1], np.inf)
    return s[..., k - 1] - s[..., k]


def router_backward(fwd: dict, x, w_down, w_up, dlog_gates, dprobs=None) -> dict:
    """fp64 adjoint of ``router_forward`` (model.py:186-220 through autograd).

    Returns dx (B,S,d), dw_down (r,d), dw_up (nb,r) and the intermediate
    dlogits. clamp_min(g, 1e-9) passes the gradient where g >= 1e-9.
    """
    g = fwd["gates"].astype(f64)
    dg = np.asarray(dlog_gates, f64) / np.maximum(g, 1e-9) * (g >= 1e-9)
    dtv = g * (dg - (g * dg).sum(-1, keepdims=True))
    nb = fwd["logits"].shape[-1]
    dlogits = np.zeros(fwd["logits"].shape, f64)
    B, S, K = fwd["top_idx"].shape
    bi, si = np.meshgrid(np.arange(B), np.arange(S), indexing="ij")
    for kk in range(K):
        np.add.at(dlogits, (bi, si, fwd["top_idx"][..., kk]), dtv[..., kk])
    if dprobs is not None:
        p = fwd["probs"].astype(f64)
        dp = np.asarray(dprobs, f64)
        dlogits += p * (dp - (p * dp).sum(-1, keepdims=True))
    a = fwd["a"].astype(f64)
    wu = np.asarray(w_up, f64)
    wd = np.asarray(w_down, f64)
    da = dlogits @ wu                                   # (B,S,r)
    dw_up = np.einsum("bse,bsr->er", dlogits, a)
    dz = da * (1.0 - a * a)
    u = suffix_scaled_sum(dz.astype(f32)).astype(f64)   # reverse scan in rank space
    dx = u @ wd                                         # (B,S,d)
    dw_down = np.einsum("bsr,bsc->rc", dz, fwd["hq"].astype(f64))
    assert dlogits.shape[-1] == nb
    return dict(dx=dx, dw_down=dw_down, dw_up=dw_up, dlogits=dlogits, dz=dz, u=u)


# ---------------------------------------------------------------- memory read
def block_bias(top_idx, log_gates, num_blocks: int) -> np.ndarray:
    """(B,S,nb) fp64: sum of log-gates on selected blocks, -inf elsewhere.

    Same values as mom_kernels/reference.py:14-29 (``build_gate_bias``) before
    its repeat over the slots of a block; a block chosen twice gets the sum of
    both log-gates (the reference's one-hot einsum sums them too).
    """
    idx = np.asarray(top_idx)
    lg = np.asarray(log_gates, f64)
    B, S, K = idx.shape
    if idx.min(initial=0) < 0 or idx.max(initial=0) >= num_blocks:
        raise ValueError("top_idx out of range")
    bias = np.zeros((B, S, num_blocks), f64)
    sel = np.zeros((B, S, num_blocks), bool)
    bi, si = np.meshgrid(np.arange(B), np.arange(S), indexing="ij")
    for kk in range(K):
        np.add.at(bias, (bi, si, idx[..., kk]), lg[..., kk])
        sel[bi, si, idx[..., kk]] = True
    bias[~sel] = -np.inf
    return bias


def read_forward(q, k, v, top_idx, log_gates, num_blocks: int, block_size: int,
                 dtype=f64) -> dict:
    """Gated memory read, mom_kernels/reference.py:39-61 with the bias of :14-29.

    q: (B,S,H,hd); k, v: shared (L, H*hd); returns out (B,S,H,hd), the
    per-row log-sum-exp lse (B,H,S) and the probabilities when asked.
    """
    q = np.asarray(q)
    B, S, H, hd = q.shape
    L = k.shape[0]
    assert L == num_blocks * block_size
    scale = 1.0 / math.sqrt(hd)
    kh = np.asarray(k, dtype).reshape(L, H, hd).transpose(1, 0, 2)   # (H,L,hd)
    vh = np.asarray(v, dtype).reshape(L, H, hd).transpose(1, 0, 2)
    bias = np.repeat(block_bias(top_idx, log_gates, num_blocks), block_size, axis=-1)
    out = np.empty((B, S, H, hd), dtype)
    lse = np.empty((B, H, S), dtype)
    for b in range(B):
        qb = np.asarray(q[b], dtype).transpose(1, 0, 2)                # (H,S,hd)
        sc = np.matmul(qb, kh.transpose(0, 2, 1)) * dtype(scale) + bias[b][None].astype(dtype)
        m = sc.max(-1, keepdims=True)
        p = np.exp(sc - m)
        l = p.sum(-1, keepdims=True)
        out[b] = np.matmul(p / l, vh).transpose(1, 0, 2)
        lse[b] = (m + np.log(l))[..., 0]
    return dict(out=out, lse=lse)


def read_backward(q, k, v, top_idx, log_gates, dout, num_blocks: int,
                  block_size: int, dtype=f64) -> dict:
    """fp64 gradients of ``read_forward`` with respect to q, k, v, log_gates.

    Same decomposition as mom_kernels/triton_gpu.py:143-320: P rebuilt from
    the scores, dS = P * (dP - delta), dq = dS k * scale, dk = dS^T q * scale,
    dv = P^T do, and dlog_gates[b,s,t] = sum_h sum_{j in block top[b,s,t]} dS.
    """
    q = np.asarray(q, dtype)
    B, S, H, hd = q.shape
    L = k.shape[0]
    scale = dtype(1.0 / math.sqrt(hd))
    kh = np.asarray(k, dtype).reshape(L, H, hd).transpose(1, 0, 2)
    vh = np.asarray(v, dtype).reshape(L, H, hd).transpose(1, 0, 2)
    bias = np.repeat(block_bias(top_idx, log_gates, num_blocks), block_size, axis=-1).astype(dtype)
    idx = np.asarray(top_idx)
    dq = np.empty((B, S, H, hd), dtype)
    dk = np.zeros((H, L, hd), dtype)
    dv = np.zeros((H, L, hd), dtype)
    dlg = np.zeros(idx.shape, dtype)
    for b in range(B):
        qb = q[b].transpose(1, 0, 2)
        dob = np.asarray(dout[b], dtype).transpose(1, 0, 2)
        sc = np.matmul(qb, kh.transpose(0, 2, 1)) * scale + bias[b][None]
        p = np.exp(sc - sc.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        dp = np.matmul(dob, vh.transpose(0, 2, 1))
        delta = (p * dp).sum(-1, keepdims=True)
        ds = p * (dp - delta)                                           # (H,S,L)
        dq[b] = (np.matmul(ds, kh) * scale).transpose(1, 0, 2)
        dk += np.matmul(ds.transpose(0, 2, 1), qb) * scale
        dv += np.matmul(p.transpose(0, 2, 1), dob)
        dblk = ds.sum(0).reshape(S, num_blocks, block_size).sum(-1)      # (S,nb)
        dlg[b] = np.take_along_axis(dblk, idx[b], axis=-1)
    dk = dk.transpose(1, 0, 2).reshape(L, H * hd)
    dv = dv.transpose(1, 0, 2).reshape(L, H * hd)
    return dict(dq=dq, dk=dk, dv=dv, dlog_gates=dlg)


# ------------------------------------------------------------------ MoM layer
def layer_forward(x, params: dict, n_heads: int, num_blocks: int, block_size: int,
                  top_k: int, compute: str = "f32", noise=None,
                  scan_mode: str = "fp64", read_dtype=f64) -> dict:
    """MoMLayer.forward (model.py:189-276) as autocast runs it in ``compute``.

    params: w_down (r,d), w_up (nb,r), wq/wk/wv/wo (d,d), mom_scale (scalar),
    M_blocks (nb, bs*d).
    """
    x = np.asarray(x, f32)
    B, S, d = x.shape
    hd = d // n_heads
    L = num_blocks * block_size
    rt = router_forward(x, params["w_down"], params["w_up"], top_k, compute, noise, scan_mode)
    q = linear(x, params["wq"], compute).reshape(B, S, n_heads, hd)
    slots = np.asarray(params["M_blocks"], f32).reshape(L, d)
    k = linear(slots, params["wk"], compute)
    v = linear(slots, params["wv"], compute)
    rd = read_forward(q, k, v, rt["top_idx"], rt["log_gates"], num_blocks, block_size, read_dtype)
    r = round_to(rd["out"], compute).reshape(B, S, d)
    o = linear(r, params["wo"], compute)
    out = (f32(params["mom_scale"]) * o).astype(f32)
    return dict(out=out, router=rt, q=q, k=k, v=v, read=rd, r=r, o=o, slots=slots)


def layer_backward(fwd: dict, x, params: dict, dout, n_heads: int, num_blocks: int,
                   block_size: int, dprobs=None, read_dtype=f64) -> dict:
    """fp64 adjoint of ``layer_forward`` (gradients of every parameter and x)."""
    x = np.asarray(x, f64)
    B, S, d = x.shape
    hd = d // n_heads
    dout = np.asarray(dout, f64)
    s = float(params["mom_scale"])
    o = fwd["o"].astype(f64)
    r = fwd["r"].astype(f64)
    d_scale = float((dout * o).sum())
    do_ = dout * s
    dwo = np.einsum("bsi,bsj->ij", do_, r)
    dr = do_ @ np.asarray(params["wo"], f64)
    rb = read_backward(fwd["q"], fwd["k"], fwd["v"], fwd["router"]["top_idx"],
                       fwd["router"]["log_gates"], dr.reshape(B, S, n_heads, hd),
                       num_blocks, block_size, read_dtype)
    dq = rb["dq"].reshape(B, S, d)
    dwq = np.einsum("bsi,bsj->ij", dq, x)
    dx = dq @ np.asarray(params["wq"], f64)
    slots = fwd["slots"].astype(f64)
    dwk = rb["dk"].T @ slots
    dwv = rb["dv"].T @ slots
    dslots = rb["dk"] @ np.asarray(params["wk"], f64) + rb["dv"] @ np.asarray(params["wv"], f64)
    rt = router_backward(fwd["router"], x, params["w_down"], params["w_up"],
                         rb["dlog_gates"], dprobs)
    dx = dx + rt["dx"]
    return dict(dx=dx, dw_down=rt["dw_down"], dw_up=rt["dw_up"], dwq=dwq, dwk=dwk,
                dwv=dwv, dwo=dwo, dmom_scale=d_scale,
                dM_blocks=dslots.reshape(num_blocks, block_size * d),
                read=rb, router=rt)


def scaled_err(a, b) -> float:
    """max|a-b| / max|b| — the reference's parity metric (tests/test_parity.py:64-67)."""
    a = np.asarray(a, f64)
    b = np.asarray(b, f64)
    return float(np.abs(a - b).max()) / max(float(np.abs(b).max()), 1e-6)


# ------------------------------------------------------- timed CPU baseline
def layer_step_fp32(x, params: dict, dout, n_heads: int, num_blocks: int, block_size: int,
                    top_k: int) -> dict:
    """One MoM layer forward + backward in plain fp32 numpy, dense over all L
    slots as the reference's eager path computes it (model.py:189-276 with
    mom_kernels/reference.py:14-61, autograd in fp32). This is the port timed
    as the CPU baseline; the fp64 functions above are the checker."""
    x = np.asarray(x, f32)
    B, S, d = x.shape
    hd = d // n_heads
    L = num_blocks * block_size
    wq, wk, wv, wo = (np.asarray(params[k], f32) for k in ("wq", "wk", "wv", "wo"))
    rt = router_forward(x, params["w_down"], params["w_up"], top_k, "f32")
    q = (x @ wq.T).reshape(B, S, n_heads, hd)
    slots = np.asarray(params["M_blocks"], f32).reshape(L, d)
    k = slots @ wk.T
    v = slots @ wv.T
    rd = read_forward(q, k, v, rt["top_idx"], rt["log_gates"], num_blocks, block_size, f32)
    r = rd["out"].reshape(B, S, d).astype(f32)
    o = r @ wo.T
    s = f32(params["mom_scale"])
    out = s * o
    do_ = np.asarray(dout, f32) * s
    dwo = do_.reshape(-1, d).T @ r.reshape(-1, d)
    dr = do_ @ wo
    rb = read_backward(q, k, v, rt["top_idx"], rt["log_gates"], dr.reshape(B, S, n_heads, hd),
                       num_blocks, block_size, f32)
    dq = rb["dq"].reshape(B, S, d)
    dwq = dq.reshape(-1, d).T @ x.reshape(-1, d)
    dx = dq @ wq
    dwk = rb["dk"].T @ slots
    dwv = rb["dv"].T @ slots
    dslots = rb["dk"] @ wk + rb["dv"] @ wv
    rtb = router_backward(rt, x, params["w_down"], params["w_up"], rb["dlog_gates"])
    dx = dx + rtb["dx"].astype(f32)
    return dict(out=out, dx=dx, dwq=dwq, dwk=dwk, dwv=dwv, dwo=dwo, dM=dslots)
