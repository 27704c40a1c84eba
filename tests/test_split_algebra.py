"""The block-split read's decomposition, checked on the CPU against the oracle.

Top-k routing with more block sets than set bucketing holds is read as one row
per (token, k) pair, each over its one block (naylis_b200/csrc/split.cu):

* forward: per row k the block's softmax with bias log-gate_k gives (out_k, lse_k);
  lse = logsumexp over the token's live rows, a_k = exp(lse_k - lse),
  out = sum_k a_k out_k;
* backward: row k runs the ordinary read backward with dO_k = a_k dO and delta
  taken from the combined output (delta_k = <a_k dO, out>); dq = sum_k dq_k, dk
  and dv accumulate, and the gate gradient of row k is sum_j dS_kj;
* a block a token chose twice is read once with the sum of its log-gates (the
  reference's one-hot bias sums them); the later slots are dead rows (a_k = 0)
  whose gate gradient is their first occurrence's.

This restates those steps in fp64 numpy and requires them to equal the oracle's
dense read (mom_kernels/reference.py:14-61 semantics) to rounding, duplicates
included. The GPU path itself is checked against the oracle in test_gpu_read.py.
"""
import math

import numpy as np

import mom_oracle as O


def _split_read(q, k, v, idx, lg, dout, nb, bs):
    B, S, H, hd = q.shape
    N, top = B * S, idx.shape[-1]
    sc = 1.0 / math.sqrt(hd)
    qn, dn = q.reshape(N, H, hd), dout.reshape(N, H, hd)
    ix, lgn = idx.reshape(N, top), lg.reshape(N, top)
    kh, vh = k.reshape(nb * bs, H, hd), v.reshape(nb * bs, H, hd)
    first = np.tile(np.arange(top), (N, 1))
    dead = np.zeros((N, top), bool)
    for t in range(N):
        for kk in range(top):
            for j in range(kk):
                if ix[t, j] == ix[t, kk]:
                    first[t, kk], dead[t, kk] = j, True
                    break
    lgr = lgn.copy()                      # rows' log-gates: first occurrence carries the sum
    for t in range(N):
        for kk in range(top):
            if not dead[t, kk]:
                lgr[t, kk] = lgn[t, kk] + sum(lgn[t, j] for j in range(kk + 1, top) if first[t, j] == kk)
    out = np.zeros((N, H, hd))
    dq = np.zeros_like(out)
    dk, dv = np.zeros_like(kh), np.zeros_like(vh)
    dlg = np.zeros((N, top))
    for t in range(N):
        for h in range(H):
            lse = np.zeros(top)
            ok = np.zeros((top, hd))
            P = []
            for kk in range(top):
                sl = slice(ix[t, kk] * bs, ix[t, kk] * bs + bs)
                s = kh[sl, h] @ qn[t, h] * sc + lgr[t, kk]
                m = s.max()
                p = np.exp(s - m)
                lse[kk] = m + np.log(p.sum())
                P.append(p / p.sum())
                ok[kk] = P[-1] @ vh[sl, h]
            live = ~dead[t]
            a = np.where(live, np.exp(lse - lse[live].max()), 0.0)
            a /= a.sum()
            o = (a[:, None] * ok).sum(0)
            out[t, h] = o
            for kk in range(top):
                sl = slice(ix[t, kk] * bs, ix[t, kk] * bs + bs)
                g = a[kk] * dn[t, h]
                ds = P[kk] * (vh[sl, h] @ g - g @ o)
                dq[t, h] += ds @ kh[sl, h] * sc
                dk[sl, h] += np.outer(ds, qn[t, h]) * sc
                dv[sl, h] += np.outer(P[kk], g)
                dlg[t, kk] += ds.sum()
    for t in range(N):
        for kk in range(top):
            if dead[t, kk]:
                dlg[t, kk] = dlg[t, first[t, kk]]
    return out.reshape(q.shape), dq.reshape(q.shape), dk.reshape(k.shape), dv.reshape(v.shape), \
        dlg.reshape(idx.shape)


def test_split_decomposition_equals_the_dense_read():
    rng = np.random.default_rng(0)
    B, S, H, hd, nb, bs, top = 1, 40, 2, 16, 6, 8, 4
    q = rng.standard_normal((B, S, H, hd))
    k = rng.standard_normal((nb * bs, H * hd))
    v = rng.standard_normal((nb * bs, H * hd))
    idx = np.argsort(rng.random((B, S, nb)), -1)[..., :top]
    idx[:, ::3, 3] = idx[:, ::3, 0]                       # a block twice
    idx[:, 1::4, 2] = idx[:, 1::4, 0]                     # a block three times
    idx[:, 1::4, 3] = idx[:, 1::4, 0]
    lg = np.log(rng.dirichlet(np.ones(top), (B, S)))
    dout = rng.standard_normal((B, S, H, hd))
    f = O.read_forward(q, k, v, idx, lg, nb, bs)
    b = O.read_backward(q, k, v, idx, lg, dout, nb, bs)
    out, dq, dk, dv, dlg = _split_read(q, k, v, idx, lg, dout, nb, bs)
    for got, ref in ((out, f["out"]), (dq, b["dq"]), (dk, b["dk"]), (dv, b["dv"]), (dlg, b["dlog_gates"])):
        assert np.abs(got - ref).max() <= 1e-12 * max(1.0, np.abs(ref).max())
