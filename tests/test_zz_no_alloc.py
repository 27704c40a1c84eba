"""mom_read_bwd_noalloc: the read backward whose delta scratch is a fixed
device array of the library, for callers that cannot allocate device memory.

The GPU test calls it through the C ABI several times in a row (different
geometries, so each call meets the previous call's leftovers in the shared
scratch, one of them at the largest size the array takes) and checks each
result against mom_read_bwd with a caller workspace:

* dq bit for bit: both entry points run the same MMAs on the same values (the
  no-alloc one only fetches dO rows by gather instead of from a plan-order
  copy), and each dQ tile is summed in one fixed order;
* dk, dv and dlog_gates to a scaled 1e-5: the kernels sum them with fp32
  atomics, whose order changes from run to run (two runs of mom_read_bwd
  differ in the same way);
* on the smallest case also against the oracle's fp64 read backward, within
  the bf16 read tolerance of the other tests (scaled 2e-2).

The file is named to be collected last; it also passes alone in a fresh
process.
"""
import numpy as np
import pytest
import torch

TOL = 2e-2          # bf16 read against the fp64 oracle
ATOMIC_TOL = 1e-5   # the same fp32 sums taken in another order


def _scaled_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _inputs(B, S, H, hd, nb, bs, top, seed, dev):
    g = torch.Generator().manual_seed(seed)
    bf = lambda t: t.to(torch.bfloat16).to(dev)
    q = bf(torch.randn(B, S, H, hd, generator=g) * 0.7)
    k = bf(torch.randn(nb * bs, H * hd, generator=g) * 0.4)
    v = bf(torch.randn(nb * bs, H * hd, generator=g) * 0.4)
    idx = torch.argsort(torch.rand(B, S, nb, generator=g), -1)[..., :top].contiguous().to(dev)
    gates = torch.softmax(torch.randn(B, S, top, generator=g), -1)
    lg = gates.clamp_min(1e-9).log().float().contiguous().to(dev)
    dout = bf(torch.randn(B, S, H, hd, generator=g))
    return q, k, v, idx, lg, dout


def _forward(lib, q, k, v, idx, lg, nb, bs, top, st):
    from naylis_b200 import _lib
    B, S, H, hd = q.shape
    N = B * S
    plan = torch.empty(lib.mom_plan_size(N, nb, top), dtype=torch.uint8, device=q.device)
    _lib.call("mom_bucket", idx.data_ptr(), _lib.I64, lg.data_ptr(), N, nb, top, plan.data_ptr(),
              plan.numel(), st)
    out = torch.empty_like(q)
    lse = torch.empty((H, N), dtype=torch.float32, device=q.device)
    q_rows = torch.empty((N, H * hd), dtype=q.dtype, device=q.device)
    _lib.call("mom_read_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.BF16, B, S, H, hd, nb, bs, top,
              plan.data_ptr(), out.data_ptr(), lse.data_ptr(), q_rows.data_ptr(), st)
    return plan, out, lse, q_rows


def _backward(lib, name, q, k, v, out, dout, lse, plan, q_rows, nb, bs, top, st):
    from naylis_b200 import _lib
    B, S, H, hd = q.shape
    dq = torch.empty_like(q)
    dk = torch.empty((nb * bs, H * hd), dtype=torch.float32, device=q.device)
    dv = torch.empty_like(dk)
    dlg = torch.empty((B * S, top), dtype=torch.float32, device=q.device)
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(), lse.data_ptr(),
            _lib.BF16, B, S, H, hd, nb, bs, top, plan.data_ptr(), q_rows.data_ptr(), dq.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), dlg.data_ptr()]
    if name == "mom_read_bwd":
        ws = torch.empty(lib.mom_read_bwd_workspace_size(B, S, H, hd), dtype=torch.uint8, device=q.device)
        args += [ws.data_ptr(), ws.numel()]
    _lib.call(name, *args, st)
    torch.cuda.synchronize()
    return {"dq": dq.float().cpu().numpy(), "dk": dk.cpu().numpy(), "dv": dv.cpu().numpy(),
            "dlog_gates": dlg.cpu().numpy()}


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """B*S*H above the fixed scratch is refused before any device work."""
    from naylis_b200 import _lib
    lib = _lib.load()
    cap = lib.mom_read_bwd_noalloc_max_bytes()
    assert cap == 4 << 20
    H = 16
    S = cap // 4 // H + 1     # one token more than fits, B = 1
    rc = lib.mom_read_bwd_noalloc(None, None, None, None, None, None, _lib.BF16, 1, S, H, 64, 8, 128, 2,
                                  None, None, None, None, None, None, None)
    assert rc == 4, _lib.last_error()   # MOM_ERR_WORKSPACE
    assert "noalloc" in _lib.last_error()


@pytest.mark.gpu
def test_noalloc_matches_read_bwd_on_consecutive_calls():
    from naylis_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda")
    st = torch.cuda.current_stream().cuda_stream
    cases = [
        dict(B=2, S=512, H=4, hd=64, nb=8, bs=128, top=2, seed=21),
        dict(B=8, S=8192, H=16, hd=64, nb=8, bs=128, top=2, seed=22),   # B*S*H at the scratch limit
        dict(B=1, S=300, H=2, hd=128, nb=8, bs=128, top=2, seed=23),    # ragged S, head_dim 128
        dict(B=1, S=300, H=2, hd=128, nb=8, bs=128, top=1, seed=24),    # head_dim 128 on the tensor cores
    ]
    assert 8 * 8192 * 16 * 4 == lib.mom_read_bwd_noalloc_max_bytes()
    for c in cases:
        c = dict(c)
        seed = c.pop("seed")
        nb, bs, top = c["nb"], c["bs"], c["top"]
        q, k, v, idx, lg, dout = _inputs(**c, seed=seed, dev=dev)
        plan, out, lse, q_rows = _forward(lib, q, k, v, idx, lg, nb, bs, top, st)
        ref = _backward(lib, "mom_read_bwd", q, k, v, out, dout, lse, plan, q_rows, nb, bs, top, st)
        got = _backward(lib, "mom_read_bwd_noalloc", q, k, v, out, dout, lse, plan, q_rows, nb, bs, top, st)
        assert all(np.isfinite(got[key]).all() for key in got)
        assert np.array_equal(got["dq"], ref["dq"]), (c, _scaled_err(got["dq"], ref["dq"]))
        errs = {key: _scaled_err(got[key], ref[key]) for key in ("dk", "dv", "dlog_gates")}
        assert all(e < ATOMIC_TOL for e in errs.values()), (c, errs)
        if seed == 21:
            _check_against_oracle(got, q, k, v, idx, lg, dout, nb, bs)


def _check_against_oracle(got, q, k, v, idx, lg, dout, nb, bs):
    import mom_oracle as O
    f = lambda t: t.float().cpu().numpy()
    ref = O.read_backward(f(q), f(k), f(v), idx.cpu().numpy(), lg.cpu().numpy(), f(dout), nb, bs)
    B, S, H, hd = q.shape
    pairs = {"dq": (got["dq"], ref["dq"]), "dk": (got["dk"], ref["dk"]), "dv": (got["dv"], ref["dv"]),
             "dlog_gates": (got["dlog_gates"].reshape(B, S, -1), ref["dlog_gates"])}
    errs = {k: _scaled_err(a.reshape(b.shape), b) for k, (a, b) in pairs.items()}
    assert all(e < TOL for e in errs.values()), errs
