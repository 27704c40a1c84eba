"""GPU parity of the sm100 gated memory read (forward and backward) through
the C ABI, against the oracle and the reference's golden vectors.

Tolerance: scaled max error (max|a-b| / max|b|) < 2e-2 in bf16, the
reference's own bar (tests/test_parity.py:477-490).
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


def _mk(B, S, H, hd, nb, bs, top, seed, routing="random", dup=False):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, S, H, hd, generator=g) * 0.7)
    k = torch.randn(nb * bs, H * hd, generator=g) * 0.4
    v = torch.randn(nb * bs, H * hd, generator=g) * 0.4
    gates = torch.softmax(torch.randn(B, S, top, generator=g), -1)
    if routing == "random":
        idx = torch.argsort(torch.rand(B, S, nb, generator=g), -1)[..., :top]
    elif routing == "skewed":
        idx = torch.arange(top).expand(B, S, top).clone()
        idx[:, ::7] = torch.argsort(torch.rand(B, S, nb, generator=g), -1)[:, ::7, :top]
    else:
        raise ValueError(routing)
    if dup:
        idx[:, ::3, -1] = idx[:, ::3, 0]
    dout = torch.randn(B, S, H, hd, generator=g)
    bf = lambda t: t.to(torch.bfloat16)
    return bf(q), bf(k), bf(v), idx, gates, bf(dout)


def _run_gpu(q, k, v, idx, gates, dout, nb, bs, split=False):
    from naylis_b200 import mom_kernels as mk
    dev = torch.device("cuda")
    qd, kd, vd = (t.detach().to(dev).requires_grad_(True) for t in (q, k, v))
    gd = gates.detach().to(dev).requires_grad_(True)
    if split:   # the block-split read on a geometry the set bucketing also takes
        lg = gd.clamp_min(1e-9).log().float()
        out = mk._MomReadSplitFunction.apply(qd, kd, vd, idx.to(dev), lg, nb, bs)
    else:
        out = mk.mom_read(qd, kd, vd, idx.to(dev), gd, num_blocks=nb, block_size=bs, mode="sm100")
    out.backward(dout.to(dev))
    torch.cuda.synchronize()
    return {"out": out.detach().float().cpu().numpy(), "dq": qd.grad.float().cpu().numpy(),
            "dk": kd.grad.float().cpu().numpy(), "dv": vd.grad.float().cpu().numpy(),
            "dgates": gd.grad.float().cpu().numpy()}


def _oracle(q, k, v, idx, gates, dout, nb, bs):
    lg = np.log(np.maximum(gates.numpy().astype(np.float64), 1e-9)).astype(np.float32)
    args = (q.float().numpy(), k.float().numpy(), v.float().numpy(), idx.numpy(), lg)
    f = O.read_forward(*args, nb, bs)
    b = O.read_backward(*args, dout.float().numpy(), nb, bs)
    return {"out": f["out"], "dq": b["dq"], "dk": b["dk"], "dv": b["dv"],
            "dgates": b["dlog_gates"] / np.maximum(gates.numpy(), 1e-9)}


def _compare(got, ref, tol=TOL):
    """Scaled error per output. A reference that is identically zero in exact
    arithmetic (the gate gradient of a token that reads a single block: top-1,
    or the same block twice, since its softmax weights sum to one) has no
    scale; there the kernel's value must be below an absolute 1e-4."""
    errs = {}
    for k in ref:
        if float(np.abs(ref[k]).max()) < 1e-9:
            errs[k] = float(np.abs(got[k]).max()) / 1e-4 * tol
        else:
            errs[k] = O.scaled_err(got[k], ref[k])
    bad = {k: e for k, e in errs.items() if not e < tol}
    assert not bad, f"scaled errors over {tol}: {bad} (all: {errs})"
    return errs


def test_read_matches_reference_golden():
    geo = gi.READ
    g = np.load(os.path.join(GOLDEN, "read_bf16.npz"))
    q, k, v, top, gates, dout = gi.read_inputs(geo, "bf16")
    got = _run_gpu(q, k, v, top, gates, dout, geo["nb"], geo["bs"])
    _compare(got, {k_: g[k_] for k_ in ("out", "dq", "dk", "dv", "dgates")})


@pytest.mark.parametrize("case", [
    dict(B=2, S=512, H=4, hd=64, nb=8, bs=128, top=2, seed=1),            # config-2 geometry, fewer tokens
    dict(B=1, S=300, H=2, hd=128, nb=8, bs=128, top=2, seed=2),           # head_dim 128, ragged S
    dict(B=2, S=129, H=2, hd=64, nb=4, bs=64, top=1, seed=3),             # top-1
    dict(B=2, S=200, H=3, hd=64, nb=4, bs=64, top=3, seed=4),             # top-3, odd head count
    dict(B=1, S=257, H=2, hd=64, nb=6, bs=48, top=2, seed=5),             # block not a multiple of 64
    dict(B=2, S=333, H=2, hd=64, nb=8, bs=128, top=2, seed=6, routing="skewed"),  # one dominant set
    dict(B=2, S=150, H=2, hd=64, nb=4, bs=64, top=2, seed=7, dup=True),   # repeated block ids
    dict(B=1, S=300, H=3, hd=128, nb=8, bs=128, top=1, seed=8),           # head_dim 128, top-1 (tensor cores)
])
def test_read_matches_oracle(case):
    case = dict(case)
    routing = case.pop("routing", "random")
    dup = case.pop("dup", False)
    seed = case.pop("seed")
    q, k, v, idx, gates, dout = _mk(**case, seed=seed, routing=routing, dup=dup)
    got = _run_gpu(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    ref = _oracle(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    _compare(got, ref)


@pytest.mark.parametrize("case", [
    dict(B=1, S=300, H=2, hd=128, nb=32, bs=128, top=4, seed=21),          # top-4 of 32 blocks, head_dim 128
    dict(B=2, S=200, H=2, hd=64, nb=32, bs=128, top=4, seed=22),           # tensor-core geometry, split rows
    dict(B=2, S=150, H=3, hd=64, nb=24, bs=64, top=4, seed=23, dup=True),  # repeated block ids
    dict(B=1, S=130, H=2, hd=64, nb=20, bs=48, top=5, seed=24),            # top-5, block not a multiple of 64
])
def test_read_split_matches_oracle(case):
    """Routing with more block sets than the set bucketing holds takes the
    block-split read ((token, k) rows combined by log-sum-exp)."""
    from naylis_b200 import _lib
    case = dict(case)
    dup = case.pop("dup", False)
    seed = case.pop("seed")
    assert _lib.load().mom_plan_size(case["B"] * case["S"], case["nb"], case["top"]) == 0
    q, k, v, idx, gates, dout = _mk(**case, seed=seed, dup=dup)
    if dup:   # a block three times in one token's top list
        idx[:, 1::4, 2] = idx[:, 1::4, 0]
        idx[:, 1::4, 3] = idx[:, 1::4, 0]
    got = _run_gpu(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    ref = _oracle(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    _compare(got, ref)


@pytest.mark.parametrize("case", [
    dict(B=2, S=300, H=4, hd=64, nb=8, bs=128, top=2, seed=31),
    dict(B=1, S=200, H=2, hd=128, nb=8, bs=64, top=3, seed=32, dup=True),
])
def test_read_split_matches_oracle_where_sets_fit(case):
    case = dict(case)
    dup = case.pop("dup", False)
    seed = case.pop("seed")
    q, k, v, idx, gates, dout = _mk(**case, seed=seed, dup=dup)
    got = _run_gpu(q, k, v, idx, gates, dout, case["nb"], case["bs"], split=True)
    ref = _oracle(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    _compare(got, ref)


def _dense_read_fp32(q, k, v, idx, gates, dout, nb, bs):
    """Plain PyTorch fp32 read and gradients on the GPU, one head at a time
    (the same decomposition as the oracle's read_backward)."""
    B, S, H, hd = q.shape
    N, L, top = B * S, k.shape[0], idx.shape[-1]
    scale = hd ** -0.5
    qf = q.reshape(N, H, hd).float()
    kf = k.reshape(L, H, hd).float()
    vf = v.reshape(L, H, hd).float()
    do = dout.reshape(N, H, hd).float()
    lg = gates.reshape(N, top).clamp_min(1e-9).log().float()
    ix = idx.reshape(N, top).long()
    bias = torch.zeros(N, nb, device=q.device).scatter_add_(1, ix, lg)
    sel = torch.zeros(N, nb, dtype=torch.bool, device=q.device).scatter_(1, ix, True)
    bias = bias.masked_fill(~sel, float("-inf")).repeat_interleave(bs, 1)
    out = torch.empty(N, H, hd, device=q.device)
    dq = torch.empty_like(out)
    dk = torch.empty(L, H, hd, device=q.device)
    dv = torch.empty_like(dk)
    dbias = torch.zeros(N, nb, device=q.device)
    for h in range(H):
        p = torch.softmax(qf[:, h] @ kf[:, h].T * scale + bias, -1)
        o = p @ vf[:, h]
        out[:, h] = o
        ds = p * (do[:, h] @ vf[:, h].T - (do[:, h] * o).sum(-1, keepdim=True))
        dq[:, h] = ds @ kf[:, h] * scale
        dk[:, h] = ds.T @ qf[:, h] * scale
        dv[:, h] = p.T @ do[:, h]
        dbias += ds.reshape(N, nb, bs).sum(-1)
    dlg = torch.gather(dbias, 1, ix)
    return {"out": out.reshape(B, S, H, hd), "dq": dq.reshape(B, S, H, hd), "dk": dk.reshape(L, H * hd),
            "dv": dv.reshape(L, H * hd), "dgates": (dlg / gates.reshape(N, top).clamp_min(1e-9)).reshape(B, S, top)}


def test_read_split_full_size_top4_of_32():
    """The top-4-of-32 geometry at full size (4 x 4096 tokens, 16 heads of 128,
    32 blocks of 128 slots) against a plain PyTorch fp32 read on the GPU."""
    B, S, H, hd, nb, bs, top = 4, 4096, 16, 128, 32, 128, 4
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(41)
    q = (torch.randn(B, S, H, hd, generator=g, device=dev) * 0.7).bfloat16()
    k = (torch.randn(nb * bs, H * hd, generator=g, device=dev) * 0.4).bfloat16()
    v = (torch.randn(nb * bs, H * hd, generator=g, device=dev) * 0.4).bfloat16()
    gates = torch.softmax(torch.randn(B, S, top, generator=g, device=dev), -1)
    idx = torch.argsort(torch.rand(B, S, nb, generator=g, device=dev), -1)[..., :top]
    dout = torch.randn(B, S, H, hd, generator=g, device=dev).bfloat16()
    got = _run_gpu(q, k, v, idx, gates, dout, nb, bs)
    with torch.no_grad():
        ref = {key: t.cpu().numpy() for key, t in _dense_read_fp32(q, k, v, idx, gates, dout, nb, bs).items()}
    _compare(got, ref)


def test_bucket_split_flags_out_of_range_index():
    from naylis_b200 import _lib
    dev = torch.device("cuda")
    N, nb, top = 100, 32, 4
    idx = torch.argsort(torch.rand(N, nb, device=dev), -1)[:, :top].contiguous()
    idx[17, 1] = -2   # out of range: must be reported, never read
    lg = torch.zeros(N, top, device=dev)
    plan = torch.empty(_lib.load().mom_plan_split_size(N, nb, top), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("mom_bucket_split", idx.data_ptr(), _lib.I64, lg.data_ptr(), N, nb, top, plan.data_ptr(),
              plan.numel(), st)
    with pytest.raises(_lib.MomError) as ei:
        _lib.call("mom_plan_check", plan.data_ptr(), N * top, nb, 1, st)
    assert ei.value.status == 7


def test_read_is_deterministic_forward_and_dq():
    q, k, v, idx, gates, dout = _mk(2, 256, 2, 64, 8, 128, 2, seed=11)
    a = _run_gpu(q, k, v, idx, gates, dout, 8, 128)
    b = _run_gpu(q, k, v, idx, gates, dout, 8, 128)
    for key in ("out", "dq", "dgates"):
        assert np.array_equal(a[key], b[key]), key


def test_read_empty_batch():
    from naylis_b200 import mom_kernels as mk
    dev = torch.device("cuda")
    q = torch.zeros(0, 16, 2, 64, dtype=torch.bfloat16, device=dev, requires_grad=True)
    k = torch.randn(256, 128, dtype=torch.bfloat16, device=dev, requires_grad=True)
    v = torch.randn(256, 128, dtype=torch.bfloat16, device=dev, requires_grad=True)
    idx = torch.zeros(0, 16, 2, dtype=torch.int64, device=dev)
    g = torch.full((0, 16, 2), 0.5, device=dev, requires_grad=True)
    out = mk.mom_read(q, k, v, idx, g, num_blocks=4, block_size=64)
    assert out.shape == q.shape
    out.sum().backward()
    assert float(k.grad.abs().sum()) == 0.0


def test_bucket_flags_out_of_range_index():
    from naylis_b200 import _lib
    dev = torch.device("cuda")
    N, nb, top = 100, 4, 2
    idx = torch.randint(0, nb, (N, top), dtype=torch.int64, device=dev)
    idx[17, 1] = nb + 3   # out of range: must be reported, never read
    lg = torch.zeros(N, top, device=dev)
    plan = torch.empty(_lib.load().mom_plan_size(N, nb, top), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("mom_bucket", idx.data_ptr(), _lib.I64, lg.data_ptr(), N, nb, top, plan.data_ptr(),
              plan.numel(), st)
    with pytest.raises(_lib.MomError) as ei:
        _lib.call("mom_plan_check", plan.data_ptr(), N, nb, top, st)
    assert ei.value.status == 7


def test_read_rejects_contract_violations():
    from naylis_b200 import mom_kernels as mk
    dev = torch.device("cuda")
    q = torch.randn(1, 8, 2, 64, device=dev)                     # fp32: rejected
    k = torch.randn(256, 128, device=dev, dtype=torch.bfloat16)
    idx = torch.zeros(1, 8, 2, dtype=torch.int64, device=dev)
    g = torch.full((1, 8, 2), 0.5, device=dev)
    with pytest.raises(RuntimeError):
        mk.mom_read(q, k, k, idx, g, num_blocks=4, block_size=64)
    with pytest.raises(RuntimeError):
        mk.mom_read(q.bfloat16(), k, k, idx, g, num_blocks=3, block_size=64)   # L mismatch
    with pytest.raises(RuntimeError):
        mk.mom_read(q.bfloat16(), k.unsqueeze(0), k.unsqueeze(0), idx, g, num_blocks=4, block_size=64)


# ---------------------------------------------------------------------- fp32 read
TOL_F32 = 1e-5     # the reference's fp32 bar (tests/test_parity.py:138-188)


def _to_f32(*ts):
    return tuple(t.float() for t in ts)


def test_read_f32_matches_reference_golden():
    """fp32 q, k, v through the door take the fp32 read; against what the
    reference's own build_gate_bias + SDPA read gave in fp32."""
    geo = gi.READ
    g = np.load(os.path.join(GOLDEN, "read_f32.npz"))
    q, k, v, top, gates, dout = gi.read_inputs(geo, "f32")
    got = _run_gpu(q, k, v, top, gates, dout, geo["nb"], geo["bs"])
    _compare(got, {k_: g[k_] for k_ in ("out", "dq", "dk", "dv", "dgates")}, tol=TOL_F32)


@pytest.mark.parametrize("case", [
    dict(B=2, S=300, H=4, hd=64, nb=8, bs=128, top=2, seed=51),            # config-2 geometry
    dict(B=1, S=200, H=2, hd=128, nb=8, bs=128, top=2, seed=52),           # head_dim 128
    dict(B=2, S=129, H=2, hd=64, nb=4, bs=64, top=1, seed=53),             # top-1
    dict(B=1, S=157, H=3, hd=64, nb=6, bs=48, top=3, seed=54, dup=True),   # top-3, block 48, repeated ids
    dict(B=1, S=130, H=2, hd=128, nb=32, bs=128, top=4, seed=55),          # top-4 of 32
])
def test_read_f32_matches_oracle(case):
    case = dict(case)
    dup = case.pop("dup", False)
    seed = case.pop("seed")
    q, k, v, idx, gates, dout = _mk(**case, seed=seed, dup=dup)
    g = torch.Generator().manual_seed(seed + 100)      # fp32 values, not bf16-rounded ones
    q = q.float() + 1e-3 * torch.randn(q.shape, generator=g)
    k, v, dout = _to_f32(k, v, dout)
    got = _run_gpu(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    assert got["out"].dtype == np.float32
    ref = _oracle(q, k, v, idx, gates, dout, case["nb"], case["bs"])
    _compare(got, ref, tol=TOL_F32)
