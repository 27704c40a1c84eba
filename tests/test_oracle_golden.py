"""Pin the oracle to the reference: every oracle function against the golden
vectors that ``tests/golden/make_golden.py`` produced by running the
reference's own ``model.MoMLayer`` / ``mom_kernels.reference`` code.

Tolerances follow the reference's parity suite: bitwise for the prefix mean
and the top-k indices, 1e-5 (scaled) in fp32 and 2e-2 (scaled) in bf16
(tests/test_parity.py:101-188, 460-490).
"""
import hashlib
import os

import numpy as np
import pytest

import golden_inputs as gi
import mom_oracle as O
from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def test_cfg1_forward_matches_reference():
    geo = gi.CFG1
    g = _load("cfg1_fwd")
    inp = gi.layer_inputs(geo)
    assert gi.input_digest(inp) == str(g["input_sha"]), "seeded input generator drifted"
    P = gi.oracle_params(inp, geo)
    f = O.layer_forward(inp["x"].numpy(), P, geo["H"], geo["nb"], geo["bs"], geo["top"], "f32")
    rt = f["router"]
    # prefix mean: bitwise (fp32 cumsum semantics of the CPU reference)
    assert _sha(rt["h"]) == str(g["h_sha"])
    # router: indices bitwise, probabilities/gates at fp32 rounding level
    assert np.array_equal(rt["top_idx"], g["top_idx"])
    assert O.scaled_err(rt["logits"], g["logits"]) < 1e-5
    assert O.scaled_err(rt["probs"], g["probs"]) < 1e-5
    assert O.scaled_err(rt["gates"], g["gates"]) < 1e-5
    # layer output, 4096-element subsample
    assert O.scaled_err(f["out"].reshape(-1)[g["out_sub_idx"]], g["out_sub"]) < 1e-5
    assert O.scaled_err(rt["h"].reshape(-1)[g["out_sub_idx"]], g["h_sub"]) == 0.0


@pytest.mark.parametrize("case,geo,compute,tol", [
    ("small_f32", gi.SMALL_F32, "f32", 1e-5),
    ("small_bf16", gi.SMALL_BF16, "bf16", 2e-2),
])
def test_layer_forward_backward_matches_reference(case, geo, compute, tol):
    g = _load(case)
    inp = gi.layer_inputs(geo)
    assert gi.input_digest(inp) == str(g["input_sha"])
    P = gi.oracle_params(inp, geo)
    f = O.layer_forward(inp["x"].numpy(), P, geo["H"], geo["nb"], geo["bs"], geo["top"], compute)
    assert np.array_equal(f["router"]["top_idx"], g["top_idx"])
    if compute == "bf16":
        # bf16 logits are bit-exact: the rounding to bf16 absorbs the
        # accumulation-order difference of the rank-r GEMMs
        assert np.array_equal(f["router"]["logits"], g["logits"])
    assert O.scaled_err(f["router"]["logits"], g["logits"]) < tol
    assert O.scaled_err(f["router"]["probs"], g["probs"]) < tol
    assert O.scaled_err(f["out"], g["out"]) < tol
    dout = gi.upstream_grad(geo).numpy()
    b = O.layer_backward(f, inp["x"].numpy(), P, dout, geo["H"], geo["nb"], geo["bs"])
    pairs = [("dx", "dx"), ("dM_blocks", "dM_blocks"), ("dw_down", "d_router_down"),
             ("dw_up", "d_router_up"), ("dwq", "d_q_proj"), ("dwk", "d_k_proj"),
             ("dwv", "d_v_proj"), ("dwo", "d_o_proj")]
    for ko, kg in pairs:
        err = O.scaled_err(b[ko], g[kg])
        assert err < tol, f"{ko}: scaled error {err:.2e} >= {tol}"
    assert abs(b["dmom_scale"] - float(g["d_mom_scale"][0])) <= tol * abs(float(g["d_mom_scale"][0]))


@pytest.mark.parametrize("dtype_name,tol", [("f32", 1e-5), ("bf16", 2e-2)])
def test_read_forward_backward_matches_reference(dtype_name, tol):
    geo = gi.READ
    g = _load(f"read_{dtype_name}")
    q, k, v, top, gates, dout = gi.read_inputs(geo, dtype_name)
    assert np.array_equal(top.numpy(), g["top_idx"])
    lg = np.log(np.maximum(gates.numpy().astype(np.float64), 1e-9)).astype(np.float32)
    args = (q.float().numpy(), k.float().numpy(), v.float().numpy(), top.numpy(), lg)
    f = O.read_forward(*args, geo["nb"], geo["bs"])
    b = O.read_backward(*args, dout.float().numpy(), geo["nb"], geo["bs"])
    dgates = b["dlog_gates"] / np.maximum(gates.numpy(), 1e-9)
    assert O.scaled_err(f["out"], g["out"]) < tol
    assert O.scaled_err(b["dq"], g["dq"]) < tol
    assert O.scaled_err(b["dk"], g["dk"]) < tol
    assert O.scaled_err(b["dv"], g["dv"]) < tol
    assert O.scaled_err(dgates, g["dgates"]) < tol


@pytest.mark.parametrize("dtype_name", ["f32", "bf16"])
def test_prefix_mean_bitwise(dtype_name):
    g = _load("scan")
    x = gi.scan_input(dtype_name).float().numpy()
    h = O.prefix_mean(x, "fp64")
    assert _sha(h) == str(g[f"h_sha_{dtype_name}"])
    # causality: perturbing the future leaves every past row bit-identical
    x2 = x.copy()
    x2[:, 512:] += 1.0
    h2 = O.prefix_mean(x2, "fp64")
    assert np.array_equal(h[:, :512], h2[:, :512])
    assert np.array_equal(h[:, 0], x[:, 0])


def test_prefix_mean_fp32_mode_is_sequential_float():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 300, 16)).astype(np.float32)
    h = O.prefix_mean(x, "fp32")
    acc = np.zeros((2, 16), np.float32)
    for t in range(300):
        acc = (acc + x[:, t]).astype(np.float32)
        assert np.array_equal(h[:, t], acc / np.float32(t + 1))


def test_suffix_scaled_sum_is_adjoint_of_prefix_mean():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 50, 3)).astype(np.float32)
    g = rng.standard_normal((2, 50, 3)).astype(np.float32)
    lhs = float((O.prefix_mean(x).astype(np.float64) * g).sum())
    rhs = float((x.astype(np.float64) * O.suffix_scaled_sum(g)).sum())
    assert abs(lhs - rhs) < 1e-4 * max(1.0, abs(lhs))


def test_topk_rule_matches_torch_cuda_on_ties():
    """The oracle's tie rule is torch's CUDA topk as measured on B200 (the
    rows below are cases recorded there): lower indices win at the k-th
    boundary, equal values are listed by descending index."""
    v = np.array([[0.5, 1.0, 1.0, 1.0, 0.2, 1.0, 0.1, 0.0],
                  [0.5, 1.0, 0.7, 0.7, 0.2, 0.7, 0.1, 0.0],
                  [2, 3, 2, 3, 3, 2, 3, 1],
                  [1, 2, 3, 2, 1, 3, 2, 2]], np.float32)
    idx, vals = O.topk_cuda_order(v, 2)
    assert idx.tolist() == [[2, 1], [1, 2], [3, 1], [5, 2]]
    assert vals.tolist() == [[1.0, 1.0], [1.0, np.float32(0.7)], [3, 3], [3, 3]]
    v3 = np.array([[2, 3, 3, 2, 2, 2, 1, 2], [1, 3, 2, 2, 2, 2, 2, 3], [3, 1, 2, 2, 3, 2, 1, 3]], np.float32)
    assert O.topk_cuda_order(v3, 3)[0].tolist() == [[2, 1, 0], [7, 1, 2], [7, 4, 0]]


def test_topk_rule_reproduces_recorded_torch_cuda_topk():
    """torch.topk outputs recorded on a B200 (tests/golden/make_topk_ties.py)
    over tie-heavy inputs, 8 / 16 / 32 columns, k = 1..8: the oracle's rule
    gives the same indices in the same order on every row."""
    path = os.path.join(GOLDEN, "topk_cuda_ties.npz")
    if not os.path.exists(path):
        pytest.skip("topk_cuda_ties.npz not recorded yet")
    g = np.load(path)
    rows = 0
    for key in g.files:
        if not key.startswith("v_"):
            continue
        v = g[key].astype(np.float32)
        want = g[key.replace("v_", "i_")].astype(np.int64)
        got = O.topk_cuda_order(v, want.shape[1])[0]
        assert np.array_equal(got, want), key
        rows += v.shape[0]
    assert rows >= 6000


def test_bf16_round_matches_torch():
    import torch
    rng = np.random.default_rng(3)
    a = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    ref = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16_round(a), ref)


def test_decoder_oracle_matches_reference_fp32():
    """oracle/decoder_oracle.py (the CPU restatement of the reference's decoder
    training forward) against the reference's own NaylisLlamaForCausalLM in
    fp32: loss to 1e-5 relative, gradients and logits to 1e-4 of their largest
    magnitude, every layer's routing equal."""
    import torch
    import decoder_oracle as D
    g = _load("decoder_small_f32")
    geo = dict(gi.DECODER)
    sd = gi.decoder_state(geo)
    assert gi.state_digest(sd) == str(g["state_sha"])
    p = {k: v.clone().requires_grad_(True) for k, v in sd.items() if k != "lm_head.weight"}
    ids = gi.decoder_tokens(geo)
    loss, stats = D.forward(ids, p, geo, labels=ids)
    loss.backward()
    assert abs(float(loss) - float(g["loss"])) <= 1e-5 * abs(float(g["loss"]))
    routing = np.stack([idx.numpy() for _, idx in stats])
    assert np.array_equal(routing.reshape(g["routing"].shape), g["routing"].astype(np.int64))
    for name, t in p.items():
        got = t.grad.reshape(-1).numpy()[g["g_" + name + "_idx"]]
        err = np.abs(got - g["g_" + name]).max() / max(float(g["g_" + name + "_absmax"]), 1e-30)
        assert err < 1e-4, (name, err)
    with torch.no_grad():
        logits, _ = D.forward(ids, p, geo)
    got = logits.reshape(-1).numpy()[g["logits_idx"]]
    assert np.abs(got - g["logits"]).max() / g["logits_absmax"] < 1e-4
