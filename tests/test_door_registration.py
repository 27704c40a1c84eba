"""naylis_b200.door.register: the sm100 backend behind the reference's own
mom_kernels door, with the reference's model.py unchanged (CPU, where the
reference checkout is importable; the reference does not travel to GPU boxes,
so the kernels themselves are checked against its golden vectors there).

* With a CPU test double registered as the "sm100" backend, the reference's
  MoMLayer(use_kernel=True) resolves through the door once, calls mom_read
  with the reference's tensor contract (q_sh (B,S,H,hd), shared k/v (L,d),
  int64 top_idx, fp32 top_gates that carry the gradient), and its output
  equals the reference's eager layer bit for bit (gradients to 1e-6) when the
  double computes the read with the reference's own math; a 2-layer
  NaylisLlamaForCausalLM does the same per layer.
* With the real backend registered, requests it takes fail loudly without a
  GPU, requests it does not take reach the reference's own branches, and
  unregister() restores the reference's functions.
"""
import importlib
import os
import sys

import pytest
import torch

REF = os.environ.get("NAYLIS_REFERENCE", "/root/reference")
pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REF, "model.py")),
                                reason="reference checkout not importable here")


@pytest.fixture()
def reference():
    sys.path.insert(0, REF)
    try:
        mk = importlib.import_module("mom_kernels")
        model = importlib.import_module("model")
        yield mk, model
    finally:
        sys.path.remove(REF)


class _Double:
    """Stands in for naylis_b200.mom_kernels on the CPU: records every call and
    computes the read with the reference's own eager math."""
    MODE = "sm100"

    def __init__(self, ref_mk):
        self.ref = ref_mk.reference
        self.calls = []

    def preflight(self, device_type):
        self.calls.append(("preflight", device_type))

    def resolve_mode(self, device, dtype, *, head_dim=None):
        self.calls.append(("resolve", str(device), dtype, head_dim))
        return self.MODE

    def announce(self, name):
        self.calls.append(("announce", name))

    def mom_read(self, q_sh, k, v, top_idx, top_gates, *, num_blocks, block_size, mode):
        self.calls.append(("read", tuple(q_sh.shape), tuple(k.shape), top_idx.dtype, tuple(top_idx.shape),
                           top_gates.dtype, top_gates.requires_grad, num_blocks, block_size, mode))
        bias = self.ref.build_gate_bias(top_idx, top_gates, num_blocks, block_size, q_sh.dtype)
        return self.ref.mom_attention_reference(q_sh, k, v, bias)


def _pair(model_mod, **kw):
    torch.manual_seed(3)
    args = dict(d_model=128, n_heads=2, mem_size=256, block_size=64, top_blocks=2, router_rank=8)
    eager = model_mod.MoMLayer(**args, use_kernel=False)
    with torch.no_grad():
        eager.mom_scale.fill_(0.7)
    door_layer = model_mod.MoMLayer(**args, use_kernel=True)
    door_layer.load_state_dict(eager.state_dict())
    for m in (eager, door_layer):
        m.train()
        m.noise_scale = 0.0
    return eager, door_layer


def test_reference_layer_reads_through_the_registered_door(reference):
    from naylis_b200 import door
    mk, model_mod = reference
    orig = {n: getattr(mk, n) for n in ("preflight", "resolve_mode", "mom_read", "announce")}
    dbl = _Double(mk)
    door.register(mk, backend=dbl, select=lambda: True, device_types=("cpu",))
    try:
        eager, via_door = _pair(model_mod)
        torch.manual_seed(0)
        x = torch.randn(2, 96, 128)
        M = torch.randn(4, 64 * 128) * 0.5
        outs, grads = [], []
        for layer in (eager, via_door):
            xi = x.clone().requires_grad_(True)
            Mi = M.clone().requires_grad_(True)
            for _ in range(2):                          # the mode is resolved once, then cached
                out = layer(xi, Mi)
            out.square().sum().backward()
            outs.append(out.detach())
            grads.append([xi.grad, Mi.grad] + [p.grad for p in layer.parameters()])
        assert torch.equal(outs[0], outs[1])
        # the eager layer expands k/v over the batch, the reference's read helper
        # broadcasts them: the same gradients summed in another order
        for a, b in zip(*grads):
            assert torch.allclose(a, b, rtol=1e-6, atol=1e-6 * float(b.abs().max())), float((a - b).abs().max())
        resolves = [c for c in dbl.calls if c[0] == "resolve"]
        reads = [c for c in dbl.calls if c[0] == "read"]
        assert resolves == [("resolve", "cpu", torch.float32, 64)]
        assert len(reads) == 2
        assert reads[0] == ("read", (2, 96, 2, 64), (256, 128), torch.int64, (2, 96, 2), torch.float32, True,
                            4, 64, "sm100")
        assert ("announce", "sm100") in dbl.calls
    finally:
        door.unregister(mk)
    assert all(getattr(mk, n) is f for n, f in orig.items())


def test_reference_decoder_reads_through_the_registered_door(reference):
    from transformers import LlamaConfig
    from naylis_b200 import door
    mk, model_mod = reference
    dbl = _Double(mk)
    door.register(mk, backend=dbl, select=lambda: True, device_types=("cpu",))
    try:
        cfg = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                          num_attention_heads=2, num_key_value_heads=2, tie_word_embeddings=True,
                          attn_implementation="sdpa", use_cache=False)
        losses = []
        for use_kernel in (False, True):
            torch.manual_seed(5)
            m = model_mod.NaylisLlamaForCausalLM(cfg, mem_size=256, mom_block_size=64, mom_top_blocks=2,
                                                 mom_router_rank=8, mom_aux_weight=0.01, use_kernel=use_kernel)
            for layer in m.modules():
                if isinstance(layer, model_mod.MoMLayer):
                    layer.noise_scale = 0.0
                    with torch.no_grad():
                        layer.mom_scale.fill_(0.5)
            m.train()
            ids = torch.randint(0, 64, (2, 48), generator=torch.Generator().manual_seed(9))
            losses.append(m(input_ids=ids, labels=ids).loss)
        assert torch.equal(losses[0], losses[1])
        assert len([c for c in dbl.calls if c[0] == "read"]) == 2      # one per layer
    finally:
        door.unregister(mk)


def test_registered_door_fails_loud_and_defers_the_rest(reference, monkeypatch):
    from naylis_b200 import door
    mk, _ = reference
    orig_resolve = mk.resolve_mode
    door.register(mk)                                   # the real backend, CUDA only
    try:
        monkeypatch.setenv("NAYLIS_KERNEL", "sm100")
        if not torch.cuda.is_available():
            with pytest.raises(RuntimeError):
                mk.preflight("cuda")
            with pytest.raises(RuntimeError):
                mk.resolve_mode("cuda", torch.bfloat16, head_dim=64)
        # device types the backend does not take reach the reference's own branch
        with pytest.raises(RuntimeError) as e:
            mk.resolve_mode("cpu", torch.float32, head_dim=64)
        with pytest.raises(RuntimeError) as e_ref:
            orig_resolve("cpu", torch.float32, head_dim=64)
        assert str(e.value) == str(e_ref.value)
        with pytest.raises(RuntimeError, match="unknown kernel mode"):
            mk.mom_read(None, None, None, None, None, num_blocks=1, block_size=1, mode="nope")
        # without the selection, CUDA requests are the reference's as well
        monkeypatch.setenv("NAYLIS_KERNEL", "")
        want = None
        try:
            want = orig_resolve("cuda", torch.bfloat16, head_dim=64)
        except RuntimeError as err:
            want = str(err)
        try:
            got = mk.resolve_mode("cuda", torch.bfloat16, head_dim=64)
        except RuntimeError as err:
            got = str(err)
        assert got == want
    finally:
        door.unregister(mk)
    assert mk.resolve_mode is orig_resolve
