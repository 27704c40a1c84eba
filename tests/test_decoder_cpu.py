"""CPU checks of the decoder that drives the MoM kernels (no GPU work): its
parameter names and shapes are the reference's NaylisLlamaForCausalLM's, its
size and FLOP count at BASELINE config 3 are the ones the measurement uses."""
import importlib
import os
import sys

import pytest

import golden_inputs as gi


def test_parameter_names_and_shapes_are_the_references():
    from naylis_b200.decoder import NaylisConfig, NaylisForCausalLM
    geo = gi.DECODER
    cfg = NaylisConfig(vocab_size=geo["vocab"], hidden_size=geo["d"], intermediate_size=geo["ffn"],
                       num_hidden_layers=geo["layers"], num_attention_heads=geo["H"],
                       mem_size=geo["nb"] * geo["bs"], mom_block_size=geo["bs"], mom_top_blocks=geo["top"],
                       mom_router_rank=geo["r"])
    ours = {k: tuple(v.shape) for k, v in NaylisForCausalLM(cfg).state_dict().items()}
    want = {k: tuple(s) for k, s in gi.decoder_param_shapes(geo)}
    want["lm_head.weight"] = want["model.embed_tokens.weight"]
    assert ours == want
    ref_root = os.environ.get("NAYLIS_REFERENCE", "/root/reference")
    if not os.path.exists(os.path.join(ref_root, "model.py")):
        pytest.skip("reference checkout not importable here")
    from transformers import LlamaConfig
    sys.path.insert(0, ref_root)
    try:
        ref_model = importlib.import_module("model")
    finally:
        sys.path.remove(ref_root)
    lc = LlamaConfig(vocab_size=geo["vocab"], hidden_size=geo["d"], intermediate_size=geo["ffn"],
                     num_hidden_layers=geo["layers"], num_attention_heads=geo["H"], num_key_value_heads=geo["H"],
                     tie_word_embeddings=True)
    ref = ref_model.NaylisLlamaForCausalLM(lc, mem_size=geo["nb"] * geo["bs"], mom_block_size=geo["bs"],
                                           mom_top_blocks=geo["top"], mom_router_rank=geo["r"], mom_aux_weight=0.01)
    assert {k: tuple(v.shape) for k, v in ref.state_dict().items()} == ours


def test_config3_size_and_flops():
    from naylis_b200.decoder import NaylisConfig, NaylisForCausalLM, flops_per_token, param_count
    cfg = NaylisConfig()
    assert abs(param_count(NaylisForCausalLM(cfg)) - 375.33e6) < 0.01e6
    # 20 layers x 35.46 MFLOP + the 65.5 MFLOP head per token forward; x3 per training token
    assert abs(3 * flops_per_token(cfg, 2048, 16384) - 2.324e9) < 0.001e9


def test_bf16_weight_buffer_is_reused_until_a_weight_changes():
    """The bf16 projections keep one bf16 buffer per group of weights (q/k/v,
    gate/up, ...): reused while no weight changed, rewritten after an in-place
    update (the version counter), and shared by the group's rows."""
    import torch
    from naylis_b200 import trunk
    w = torch.nn.Parameter(torch.randn(4, 3))
    w2 = torch.nn.Parameter(torch.randn(2, 3))
    b = trunk._bf16_weights([w, w2])
    assert b.shape == (6, 3) and torch.equal(b, torch.cat([w, w2]).detach().bfloat16())
    assert trunk.bf16_copy(w).data_ptr() == b.data_ptr()
    assert trunk._bf16_weights([w, w2]) is b
    with torch.no_grad():
        w2.mul_(2)
    b2 = trunk._bf16_weights([w, w2])
    assert b2 is b and torch.equal(b2[4:], w2.detach().bfloat16())


def test_optimizer_table_layout():
    """The one-launch AdamW's device table: 48-byte entries of five 64-bit
    addresses and an int64 count, in the order csrc/launch.h's OptTensor
    declares them."""
    import struct
    from naylis_b200.optim import _pack_entries
    raw = _pack_entries([(1, 2, 3, 4, 0, 70000), (0x7FFF00001000, 6, 7, 8, 9, 5)])
    assert len(raw) == 96
    assert struct.unpack("<5Qq", raw[:48]) == (1, 2, 3, 4, 0, 70000)
    assert struct.unpack("<5Qq", raw[48:]) == (0x7FFF00001000, 6, 7, 8, 9, 5)


def test_gradient_buckets_keep_fused_projection_groups_contiguous():
    """GradAllReduce lays the decoder's q/k/v and gate/up weights next to each
    other in one bucket in the fused GEMM's row order, starts every parameter on
    a 16-byte boundary (the GEMMs writing there need it), registers every slot, and
    zero_grad clears the gradients to None; finish() gives a parameter that got
    no gradient its zero-filled slot."""
    import torch
    from naylis_b200 import trunk
    from naylis_b200.data_parallel import GradAllReduce
    from naylis_b200.decoder import NaylisConfig, NaylisForCausalLM
    cfg = NaylisConfig(vocab_size=64, hidden_size=32, intermediate_size=48, num_hidden_layers=2,
                       num_attention_heads=2, mem_size=32, mom_block_size=8, mom_top_blocks=2, mom_router_rank=4)
    model = NaylisForCausalLM(cfg)
    dp = GradAllReduce(model, bucket_mb=0.01)
    try:
        assert len(dp.buckets) > 2
        for g in model.grad_groups():
            ents = [trunk._GRAD_SLOTS[w] for w in g]
            assert all(e[0] is ents[0][0] for e in ents)
            offs = [e[1] for e in ents]
            assert offs == [offs[0] + sum(w.numel() for w in g[:i]) for i in range(len(g))]
        # every unit starts on a 16-byte boundary (mom_scale holds one value)
        assert all(trunk._GRAD_SLOTS[g[0]][1] % 4 == 0 for g in model.grad_groups())
        assert all(trunk._GRAD_SLOTS[p][1] % 4 == 0 for p in model.parameters())
        total = sum(p.numel() for p in model.parameters())
        assert total <= sum(b.numel() for b in dp.flat) <= total + 3 * len(list(model.parameters()))
        dp.zero_grad()
        assert all(p.grad is None for p in model.parameters())
        dp.finish()
        assert all(p.grad is not None and not p.grad.any() for p in model.parameters())
    finally:
        dp.remove()
    assert all(w not in trunk._GRAD_SLOTS for w in model.parameters())


def test_gradient_slot_claims():
    """A fused GEMM may write a group's gradients into their slots only when the
    slots follow each other in order, no weight has a gradient yet and no other
    GEMM of this backward claimed them; release re-arms them."""
    import torch
    from naylis_b200 import trunk
    flat = torch.zeros(40)
    a, b, c = (torch.nn.Parameter(torch.randn(2, 4)) for _ in range(3))
    trunk.register_grad_slot(a, flat, 0)
    trunk.register_grad_slot(b, flat, 8)
    trunk.register_grad_slot(c, flat, 24)
    try:
        assert trunk._claim_grad_rows([b, a], 4) is None          # out of order
        assert trunk._claim_grad_rows([a, c], 4) is None          # not adjacent
        rows = trunk._claim_grad_rows([a, b], 4)
        assert rows.shape == (4, 4) and rows.data_ptr() == flat.data_ptr()
        assert trunk._claim_grad_rows([a, b], 4) is None          # claimed in this backward
        c.grad = torch.zeros(2, 4)
        assert trunk._claim_grad_rows([c], 4) is None             # already has a gradient
        trunk.release_grad_slots([a, b, c])
        c.grad = None
        assert trunk._claim_grad_rows([c], 4).data_ptr() == flat[24:].data_ptr()
        assert trunk._claim_grad_rows([a, b], 4) is not None
    finally:
        trunk.unregister_grad_slots([a, b, c])


def test_side_by_side_views_and_copies():
    """The bank projection's backward reads [dK | dV] as one (L, 2n) operand: a
    view when the read's backward returned the two halves of one buffer, a copy
    otherwise."""
    import torch
    from naylis_b200 import trunk
    both = torch.randn(5, 8)
    a, b = both[:, :4], both[:, 4:]
    v = trunk._side_by_side(a, b)
    assert v.data_ptr() == both.data_ptr() and torch.equal(v, both)
    a2, b2 = torch.randn(5, 4), torch.randn(5, 4)
    c = trunk._side_by_side(a2, b2)
    assert torch.equal(c, torch.cat([a2, b2], 1))
    assert torch.equal(trunk._side_by_side(b, a), torch.cat([b, a], 1))


def test_graphed_step_refuses_what_it_cannot_capture():
    """GraphedTrainStep takes CUDA token ids only, and on more than one process a
    GradAllReduce whose hooks launch no collective (overlap=False): a capture
    cannot hold the hooks' all-reduces."""
    import types
    import pytest
    import torch
    from naylis_b200.graph_step import GraphedTrainStep
    with pytest.raises(RuntimeError, match="CUDA"):
        GraphedTrainStep(None, types.SimpleNamespace(world=1, overlap=True), torch.zeros(1, 4, dtype=torch.long))
    meta = torch.zeros(1, 4, dtype=torch.long, device="meta")
    meta_cuda = types.SimpleNamespace(is_cuda=True, device=meta.device)
    with pytest.raises(RuntimeError, match="overlap=False"):
        GraphedTrainStep(None, types.SimpleNamespace(world=2, overlap=True), meta_cuda)
