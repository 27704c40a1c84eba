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
