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
