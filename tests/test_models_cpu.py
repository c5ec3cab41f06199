"""The patched attention modules on CPU: replacing keeps every parameter in
place, and without a QuantizedKVCache the patched model computes exactly
what the stock Hugging Face model computes (the module only takes over the
cached INT4 route, which needs the GPU)."""

from __future__ import annotations

import pytest
import torch


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=97, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def _tiny_gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel
    cfg = GPT2Config(vocab_size=97, n_embd=64, n_layer=2, n_head=4, n_positions=64)
    torch.manual_seed(0)
    return GPT2LMHeadModel(cfg).eval()


@pytest.mark.parametrize("family", ["llama", "gpt2"])
def test_replace_keeps_parameters_and_stock_outputs(family):
    if family == "llama":
        from models.llama3.llama3_quant import (LlamaAttentionQuantized as Q,
                                                replace_llama_attention_with_quantized as rep)
        model = _tiny_llama()
        mods = lambda m: [l.self_attn for l in m.model.layers]  # noqa: E731
    else:
        from models.gpt2.gpt2_quant import (GPT2AttentionQuantized as Q,
                                            replace_gpt2_attention_with_quantized as rep)
        model = _tiny_gpt2()
        mods = lambda m: [b.attn for b in m.transformer.h]  # noqa: E731
    ids = torch.randint(0, 97, (2, 9), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(ids).logits
    before = {n: p.data_ptr() for n, p in model.named_parameters()}
    rep(model, group_size=16)
    assert all(type(m) is Q and m.quant_group_size == 16 for m in mods(model))
    assert {n: p.data_ptr() for n, p in model.named_parameters()} == before
    with torch.no_grad():
        out = model(ids).logits
    assert torch.equal(out, ref)
    rep(model, group_size=32)  # idempotent; updates the group size
    assert all(type(m) is Q and m.quant_group_size == 32 for m in mods(model))


def test_replace_rejects_non_models():
    from models.gpt2.gpt2_quant import replace_gpt2_attention_with_quantized
    from models.llama3.llama3_quant import replace_llama_attention_with_quantized
    with pytest.raises(ValueError):
        replace_llama_attention_with_quantized(torch.nn.Linear(2, 2))
    with pytest.raises(ValueError):
        replace_gpt2_attention_with_quantized(torch.nn.Linear(2, 2))


def test_replace_rebinds_accelerate_hook_forward():
    """A module dispatched by accelerate (device_map) keeps its hook, and the
    hook's saved forward calls the patched forward."""
    accelerate = pytest.importorskip("accelerate")
    from accelerate.hooks import ModelHook, add_hook_to_module

    from models.llama3.llama3_quant import (LlamaAttentionQuantized,
                                            replace_llama_attention_with_quantized)
    model = _tiny_llama()
    attn = model.model.layers[0].self_attn
    add_hook_to_module(attn, ModelHook())
    replace_llama_attention_with_quantized(model)
    assert attn._old_forward.__func__ is LlamaAttentionQuantized.forward
    del accelerate
