"""Model glue on the GPU: tiny random Llama / GPT-2 with the INT4 cache vs the
stock DynamicCache (ports of the reference's tests/llama3/test_llama3_quant_decode.py
and test_llama3_generate_parity.py, same shapes and tolerances)."""

from __future__ import annotations

import pytest
import torch
from transformers import GPT2Config, GPT2LMHeadModel, LlamaConfig, LlamaForCausalLM
from transformers.cache_utils import DynamicCache

pytestmark = pytest.mark.gpu


def _tiny_llama(device, dtype=torch.bfloat16):
    cfg = LlamaConfig(vocab_size=256, hidden_size=128, intermediate_size=256,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=64, max_position_embeddings=512, rms_norm_eps=1e-5,
                      tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def test_llama_prefill_plus_decode_matches_reference():
    from models.llama3.kv_cache import QuantizedKVCache
    from models.llama3.llama3_quant import replace_llama_attention_with_quantized
    dev = torch.device("cuda")
    model_ref = _tiny_llama(dev)
    model_q = _tiny_llama(dev)
    model_q.load_state_dict(model_ref.state_dict())
    replace_llama_attention_with_quantized(model_q, group_size=32)
    torch.manual_seed(123)
    prompt = torch.randint(0, 256, (1, 32), device=dev)
    with torch.no_grad():
        cache_ref = DynamicCache()
        out_ref = model_ref(input_ids=prompt, past_key_values=cache_ref, use_cache=True)
        cache_q = QuantizedKVCache(group_size=32)
        out_q = model_q(input_ids=prompt, past_key_values=cache_q, use_cache=True)
        lr, lq = out_ref.logits[:, -1], out_q.logits[:, -1]
        assert (lr.float() - lq.float()).abs().max().item() < 1.0
        assert lr.argmax(-1).item() == lq.argmax(-1).item()
        for _ in range(8):
            nxt = torch.randint(0, 256, (1, 1), device=dev)
            out_ref = model_ref(input_ids=nxt, past_key_values=cache_ref, use_cache=True)
            out_q = model_q(input_ids=nxt, past_key_values=cache_q, use_cache=True)
            diff = (out_ref.logits[:, -1].float() - out_q.logits[:, -1].float()).abs().max()
            assert diff.item() < 2.0


def test_llama_cache_tracks_seq_len_and_bytes():
    from models.llama3.kv_cache import QuantizedKVCache
    from models.llama3.llama3_quant import replace_llama_attention_with_quantized
    dev = torch.device("cuda")
    model = _tiny_llama(dev)
    replace_llama_attention_with_quantized(model, group_size=32)
    with torch.no_grad():
        cache = QuantizedKVCache(group_size=32)
        model(input_ids=torch.randint(0, 256, (1, 16), device=dev), past_key_values=cache,
              use_cache=True)
        assert cache.get_seq_length(0) == 16
        for step in range(4):
            model(input_ids=torch.randint(0, 256, (1, 1), device=dev), past_key_values=cache,
                  use_cache=True)
            assert cache.get_seq_length(0) == 16 + step + 1
    assert cache.nbytes() > 0
    seq = 128
    with torch.no_grad():
        cache = QuantizedKVCache(group_size=32)
        model(input_ids=torch.randint(0, 256, (1, seq), device=dev), past_key_values=cache,
              use_cache=True)
    cfg = model.config
    baseline = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * seq * cfg.head_dim * 2
    assert cache.nbytes() < baseline / 2


def _greedy(model, prompt, cache, n_new):
    tokens = []
    with torch.no_grad():
        out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
        nxt = out.logits[:, -1, :].argmax(-1, keepdim=True)
        tokens.append(int(nxt.item()))
        for _ in range(n_new - 1):
            out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            nxt = out.logits[:, -1, :].argmax(-1, keepdim=True)
            tokens.append(int(nxt.item()))
    return tokens


def test_llama_greedy_generate_prefix_agreement():
    """Greedy prefix agreement >= 4 of 16 tokens, same model, seeds and prompt as
    the reference's tests/llama3/test_llama3_generate_parity.py:52-74."""
    from models.llama3.kv_cache import QuantizedKVCache
    from models.llama3.llama3_quant import replace_llama_attention_with_quantized
    dev = torch.device("cuda")
    model_ref = _tiny_llama(dev)
    model_q = _tiny_llama(dev)
    model_q.load_state_dict(model_ref.state_dict())
    replace_llama_attention_with_quantized(model_q, group_size=32)
    torch.manual_seed(321)
    prompt = torch.randint(0, 256, (1, 24), device=dev, dtype=torch.long)
    a = _greedy(model_ref, prompt, DynamicCache(), 16)
    b = _greedy(model_q, prompt, QuantizedKVCache(group_size=32), 16)
    agree = 0
    for x, y in zip(a, b):
        if x != y:
            break
        agree += 1
    assert agree >= 4, (a, b)


def test_gpt2_random_decode_matches_dynamic_cache():
    """Random-init tiny GPT-2 (no checkpoint download), fp32, INT4 cache vs DynamicCache."""
    from models.gpt2.gpt2_quant import replace_gpt2_attention_with_quantized
    from models.gpt2.kv_cache import QuantizedKVCache
    dev = torch.device("cuda")
    cfg = GPT2Config(vocab_size=256, n_positions=256, n_embd=128, n_layer=2, n_head=2)
    torch.manual_seed(0)
    ref = GPT2LMHeadModel(cfg).to(dev).eval()
    qm = GPT2LMHeadModel(cfg).to(dev).eval()
    qm.load_state_dict(ref.state_dict())
    replace_gpt2_attention_with_quantized(qm, group_size=32)
    prompt = torch.randint(0, 256, (2, 20), device=dev)
    with torch.no_grad():
        c_ref, c_q = DynamicCache(), QuantizedKVCache(group_size=32)
        o_ref = ref(input_ids=prompt, past_key_values=c_ref, use_cache=True)
        o_q = qm(input_ids=prompt, past_key_values=c_q, use_cache=True)
        assert (o_ref.logits[:, -1] - o_q.logits[:, -1]).abs().max().item() < 1.0
        for _ in range(6):
            nxt = torch.randint(0, 256, (2, 1), device=dev)
            o_ref = ref(input_ids=nxt, past_key_values=c_ref, use_cache=True)
            o_q = qm(input_ids=nxt, past_key_values=c_q, use_cache=True)
            assert (o_ref.logits[:, -1] - o_q.logits[:, -1]).abs().max().item() < 2.0
    assert c_q.get_seq_length(0) == 26


def test_llama_hf_generate_accepts_quantized_cache():
    """model.generate() threads the INT4 cache through prefill and decode
    (the reference's scripts/llama3_smoke.py:110-130 does the same); greedy
    output agrees with the same model on DynamicCache for >= 4 tokens and
    the cache ends at prompt + new tokens - 1 rows."""
    from models.llama3.kv_cache import QuantizedKVCache
    from models.llama3.llama3_quant import replace_llama_attention_with_quantized
    dev = torch.device("cuda")
    model_ref = _tiny_llama(dev)
    model_q = _tiny_llama(dev)
    model_q.load_state_dict(model_ref.state_dict())
    replace_llama_attention_with_quantized(model_q, group_size=32)
    torch.manual_seed(321)
    prompt = torch.randint(0, 256, (2, 24), device=dev, dtype=torch.long)
    mask = torch.ones_like(prompt)
    with torch.inference_mode():
        a = model_ref.generate(input_ids=prompt, attention_mask=mask, max_new_tokens=12,
                               do_sample=False, past_key_values=DynamicCache())
        cache = QuantizedKVCache(group_size=32)
        b = model_q.generate(input_ids=prompt, attention_mask=mask, max_new_tokens=12,
                             do_sample=False, past_key_values=cache)
    assert b.shape == a.shape == (2, 36)
    assert torch.equal(a[:, :24], b[:, :24])
    assert torch.equal(a[:, 24], b[:, 24]), (a[:, 24:], b[:, 24:])
    assert cache.get_seq_length(0) == 24 + 12 - 1


def test_gpt2_hf_generate_accepts_quantized_cache():
    from models.gpt2.gpt2_quant import replace_gpt2_attention_with_quantized
    from models.gpt2.kv_cache import QuantizedKVCache
    dev = torch.device("cuda")
    cfg = GPT2Config(vocab_size=256, n_positions=256, n_embd=128, n_layer=2, n_head=2)
    torch.manual_seed(0)
    ref = GPT2LMHeadModel(cfg).to(dev).eval()
    qm = GPT2LMHeadModel(cfg).to(dev).eval()
    qm.load_state_dict(ref.state_dict())
    replace_gpt2_attention_with_quantized(qm, group_size=32)
    prompt = torch.randint(0, 256, (2, 20), device=dev)
    mask = torch.ones_like(prompt)
    with torch.inference_mode():
        a = ref.generate(input_ids=prompt, attention_mask=mask, max_new_tokens=10,
                         do_sample=False, past_key_values=DynamicCache())
        cache = QuantizedKVCache(group_size=32)
        b = qm.generate(input_ids=prompt, attention_mask=mask, max_new_tokens=10,
                        do_sample=False, past_key_values=cache)
    assert b.shape == a.shape == (2, 30)
    assert torch.equal(a[:, :21], b[:, :21]), (a[:, 20:], b[:, 20:])
    assert cache.get_seq_length(0) == 29
