"""End-to-end decode with the INT4 cache on a random-init Llama-3.1-8B.

The reference measures its path end to end with Hugging Face models
(``benchmarks/llama3/run_llama3_benchmark.py``); here the model is the
Llama-3.1-8B architecture with random N(0, 0.02) bf16 weights (no
checkpoint is available offline) and uniform random prompt ids.

One model instance serves both runs: ``replace_llama_attention_with_quantized``
keeps stock behaviour when the cache is not a ``QuantizedKVCache``.

    python kv-cache-triton_b200/benchmarks/llama3_e2e.py [--batch 8] [--prompt 16384]
        [--steps 64] [--layers 32]

Prints one JSON line: decode ms/token (CUDA events, per greedy step, both
caches), cache bytes, the largest logit difference per step and how many
greedy tokens agree, against the bf16 cache and against a third run whose
DynamicCache stores quantize-dequantized K/V (same quantization error, stock
attention: isolates the kernels' arithmetic).  Each run prefills the same prompt and then feeds its
OWN greedy tokens (like ``generate``); logits are compared while the token
streams agree.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def llama31_8b_config(layers: int = 32, **over):
    from transformers import LlamaConfig
    kw = dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
              num_hidden_layers=layers, num_attention_heads=32, num_key_value_heads=8,
              head_dim=128, max_position_embeddings=131072, rope_theta=500000.0,
              rms_norm_eps=1e-5, initializer_range=0.02, tie_word_embeddings=False,
              attention_bias=False, mlp_bias=False)
    kw.update(over)
    return LlamaConfig(**kw)


def _decode(model, cache, prompt, steps):
    """Prefill, then `steps` greedy steps; returns (tokens, last logits per
    step, ms per decode step)."""
    with torch.inference_mode():
        out = model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1)
        nxt = out.logits[:, -1, :].argmax(-1, keepdim=True)
        toks, logits, ms = [nxt], [out.logits[:, -1, :].float()], []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = model(input_ids=nxt, past_key_values=cache, use_cache=True, logits_to_keep=1)
            e1.record()
            nxt = out.logits[:, -1, :].argmax(-1, keepdim=True)
            toks.append(nxt)
            logits.append(out.logits[:, -1, :].float())
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
    return torch.cat(toks, 1), logits, ms


def _fake_quant_cache(group_size):
    """DynamicCache whose stored K/V went through INT4 quantize + dequantize:
    the same quantization error as the INT4 cache, attention by the stock
    path.  Separates the kernels' arithmetic from the quantization error."""
    from transformers.cache_utils import DynamicCache

    from kernels.llama3.quantize import dequantize_int4, quantize_int4

    class FakeQuantCache(DynamicCache):
        def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
            d = key_states.shape[-1]
            kq = dequantize_int4(*quantize_int4(key_states, group_size), group_size, d,
                                 key_states.dtype)
            vq = dequantize_int4(*quantize_int4(value_states, group_size), group_size, d,
                                 value_states.dtype)
            return super().update(kq, vq, layer_idx, cache_kwargs)

    return FakeQuantCache()


def run(batch=8, prompt_len=16384, steps=64, layers=32, seed=0, group_size=32, config=None):
    from transformers import LlamaForCausalLM
    from transformers.cache_utils import DynamicCache

    from models.llama3.kv_cache import QuantizedKVCache
    from models.llama3.llama3_quant import replace_llama_attention_with_quantized

    dev = torch.device("cuda")
    cfg = config or llama31_8b_config(layers)
    torch.manual_seed(seed)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    replace_llama_attention_with_quantized(model, group_size=group_size)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    prompt = torch.randint(0, cfg.vocab_size, (batch, prompt_len), device=dev, generator=g)

    ref_cache = DynamicCache()
    t_ref, l_ref, ms_ref = _decode(model, ref_cache, prompt, steps)
    ref_bytes = sum(t.numel() * t.element_size() for lay in ref_cache.layers
                    for t in (lay.keys, lay.values))
    del ref_cache
    torch.cuda.empty_cache()
    q_cache = QuantizedKVCache(group_size=group_size)
    t_q, l_q, ms_q = _decode(model, q_cache, prompt, steps)
    fq_cache = _fake_quant_cache(group_size)
    t_fq, l_fq, _ = _decode(model, fq_cache, prompt, steps)
    del fq_cache

    def _agree(x, y):
        n = 0
        for i in range(x.shape[1]):
            if not torch.equal(x[:, i], y[:, i]):
                break
            n += 1
        return n

    agree_fq = _agree(t_fq, t_q)
    diffs_fq = [float((a - b).abs().max()) for a, b in zip(l_fq[:agree_fq + 1], l_q[:agree_fq + 1])]

    agree = 0  # leading greedy tokens identical in every batch row
    for i in range(t_ref.shape[1]):
        if not torch.equal(t_ref[:, i], t_q[:, i]):
            break
        agree += 1
    diffs = [float((a - b).abs().max()) for a, b in zip(l_ref[:agree + 1], l_q[:agree + 1])]
    return {
        "workload": f"llama3.1-8b arch random-init bf16, {layers} layers, batch {batch}, "
                    f"prefill {prompt_len} uniform ids, {steps} greedy steps",
        "decode_ms_per_token_int4": round(statistics.median(ms_q), 3),
        "decode_ms_per_token_bf16_dynamic": round(statistics.median(ms_ref), 3),
        "cache_bytes_int4": int(q_cache.nbytes()),
        "cache_bytes_bf16": int(ref_bytes),
        "greedy_tokens_agreeing": agree,
        "greedy_tokens_total": int(t_ref.shape[1]),
        "logits_max_abs_diff_first_step": round(diffs[0], 4),
        "logits_max_abs_diff_while_agreeing": round(max(diffs), 4),
        "logits_ref_abs_max": round(float(l_ref[0].abs().max()), 4),
        # against bf16 attention over the same quantize-dequantized K/V:
        "fakequant_greedy_tokens_agreeing": agree_fq,
        "fakequant_logits_max_abs_diff_first_step": round(diffs_fq[0], 4),
        "fakequant_logits_max_abs_diff_while_agreeing": round(max(diffs_fq), 4),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=16384)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    print(json.dumps(run(a.batch, a.prompt, a.steps, a.layers, a.seed)), flush=True)


if __name__ == "__main__":
    main()
