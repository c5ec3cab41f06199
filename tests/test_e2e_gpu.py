"""The end-to-end runner (kv-cache-triton_b200/benchmarks/llama3_e2e.py) on a
small random Llama: prefill + greedy decode with the INT4 cache against the
same model on DynamicCache."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_llama_e2e_runner_small():
    from benchmarks.llama3_e2e import llama31_8b_config, run
    cfg = llama31_8b_config(2, vocab_size=1000, hidden_size=512, intermediate_size=1024,
                            num_attention_heads=8, num_key_value_heads=2, head_dim=64)
    r = run(batch=2, prompt_len=300, steps=8, layers=2, config=cfg)
    assert r["greedy_tokens_total"] == 9
    # a tiny random model has nearly tied logits, so greedy tokens may part
    # early; the first step's logits must still be close
    assert r["greedy_tokens_agreeing"] >= 1, r
    # INT4 K/V perturb the logits a little; far below their spread
    assert r["logits_max_abs_diff_first_step"] < 0.25 * r["logits_ref_abs_max"], r
    assert r["cache_bytes_int4"] * 3 < r["cache_bytes_bf16"], r
    # against stock attention over the same quantize-dequantized K/V the only
    # difference left is arithmetic order and bf16 rounding: a few hundredths
    # of the logit range (the tiny model's top logits are often closer than
    # that, so its greedy tokens are not compared here)
    assert r["fakequant_logits_max_abs_diff_first_step"] < 0.05 * r["logits_ref_abs_max"], r
