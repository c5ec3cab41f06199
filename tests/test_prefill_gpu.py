"""Tensor-core prefill kernel (``kv4_prefill_attention``) vs the CPU oracle
(float64 attention over the same dequantized cache).  bf16 tolerance 2e-2
max-abs, as for the other attention paths."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import ATOL, f32, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


def _cache(b, hkv, sk, d, gs, seed):
    from kvint4.cache import Int4KVStore
    k, v = kv_inputs(b, hkv, sk, d, dtype=torch.bfloat16, seed=seed, device="cuda")
    store = Int4KVStore(gs)
    store.append(k, v, 0)
    return store.layer(0).views()


def _query(b, hq, sq, d, seed):
    g = torch.Generator().manual_seed(seed + 100)
    return torch.randn(b, hq, sq, d, generator=g).to(torch.bfloat16).cuda()


def _check(b, hq, hkv, sq, sk, gs, causal, seed=0, out_view=False):
    from kvint4 import ops
    cache = _cache(b, hkv, sk, 128, gs, seed)
    q = _query(b, hq, sq, 128, seed)
    if out_view:  # [B, s, n, d] storage seen as [B, n, s, d], as the Llama module writes it
        out = torch.full((b, sq, hq, 128), float("nan"), dtype=torch.bfloat16,
                         device="cuda").transpose(1, 2)
    else:
        out = torch.full_like(q, float("nan"))
    assert ops.prefill_attention_into(q, *cache, out, gs, causal)
    torch.cuda.synchronize()
    ref = oracle_attention(q, *cache, n_q_heads=hq, n_kv_heads=hkv, group_size=gs,
                           is_causal=causal)
    got = f32(out)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err < ATOL[torch.bfloat16], err
    assert ops.device_error() == 0
    return err


@pytest.mark.parametrize("gs", [16, 32, 64, 128])
def test_prefill_square_causal(gs):
    _check(1, 8, 2, 300, 300, gs, True)


def test_prefill_chunk_bottom_right():
    # a second prefill chunk: 200 new queries over 1000 cached keys
    _check(2, 32, 8, 200, 1000, 32, True, seed=1)


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 2), (32, 1), (128, 1)])
def test_prefill_group_ratios(hq, hkv):
    _check(1, hq, hkv, 129, 257, 32, True, seed=2)


def test_prefill_not_causal():
    _check(2, 8, 2, 77, 513, 64, False, seed=3)


def test_prefill_single_tile_edges():
    _check(1, 4, 1, 1, 1, 32, True, seed=4)
    _check(1, 4, 1, 5, 128, 32, True, seed=5)
    _check(1, 4, 1, 128, 128, 32, True, seed=6)


def test_prefill_strided_out():
    _check(1, 32, 8, 96, 96, 32, True, seed=7, out_view=True)


def test_prefill_llama_shape_2048():
    """Llama-3.1-8B heads, a 2048-token prompt; checked against torch fp32
    attention over the same dequantized cache (the float64 oracle is slow at
    this size)."""
    import torch.nn.functional as F
    from torch.nn.attention.bias import causal_lower_right
    from kernels.llama3.quantize import dequantize_int4
    from kvint4 import ops
    b, hq, hkv, s, gs = 1, 32, 8, 2048, 32
    kp, ks, vp, vs = _cache(b, hkv, s, 128, gs, 8)
    q = _query(b, hq, s, 128, 8)
    out = torch.empty_like(q)
    assert ops.prefill_attention_into(q, kp, ks, vp, vs, out, gs, True)
    k = dequantize_int4(kp, ks, gs, 128, torch.float32)
    v = dequantize_int4(vp, vs, gs, 128, torch.float32)
    ref = F.scaled_dot_product_attention(q.float(), k, v, attn_mask=causal_lower_right(s, s),
                                         enable_gqa=True)
    err = (out.float() - ref).abs().max().item()
    assert err < ATOL[torch.bfloat16], err


def test_prefill_unsupported_shapes_report_back():
    from kvint4 import ops
    cache = _cache(1, 2, 64, 64, 32, 0)  # d = 64: not taken
    q = _query(1, 8, 16, 64, 0)
    out = torch.empty_like(q)
    assert not ops.prefill_attention_into(q, *cache, out, 32, True, strict=False)
    cache = _cache(1, 2, 64, 128, 32, 0)
    q = _query(1, 8, 100, 128, 0)  # causal with sq > sk
    out = torch.empty_like(q)
    assert not ops.prefill_attention_into(q, *cache, out, 32, True, strict=False)
    q = _query(1, 6, 16, 128, 0)  # 128 % (6 / 2) != 0
    out = torch.empty_like(q)
    assert not ops.prefill_attention_into(q, *cache, out, 32, True, strict=False)
