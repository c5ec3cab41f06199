"""Fused INT4 attention on the GPU vs the CPU oracle (float64 attention over the
same dequantized cache).  Tolerances (max-abs): fp32 1e-3, fp16 5e-3,
bf16 2e-2 -- the bounds the north star states for fp32 and bf16."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import cases, load, to_f32
from helpers import ATOL, f32, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


def _run(b, hq, hkv, sq, sk, d, gs, qdt, causal=False, seed=0, sdt=None, contiguous=False,
         **kw):
    """Quantize seeded K/V into a capacity-buffer cache (or contiguous tensors),
    run the kernel and the oracle."""
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from kernels.llama3.quantize import quantize_int4
    from kvint4 import frontend
    from kvint4.cache import Int4KVStore
    k, v = kv_inputs(b, hkv, sk, d, dtype=qdt, seed=seed, device="cuda")
    g = torch.Generator().manual_seed(seed + 100)
    q = torch.randn(b, hq, sq, d, generator=g).to(qdt).cuda()
    if contiguous:
        kp, ks = quantize_int4(k, gs)
        vp, vs = quantize_int4(v, gs)
        if sdt is not None:
            ks, vs = ks.to(sdt), vs.to(sdt)
    else:
        store = Int4KVStore(gs, scale_dtype=sdt)
        store.append(k, v, 0)
        kp, ks, vp, vs = store.layer(0).views()
    if kw:
        out = frontend.attention(q, kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv,
                                 group_size=gs, is_causal=causal, **kw)
    else:
        out = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv,
                                          group_size=gs, is_causal=causal)
    ref = oracle_attention(q, kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv, group_size=gs,
                           is_causal=causal)
    return q, (kp, ks, vp, vs), out, ref


def _plan_path(q, cache, gs, causal=False, **kw):
    from kvint4 import ops
    out = torch.empty_like(q)
    return ops.plan(q, *cache, out, gs, causal, **kw).path


@pytest.mark.parametrize("qdt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d,gs", [(128, 32), (128, 64), (128, 128), (64, 32), (64, 64),
                                  (256, 32), (256, 128)])
def test_decode_fast_path_matches_oracle(qdt, d, gs):
    q, cache, out, ref = _run(2, 8, 2, 1, 301, d, gs, qdt)
    assert _plan_path(q, cache, gs) == 1
    assert out.dtype == qdt and torch.isfinite(out).all()
    np.testing.assert_allclose(f32(out), ref, atol=ATOL[qdt], rtol=0)


@pytest.mark.parametrize("ratio", [1, 2, 4, 8, 16])
def test_decode_gqa_ratios(ratio):
    q, cache, out, ref = _run(2, 2 * ratio, 2, 1, 200, 128, 32, torch.bfloat16)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)


@pytest.mark.parametrize("sk", [1, 2, 15, 63, 64, 65, 127, 129, 1000, 4099])
def test_decode_ragged_lengths(sk):
    q, cache, out, ref = _run(3, 8, 2, 1, sk, 128, 32, torch.float32, seed=sk)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)


@pytest.mark.parametrize("tiles_per_cta", [1, 2, 3, 5, 7, 64])
def test_stream_k_split_invariance(tiles_per_cta):
    """Every split of the sequence across CTAs gives the oracle's answer."""
    q, cache, out, ref = _run(2, 8, 2, 1, 1000, 128, 32, torch.float32, seed=3,
                              tiles_per_cta=tiles_per_cta)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)


@pytest.mark.parametrize("sq,causal", [(2, True), (3, False), (5, True), (16, True)])
def test_multi_query_rows_causal_bottom_right(sq, causal):
    q, cache, out, ref = _run(1, 8, 2, sq, 90, 128, 32, torch.float32, causal=causal, seed=sq)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)


@pytest.mark.parametrize("sk", [77, 301, 4096])
def test_contiguous_tensors_any_length(sk):
    """Freshly quantized contiguous tensors (the reference API's usual input):
    aligned lengths take the TMA path, others the generic kernel; both agree
    with the oracle."""
    q, cache, out, ref = _run(2, 8, 2, 1, sk, 128, 32, torch.bfloat16, contiguous=True)
    assert _plan_path(q, cache, 32) == (1 if sk % 2 == 0 else 2)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)


def test_generic_path_matches_oracle():
    q, cache, out, ref = _run(2, 8, 2, 1, 333, 128, 32, torch.float32, force_generic=True)
    assert _plan_path(q, cache, 32, force_generic=True) == 2
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)
    # odd head dim and group size only the generic kernel takes
    q, cache, out, ref = _run(1, 4, 2, 1, 50, 80, 16, torch.float32)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)


@pytest.mark.parametrize("sdt", [torch.float16, torch.float32])
def test_scale_dtypes(sdt):
    q, cache, out, ref = _run(2, 8, 2, 1, 257, 128, 32, torch.float32, sdt=sdt)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)


def test_cache_views_read_in_place_and_odd_lengths():
    """The capacity-buffer views (token stride = row, plane stride = capacity)
    go through the TMA path without copies."""
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from models.llama3.kv_cache import QuantizedKVCache
    k, v = kv_inputs(2, 2, 77, 128, device="cuda", seed=9)
    cache = QuantizedKVCache(group_size=32, capacity=256)
    cache.append(k, v, 0)
    kp, ks, vp, vs = cache.get_quantized(0)
    assert not kp.is_contiguous()
    q = torch.randn(2, 8, 1, 128, device="cuda").to(torch.bfloat16)
    assert _plan_path(q, (kp, ks, vp, vs), 32) == 1
    out = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=8, n_kv_heads=2)
    ref = oracle_attention(q, kp, ks, vp, vs, n_q_heads=8, n_kv_heads=2, group_size=32)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)


def _oracle_rows(q, kp, ks, vp, vs, hq, hkv):
    """The float64 oracle one batch row at a time (full-size shapes)."""
    return np.concatenate([
        oracle_attention(q[b:b + 1], kp[b:b + 1], ks[b:b + 1], vp[b:b + 1], vs[b:b + 1],
                         n_q_heads=hq, n_kv_heads=hkv, group_size=32)
        for b in range(q.shape[0])])


def test_llama8b_batch16_every_row_matches_oracle():
    """Llama-3.1-8B decode shape (B16, 32/8 heads, S 4096, d 128, G 32): every
    batch row against the oracle; split invariance; determinism."""
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from kernels.llama3.quantize import quantize_int4
    from kvint4 import frontend
    k, v = kv_inputs(16, 8, 4096, 128, device="cuda", seed=0)
    q = torch.randn(16, 32, 1, 128, device="cuda").to(torch.bfloat16)
    kp, ks = quantize_int4(k, 32)
    vp, vs = quantize_int4(v, 32)
    out = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8)
    out2 = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8)
    assert torch.equal(out, out2)  # deterministic
    one = frontend.attention(q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8, group_size=32,
                             is_causal=False, tiles_per_cta=64)  # one CTA per unit
    assert (out.float() - one.float()).abs().max().item() <= 2e-2
    ref = _oracle_rows(q, kp, ks, vp, vs, 32, 8)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)


def test_llama70b_head_shard_shape_every_row_matches_oracle():
    """Llama-3.1-70B decode with one KV head per GPU: B32, 8 q heads over 1 KV
    head (GQA 8), S 16384, d 128, G 32; every batch row against the oracle."""
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from kernels.llama3.quantize import quantize_int4
    k, v = kv_inputs(32, 1, 16384, 128, device="cuda", seed=70)
    q = torch.randn(32, 8, 1, 128, device="cuda").to(torch.bfloat16)
    kp, ks = quantize_int4(k, 32)
    vp, vs = quantize_int4(v, 32)
    out = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=8, n_kv_heads=1)
    assert _plan_path(q, (kp, ks, vp, vs), 32) == 1
    ref = _oracle_rows(q, kp, ks, vp, vs, 8, 1)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)


def test_gpt2_small_decode_entry_point_matches_oracle():
    """GPT-2-small decode through kernels.gpt2.attention_quant.attention_forward_quant:
    fp32 q [4, 12, 1, 64], K/V [4, 12, 1024, 64] N(0,1), G 32, fp16 scales
    (reference tests/gpt2/test_attention_quant.py:13-62)."""
    from kernels.gpt2.attention_quant import attention_forward_quant
    from kernels.gpt2.quantize import quantize_int4
    g = torch.Generator().manual_seed(0)
    q = torch.randn(4, 12, 1, 64, generator=g).cuda()
    k = torch.randn(4, 12, 1024, 64, generator=g).cuda()
    v = torch.randn(4, 12, 1024, 64, generator=g).cuda()
    kp, ks = quantize_int4(k, group_size=32)
    vp, vs = quantize_int4(v, group_size=32)
    assert ks.dtype == torch.float16
    out = attention_forward_quant(q, kp, ks, vp, vs, group_size=32)
    assert out.dtype == torch.float32 and out.shape == q.shape
    ref = oracle_attention(q, kp, ks, vp, vs, n_q_heads=12, n_kv_heads=12, group_size=32)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)
    # fp16 q as well (the reference accepts fp16 and fp32)
    out16 = attention_forward_quant(q.half(), kp, ks, vp, vs, group_size=32)
    ref16 = oracle_attention(q.half(), kp, ks, vp, vs, n_q_heads=12, n_kv_heads=12,
                             group_size=32)
    np.testing.assert_allclose(f32(out16), ref16, atol=5e-3, rtol=0)


def test_gpt2_golden_mha_case():
    """The golden d64 MHA decode case through the GPT-2 entry point."""
    from kernels.gpt2.attention_quant import attention_forward_quant
    names = [c for c in cases(A) if "mha" in c and "d64" in c]
    if not names:
        pytest.skip("no golden MHA d64 case")
    for case in names:
        b, hq, hkv, sq, sk, d, gs, causal = (int(x) for x in A[case + ".meta"])
        qdt = str(A[case + ".q_dtype"])
        sdt = str(A[case + ".scale_dtype"])
        if qdt not in ("f16", "f32") or sdt != "f16" or hq != hkv:
            continue
        tdt = {"f16": torch.float16, "f32": torch.float32}
        q = torch.from_numpy(to_f32(A[case + ".q"], qdt)).to(tdt[qdt]).cuda()
        ks = torch.from_numpy(to_f32(A[case + ".k_scales"], sdt)).half().cuda()
        vs = torch.from_numpy(to_f32(A[case + ".v_scales"], sdt)).half().cuda()
        kp = torch.from_numpy(A[case + ".k_packed"]).cuda()
        vp = torch.from_numpy(A[case + ".v_packed"]).cuda()
        out = attention_forward_quant(q, kp, ks, vp, vs, group_size=gs, is_causal=bool(causal))
        np.testing.assert_allclose(f32(out), A[case + ".out_ref_f32"], atol=ATOL[tdt[qdt]],
                                   rtol=0)


A = load("attn_cases.npz")


@pytest.mark.parametrize("case", cases(A))
def test_attention_golden_reference_cases(case):
    """The reference's own GQA reference (looped fp32 / SDPA) on the golden inputs."""
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    b, hq, hkv, sq, sk, d, gs, causal = (int(x) for x in A[case + ".meta"])
    qdt = str(A[case + ".q_dtype"])
    sdt = str(A[case + ".scale_dtype"])
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
    q = torch.from_numpy(to_f32(A[case + ".q"], qdt)).to(tdt[qdt]).cuda()
    ks = torch.from_numpy(to_f32(A[case + ".k_scales"], sdt)).to(tdt[sdt]).cuda()
    vs = torch.from_numpy(to_f32(A[case + ".v_scales"], sdt)).to(tdt[sdt]).cuda()
    kp = torch.from_numpy(A[case + ".k_packed"]).cuda()
    vp = torch.from_numpy(A[case + ".v_packed"]).cuda()
    out = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv,
                                      group_size=gs, is_causal=bool(causal))
    np.testing.assert_allclose(f32(out), A[case + ".out_ref_f32"], atol=ATOL[tdt[qdt]], rtol=0)


def test_partial_and_lse_combine_equal_full():
    """Sequence shards (kv4_attention_partial) merged by kv4_lse_combine equal
    the unsharded result -- the math of the multi-GPU sequence-shard layer."""
    from kernels.llama3.quantize import quantize_int4
    from kvint4 import ops
    k, v = kv_inputs(2, 2, 700, 128, dtype=torch.float32, device="cuda", seed=4)
    q = torch.randn(2, 8, 3, 128, device="cuda")
    kp, ks = quantize_int4(k, 32)
    vp, vs = quantize_int4(v, 32)
    ref = oracle_attention(q, kp, ks, vp, vs, n_q_heads=8, n_kv_heads=2, group_size=32,
                           is_causal=True)
    bounds = [0, 150, 301, 650, 700]
    po = torch.empty(4, 2, 8, 3, 128, device="cuda")
    pl = torch.empty(4, 2, 8, 3, device="cuda")
    for r in range(4):
        a, e = bounds[r], bounds[r + 1]
        ops.attention_partial_into(q, kp[:, :, a:e], ks[:, :, a:e], vp[:, :, a:e],
                                   vs[:, :, a:e], po[r], pl[r], a, 700, 32, True)
    out = torch.empty(2, 8, 3, 128, device="cuda")
    ops.lse_combine_into(po.reshape(4, -1, 128), pl.reshape(4, -1), out)
    np.testing.assert_allclose(f32(out), ref, atol=1e-3, rtol=0)


def test_prefill_long_block_routes_and_matches():
    q, cache, out, ref = _run(1, 4, 2, 300, 300, 128, 32, torch.bfloat16, causal=True)
    np.testing.assert_allclose(f32(out), ref, atol=3e-2, rtol=0)


def test_no_device_error_flag_after_runs():
    from kvint4 import ops
    _run(2, 8, 2, 1, 500, 128, 32, torch.bfloat16)
    assert ops.device_error() == 0


@pytest.mark.parametrize("sk", [16384, 131072])
def test_config3_long_context_batch1(sk):
    """Batch-1 long-context shape (B=1, 32/8 heads, d=128, G=32) at full length:
    KV head 0 (q heads 0-3) against the oracle, plus agreement of the fused
    kernel with a 4-way sequence-shard decomposition for all heads."""
    from kvint4 import ops
    from kvint4.cache import Int4KVStore
    from kvint4.shard import shard_range
    k, v = kv_inputs(1, 8, sk, 128, device="cuda", seed=sk % 97)
    st = Int4KVStore(32)
    st.append(k, v, 0)
    kp, ks, vp, vs = st.layer(0).views()
    q = torch.randn(1, 32, 1, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    ops.attention_into(q, kp, ks, vp, vs, out, 32)
    ref = oracle_attention(q[:, :4], kp[:, :1], ks[:, :1], vp[:, :1], vs[:, :1], n_q_heads=4,
                           n_kv_heads=1, group_size=32)
    np.testing.assert_allclose(f32(out[:, :4]), ref, atol=2e-2, rtol=0)
    po = torch.empty(4, 1, 32, 1, 128, device="cuda")
    pl = torch.empty(4, 1, 32, 1, device="cuda")
    for r in range(4):
        a, e = shard_range(sk, 4, r)
        ops.attention_partial_into(q, kp[:, :, a:e], ks[:, :, a:e], vp[:, :, a:e], vs[:, :, a:e],
                                   po[r], pl[r], a, sk, 32)
    comb = torch.empty_like(q)
    ops.lse_combine_into(po.reshape(4, -1, 128), pl.reshape(4, -1), comb)
    assert (comb.float() - out.float()).abs().max().item() <= 2e-2
