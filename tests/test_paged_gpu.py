"""Paged (block-table) INT4 cache on the GPU: kv4_append_kv_paged writes the
same bytes as the contiguous quantizer, and kv4_attention_paged over ragged
sequences matches the CPU oracle run on each sequence's own contiguous
cache (tolerances of tests/helpers.py), including shuffled page order,
several page sizes, head dims and query dtypes, multi-token causal steps, and
agreement with the contiguous kernel when every sequence has the same
length."""

from __future__ import annotations

import ctypes
import random

import numpy as np
import pytest
import torch

from helpers import ATOL, f32, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


def _fill(cache, lens, hkv, d, dt, seed, shuffle=True):
    """Prefill sequences 0..len(lens)-1 with seeded K/V; returns the K/V."""
    if shuffle:
        random.Random(seed).shuffle(cache._free)
    kv = []
    for sid, n in enumerate(lens):
        cache.add_sequence(sid)
        k, v = kv_inputs(1, hkv, n, d, dtype=dt, seed=seed + sid, device="cuda")
        st = cache.begin_step([sid], n)
        for layer in range(len(cache.k_pages)):
            cache.append(layer, st, k, v)
        cache.commit(st)
        kv.append((k, v))
    return kv


def _decode(cache, lens, hq, hkv, d, dt, seed, sq=1, causal=False):
    g = torch.Generator().manual_seed(seed + 99)
    b = len(lens)
    kn = torch.randn(b, hkv, sq, d, generator=g).to(dt).cuda()
    vn = torch.randn(b, hkv, sq, d, generator=g).to(dt).cuda()
    q = torch.randn(b, hq, sq, d, generator=g).to(dt).cuda()
    st = cache.begin_step(list(range(b)), sq)
    cache.append(0, st, kn, vn)
    out = cache.attend(0, st, q, is_causal=causal)
    cache.commit(st)
    torch.cuda.synchronize()
    return q, kn, vn, out


@pytest.mark.parametrize("page", [8, 16, 64, 128])
def test_paged_ragged_decode_matches_oracle(page):
    from kvint4.paged import PagedInt4KVCache
    lens = [1, 127, 128, 1000, 2999]
    hq, hkv, d, gs = 32, 8, 128, 32
    cache = PagedInt4KVCache(1024, page, hkv, d, group_size=gs)
    _fill(cache, lens, hkv, d, torch.bfloat16, seed=page)
    q, kn, vn, out = _decode(cache, lens, hq, hkv, d, torch.bfloat16, seed=page)
    for i in range(len(lens)):
        kp, ks, vp, vs = cache.gather(0, i)
        exp = oracle_attention(q[i:i + 1], kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv,
                               group_size=gs)
        np.testing.assert_allclose(f32(out[i:i + 1]), exp, atol=ATOL[torch.bfloat16], rtol=0)


def test_paged_append_bytes_match_contiguous_quantizer():
    from kvint4.cache import Int4KVStore
    from kvint4.paged import PagedInt4KVCache
    lens = [5, 300, 77]
    hkv, d, gs = 4, 128, 32
    cache = PagedInt4KVCache(64, 16, hkv, d, group_size=gs)
    kv = _fill(cache, lens, hkv, d, torch.bfloat16, seed=3)
    for sid, (k, v) in enumerate(kv):
        ref = Int4KVStore(gs)
        ref.append(k, v, 0)
        for x, y in zip(cache.gather(0, sid), ref.layer(0).views()):
            assert torch.equal(x, y)


@pytest.mark.parametrize("d,gs,qdt", [(64, 32, torch.float16), (256, 64, torch.float32),
                                      (128, 128, torch.bfloat16)])
def test_paged_shapes_and_dtypes(d, gs, qdt):
    from kvint4.paged import PagedInt4KVCache
    lens = [33, 700, 129]
    hq, hkv = 8, 2
    cache = PagedInt4KVCache(256, 32, hkv, d, group_size=gs, scale_dtype=qdt)
    _fill(cache, lens, hkv, d, qdt, seed=7)
    q, kn, vn, out = _decode(cache, lens, hq, hkv, d, qdt, seed=7)
    for i in range(len(lens)):
        exp = oracle_attention(q[i:i + 1], *cache.gather(0, i), n_q_heads=hq, n_kv_heads=hkv,
                               group_size=gs)
        np.testing.assert_allclose(f32(out[i:i + 1]), exp, atol=ATOL[qdt], rtol=0)


def test_paged_multi_token_causal_step():
    """4 new tokens per sequence, each query sees keys up to its own position."""
    from kvint4.paged import PagedInt4KVCache
    lens = [3, 200, 1000]
    hq, hkv, d, gs = 16, 4, 128, 32
    cache = PagedInt4KVCache(256, 16, hkv, d, group_size=gs)
    _fill(cache, lens, hkv, d, torch.bfloat16, seed=11)
    q, kn, vn, out = _decode(cache, lens, hq, hkv, d, torch.bfloat16, seed=11, sq=4,
                             causal=True)
    for i in range(len(lens)):
        exp = oracle_attention(q[i:i + 1], *cache.gather(0, i), n_q_heads=hq, n_kv_heads=hkv,
                               group_size=gs, is_causal=True)
        np.testing.assert_allclose(f32(out[i:i + 1]), exp, atol=ATOL[torch.bfloat16], rtol=0)


def test_paged_equal_lengths_match_contiguous_kernel():
    from kvint4 import ops
    from kvint4.cache import Int4KVStore
    from kvint4.paged import PagedInt4KVCache
    b, hq, hkv, s, d, gs = 3, 32, 8, 1500, 128, 32
    cache = PagedInt4KVCache(512, 64, hkv, d, group_size=gs)
    k, v = kv_inputs(b, hkv, s, d, dtype=torch.bfloat16, seed=5, device="cuda")
    random.Random(1).shuffle(cache._free)
    for i in range(b):
        cache.add_sequence(i)
    st = cache.begin_step(list(range(b)), s)
    cache.append(0, st, k, v)
    cache.commit(st)
    q = torch.randn(b, hq, 1, d, generator=torch.Generator().manual_seed(2)).to(
        torch.bfloat16).cuda()
    st0 = cache.begin_step(list(range(b)), 0)
    out = cache.attend(0, st0, q)
    ref_store = Int4KVStore(gs)
    ref_store.append(k, v, 0)
    ref = torch.empty_like(q)
    ops.attention_into(q, *ref_store.layer(0).views(), ref, gs)
    torch.cuda.synchronize()
    # same split of the sequence; the two kernels are separate instantiations,
    # so agreement is to bf16 rounding, not bit for bit
    np.testing.assert_allclose(f32(out), f32(ref), atol=1e-2, rtol=0)


def test_paged_bad_page_id_is_reported_not_read():
    """A block-table entry outside the pool is skipped and flagged (bit 2)."""
    from kvint4 import _lib, ops
    from kvint4.paged import PagedInt4KVCache
    hq, hkv, d, gs = 8, 2, 128, 32
    cache = PagedInt4KVCache(16, 16, hkv, d, group_size=gs)
    _fill(cache, [40], hkv, d, torch.bfloat16, seed=1, shuffle=False)
    st = cache.begin_step([0], 0)
    st.block_table[0, 1] = 1000  # not a page of the pool
    q = torch.randn(1, hq, 1, d, device="cuda").to(torch.bfloat16)
    cache.attend(0, st, q)  # the values of the skipped page's rows are undefined
    assert ops.device_error() & 2
    assert ops.device_error() == 0  # read-and-clear


def test_paged_argument_errors():
    from kvint4 import _lib, ops
    from kvint4.paged import PagedInt4KVCache
    with pytest.raises(ValueError):
        PagedInt4KVCache(4, 24, 2, 128)
    cache = PagedInt4KVCache(8, 16, 2, 128)
    cache.add_sequence(0)
    st = cache.begin_step([0], 20)
    q = torch.randn(1, 8, 1, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    with pytest.raises(_lib.Kv4Error):  # max_seq_len beyond the block table
        ops.attention_paged_into(q, cache.k_pages[0], cache.k_scales[0], cache.v_pages[0],
                                 cache.v_scales[0], st.block_table, st.seq_lens, 10_000, out, 32)
    with pytest.raises(RuntimeError):  # pool exhausted
        cache.begin_step([0], 8 * 16 + 1)
