"""kv4_attn_opts.early_start: the decode kernel launched with programmatic
stream serialization starts while the kernel before it drains.

The risky case is a decode loop on ONE layer with nothing in between: step t
writes row t, and step t+1 (started early) streams the cache before step t
has finished.  The kernel holds back the tile of row app_row - 1 until the
previous grid completed, so every step must give bit-identical output and
cache bytes to the same loop run in plain stream order, eagerly and replayed
from a CUDA graph.  ``QuantizedKVCache.append_attend`` turns early start on
only after its own fused step; an ``append`` in between turns it off.
"""

from __future__ import annotations

import pytest
import torch

from helpers import kv_inputs

pytestmark = pytest.mark.gpu


def _stores(b, hkv, s0, d, gs, n_steps):
    from kvint4.cache import Int4KVStore
    k, v = kv_inputs(b, hkv, s0, d, dtype=torch.bfloat16, seed=3, device="cuda")
    out = []
    for _ in range(2):
        st = Int4KVStore(gs, capacity=s0 + n_steps + 64)
        st.append(k, v, 0)
        out.append(st)
    return out


def _rows(b, hq, hkv, d, n_steps):
    g = torch.Generator().manual_seed(11)
    q = torch.randn(n_steps, b, hq, 1, d, generator=g).to(torch.bfloat16).cuda()
    kn = (torch.randn(n_steps, b, hkv, 1, d, generator=g) * 2).to(torch.bfloat16).cuda()
    vn = torch.randn(n_steps, b, hkv, 1, d, generator=g).to(torch.bfloat16).cuda()
    return q, kn, vn


def _loop(store, q, kn, vn, outs, early, gs):
    """n decode steps on layer 0, back to back on one stream."""
    from kvint4 import ops
    layer = store.layer(0)
    for t in range(q.shape[0]):
        n = layer.seq_len + 1
        ops.append_attention_descs(q[t], kn[t], vn[t], layer.view_descs(n), outs[t], gs,
                                   early_start=early)
        layer.seq_len = n


# (b, hq, hkv, s0, d): split-K parts, clusters, the row crossing a tile boundary
CASES = [(16, 32, 8, 4095 - 6, 128), (1, 32, 8, 16384 - 100, 128), (2, 8, 2, 125, 128),
         (4, 16, 4, 1021, 64)]


@pytest.mark.parametrize("b,hq,hkv,s0,d", CASES)
def test_early_start_decode_loop_matches_stream_order(b, hq, hkv, s0, d):
    gs, n = 32, 12
    plain, early = _stores(b, hkv, s0, d, gs, n)
    q, kn, vn = _rows(b, hq, hkv, d, n)
    o_plain = torch.empty(n, b, hq, 1, d, dtype=torch.bfloat16, device="cuda")
    o_early = torch.full_like(o_plain, float("nan"))
    _loop(plain, q, kn, vn, o_plain, False, gs)
    _loop(early, q, kn, vn, o_early, True, gs)
    torch.cuda.synchronize()
    assert torch.equal(o_plain, o_early)
    for a, c in zip(plain.layer(0).views(), early.layer(0).views()):
        assert torch.equal(a, c)


def test_early_start_in_cuda_graph():
    b, hq, hkv, s0, d, gs, n = 4, 32, 8, 2047 - 5, 128, 32, 10
    plain, early = _stores(b, hkv, s0, d, gs, n)
    q, kn, vn = _rows(b, hq, hkv, d, n)
    o_plain = torch.empty(n, b, hq, 1, d, dtype=torch.bfloat16, device="cuda")
    o_early = torch.full_like(o_plain, float("nan"))
    _loop(plain, q, kn, vn, o_plain, False, gs)
    # warm the early store's workspace on a side copy, then capture the loop
    s1 = early.layer(0).seq_len
    _loop(early, q[:1], kn[:1], vn[:1], o_early[:1], True, gs)
    early.layer(0).seq_len = s1
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _loop(early, q, kn, vn, o_early, True, gs)
    early.layer(0).seq_len = s1
    g.replay()
    early.layer(0).seq_len = s1 + n
    torch.cuda.synchronize()
    assert torch.equal(o_plain, o_early)
    for a, c in zip(plain.layer(0).views(), early.layer(0).views()):
        assert torch.equal(a, c)


def test_cache_turns_early_start_on_only_after_its_own_step():
    from models.llama3.kv_cache import QuantizedKVCache
    b, hq, hkv, d = 2, 8, 2, 128
    k, v = kv_inputs(b, hkv, 300, d, dtype=torch.bfloat16, seed=5, device="cuda")
    cache = QuantizedKVCache(group_size=32)
    ref = QuantizedKVCache(group_size=32)
    cache.append(k, v, 0)
    ref.append(k, v, 0)
    layer = cache._store.layer(0)
    assert layer.early_ok is False
    q, kn, vn = _rows(b, hq, hkv, d, 6)
    outs, refs = [], []
    from kvint4 import ops
    for t in range(6):
        o = torch.empty(b, hq, 1, d, dtype=torch.bfloat16, device="cuda")
        cache.append_attend(q[t], kn[t], vn[t], 0, o, n_q_heads=hq, n_kv_heads=hkv)
        assert layer.early_ok is True
        outs.append(o)
        if t == 2:  # a separate append: the next fused step runs in stream order
            cache.append(kn[t], vn[t], 0)
            assert layer.early_ok is False
        r = torch.empty_like(o)
        ref._store.append(kn[t], vn[t], 0)
        ops.attention_into(q[t], *ref._store.layer(0).views(), r, 32)
        refs.append(r)
        if t == 2:
            ref._store.append(kn[t], vn[t], 0)
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
