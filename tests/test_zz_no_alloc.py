"""kv4_attention_noalloc: the attention entry point for callers that cannot
allocate device memory where they call us (their runtime offers no allocator
at that point, or the step must not touch one).  It must give the same
results as kv4_attention, which takes a caller-provided workspace, call
after call, while allocating nothing itself.

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import ATOL, f32, kv_inputs

pytestmark = pytest.mark.gpu


def _cache(b, hkv, s, d, gs, seed):
    from kvint4.cache import Int4KVStore
    k, v = kv_inputs(b, hkv, s, d, dtype=torch.bfloat16, seed=seed, device="cuda")
    store = Int4KVStore(gs)
    store.append(k, v, 0)
    return store.layer(0).views()


def _noalloc(q, cache, out, gs, causal=False, stream=None):
    """Call the allocation-free entry point straight through the C ABI."""
    from kvint4 import _lib, ops
    L = _lib.lib()
    ds = [ops.desc(t) for t in (q, *cache, out)]
    st = stream if stream is not None else torch.cuda.current_stream()
    return L.kv4_attention_noalloc(*[ctypes.byref(x) for x in ds], gs, int(causal),
                                   ctypes.c_float(0.0), ctypes.c_void_p(st.cuda_stream))


@pytest.mark.parametrize("order", [0, 1])
def test_noalloc_matches_workspace_entry_point_two_calls(order):
    from kvint4 import ops
    shapes = [(2, 8, 2, 3000, 128, 32, 1), (3, 32, 8, 2000, 128, 64, 2)]
    if order:
        shapes = shapes[::-1]
    for (b, hq, hkv, s, d, gs, seed) in shapes:  # two calls in a row, different geometry
        cache = _cache(b, hkv, s, d, gs, seed)
        q = torch.randn(b, hq, 1, d, device="cuda", generator=torch.Generator(
            device="cuda").manual_seed(seed)).to(torch.bfloat16)
        plan = ops.plan(q, *cache, torch.empty_like(q), gs)
        assert plan.path == 1 and plan.workspace_bytes > 0  # the scratch-using kernel
        ref = torch.empty_like(q)
        ops.attention_into(q, *cache, ref, gs)
        for _ in range(2):
            out = torch.full_like(q, float("nan"))
            assert _noalloc(q, cache, out, gs) == 0
            torch.cuda.synchronize()
            # the same plan and kernel as the workspace entry point: bit-identical
            assert torch.equal(out, ref)


def test_noalloc_causal_multi_query_matches_workspace_entry_point():
    from kvint4 import ops
    cache = _cache(2, 4, 2500, 128, 32, 5)
    q = torch.randn(2, 16, 2, 128, device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(5)).to(torch.bfloat16)
    ref = torch.empty_like(q)
    ops.attention_into(q, *cache, ref, 32, True)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _noalloc(q, cache, out, 32, causal=True) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_rejects_a_stream_of_another_device():
    from kvint4 import _lib
    cache = _cache(2, 2, 3000, 128, 32, 1)
    q = torch.randn(2, 8, 1, 128, device="cuda:0").to(torch.bfloat16)
    out = torch.empty_like(q)
    other = torch.cuda.Stream(device="cuda:1")
    with torch.cuda.device(0):
        assert _noalloc(q, cache, out, 32, stream=other) == _lib.KV4_ERR_INVALID


def test_noalloc_scratch_covers_default_plans():
    """A plan's partials are bounded by one wave of CTAs, so the fixed area
    (4 MiB, the last 64 KiB for counters) holds every default plan; the
    entry point returns KV4_ERR_SCRATCH_LIMIT otherwise."""
    from kvint4 import _lib, ops
    limit = (4 << 20) - (64 << 10)
    for (b, hq, hkv, s, d) in [(1, 64, 8, 131072, 256), (1, 32, 8, 131072, 128),
                               (16, 32, 8, 4096, 128), (4, 8, 1, 65536, 64)]:
        q = torch.empty(b, hq, 1, d, device="cuda", dtype=torch.bfloat16)
        kp = torch.empty(b, hkv, s, d // 2, device="cuda", dtype=torch.uint8)
        ks = torch.empty(b, hkv, s, d // 32, device="cuda", dtype=torch.bfloat16)
        plan = ops.plan(q, kp, ks, kp, ks, q, 32)
        assert plan.workspace_bytes <= limit, (b, hq, hkv, s, d, plan.workspace_bytes)
    assert b"scratch" in _lib.lib().kv4_strerror(_lib.KV4_ERR_SCRATCH_LIMIT)
