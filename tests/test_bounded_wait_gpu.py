"""A bounded mbarrier wait that runs out, made on purpose without faulting
the GPU: the test knob debug_drop_last_tile makes the producer skip the
load of each CTA's last tile and shortens the wait limit to 16 polls of at
most 1 ms.  The kernel must set the device error word (bit 1), drain the
loads it did issue, return, and leave the context usable: the next call is
correct and the error word is clean again."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import f32, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,hkv,s", [(2, 2, 3000), (1, 8, 20000)])
def test_expired_wait_sets_error_word_and_context_survives(b, hkv, s):
    from kvint4 import ops
    from kvint4.cache import Int4KVStore
    k, v = kv_inputs(b, hkv, s, 128, device="cuda", seed=8)
    st = Int4KVStore(32)
    st.append(k, v, 0)
    views = st.layer(0).views()
    q = torch.randn(b, 4 * hkv, 1, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    assert ops.device_error() == 0
    assert ops.plan(q, *views, out, 32).path == 1
    ops.attention_into(q, *views, out, 32, debug_drop_last_tile=True)
    err = ops.device_error()  # synchronizes; the kernel returned
    assert err & 1, err
    assert ops.device_error() == 0  # read-and-clear
    ops.attention_into(q, *views, out, 32)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = oracle_attention(q, *views, n_q_heads=4 * hkv, n_kv_heads=hkv, group_size=32)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)
