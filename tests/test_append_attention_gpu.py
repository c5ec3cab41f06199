"""kv4_append_attention: quantize-on-append fused into the decode attention.

The fused call must leave the cache bit-identical to the quantize kernel's
append (``kv4_append_kv``) and give bit-identical attention output to
append-then-``kv4_attention`` on the same inputs, on every fast-path shape
and at every position of the new row inside a 128-token tile (first row,
last row, split-K part boundaries, several column chunks per KV head).  Routes that are not
fused (several new rows, generic kernel, strided new rows) must give the
same results too.  One case is also checked against the CPU oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import ATOL, f32, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


def _caches(b, hkv, s_old, d, gs, dt, sdt, seed, cap=None):
    """Two identical capacity-buffer caches holding s_old tokens."""
    from kvint4.cache import Int4KVStore
    k, v = kv_inputs(b, hkv, s_old, d, dtype=dt, seed=seed, device="cuda")
    out = []
    for _ in range(2):
        st = Int4KVStore(gs, scale_dtype=sdt, capacity=cap)
        if s_old:
            st.append(k, v, 0)
        else:
            st._layers[0] = st._reserve(k[:, :, :1], v[:, :, :1], 0)
        out.append(st)
    return out


def _new_rows(b, hq, hkv, n, d, dt, seed):
    g = torch.Generator().manual_seed(seed + 7)
    q = torch.randn(b, hq, 1, d, generator=g).to(dt).cuda()
    kn = (torch.randn(b, hkv, n, d, generator=g) * 3).to(dt).cuda()
    vn = torch.randn(b, hkv, n, d, generator=g).to(dt).cuda()
    return q, kn, vn


def _both(b, hq, hkv, s_old, d, gs, dt=torch.bfloat16, sdt=None, n=1, seed=0, tie=0,
          causal=False, strided=False, **kw):
    from kvint4 import ops
    a, f = _caches(b, hkv, s_old, d, gs, dt, sdt, seed)
    q, kn, vn = _new_rows(b, hq, hkv, n, d, dt, seed)
    if strided:  # new rows with a non-unit dim stride
        kn = torch.stack([kn, kn], -1)[..., 0]
        vn = torch.stack([vn, vn], -1)[..., 0]
        assert kn.stride(3) == 2
    # reference route: the quantize kernel's append, then attention
    a.tie_mode = tie
    a.append(kn, vn, 0)
    ref = torch.empty_like(q)
    views_a = a.layer(0).views()
    ops.attention_into(q, *views_a, ref, gs, causal, **kw)
    # fused route
    lay = f.layer(0)
    S = lay.seq_len + n
    f._reserve(kn, vn, 0)
    lay = f.layer(0)
    views_f = (lay.k_packed_buf[:, :, :S], lay.k_scales_buf[:, :, :S],
               lay.v_packed_buf[:, :, :S], lay.v_scales_buf[:, :, :S])
    out = torch.full_like(q, float("nan"))
    ops.append_attention_into(q, kn, vn, *views_f, out, gs, causal, tie, **kw)
    torch.cuda.synchronize()
    p = ops.plan(q, *views_f, out, gs, causal, **kw)
    return q, views_a, views_f, ref, out, p


def _assert_same(views_a, views_f, ref, out):
    for x, y in zip(views_a, views_f):
        assert torch.equal(x, y), "cache bytes differ from the quantize kernel's append"
    assert torch.equal(out, ref), "output differs from append-then-attention"


@pytest.mark.parametrize("d,gs", [(128, 32), (128, 64), (128, 128), (64, 32), (64, 64),
                                  (256, 32), (256, 128)])
@pytest.mark.parametrize("qdt", [torch.bfloat16, torch.float16, torch.float32])
def test_fused_append_bit_identical(d, gs, qdt):
    q, va, vf, ref, out, p = _both(2, 8, 2, 300, d, gs, dt=qdt)
    assert p.path == 1
    _assert_same(va, vf, ref, out)


@pytest.mark.parametrize("s_old", [0, 1, 126, 127, 128, 255, 1000, 4095])
def test_fused_append_every_tile_position(s_old):
    """New row as the only row, first / last row of a tile, mid-tile."""
    q, va, vf, ref, out, p = _both(3, 32, 8, s_old, 128, 32, seed=s_old)
    assert p.path == 1
    _assert_same(va, vf, ref, out)


@pytest.mark.parametrize("tpc", [1, 2, 3])
def test_fused_append_split_parts(tpc):
    """The new row's tile sits in the last split-K part; several parts per unit."""
    q, va, vf, ref, out, p = _both(1, 8, 1, 2000, 128, 32, tiles_per_cta=tpc, seed=5)
    assert p.path == 1 and p.max_parts > 1
    _assert_same(va, vf, ref, out)


def test_fused_append_several_column_chunks():
    """GQA ratio 16: two column chunks (units) stage the new row; one writes it."""
    q, va, vf, ref, out, p = _both(2, 32, 2, 700, 128, 32, seed=3)
    assert p.units == 2 * 2 * 2
    _assert_same(va, vf, ref, out)


@pytest.mark.parametrize("tie", [0, 1])
@pytest.mark.parametrize("sdt", [torch.float32, torch.float16])
def test_fused_append_tie_and_scale_dtypes(tie, sdt):
    q, va, vf, ref, out, p = _both(2, 8, 2, 513, 128, 32, sdt=sdt, tie=tie, seed=11)
    assert p.path == 1
    _assert_same(va, vf, ref, out)


def test_fused_append_exact_ties_both_modes_differ():
    """Values at exact .5 code ties: each tie mode matches its own append kernel."""
    from kvint4 import ops
    from kvint4.cache import Int4KVStore
    b, hkv, d, gs = 1, 1, 128, 32
    # every group holds 7.0, so its scale is exactly 1 and x.5 values are code ties
    base = torch.tensor([7.0, 2.5, -3.5, 0.5, -1.5, 1.5, -0.5, 3.5]).repeat(d // 8)
    kn = base.view(1, 1, 1, d).cuda()
    q = torch.randn(1, 4, 1, d).cuda()
    got = {}
    for tie in (0, 1):
        st = Int4KVStore(gs, tie_mode=tie)
        k, v = kv_inputs(b, hkv, 10, d, dtype=torch.float32, seed=1, device="cuda")
        st.append(k, v, 0)
        out = torch.empty_like(q)
        st.append_attend(q, kn, kn, 0, out, n_q_heads=4, n_kv_heads=1)
        ref_st = Int4KVStore(gs, tie_mode=tie)
        ref_st.append(k, v, 0)
        ref_st.append(kn, kn, 0)
        for x, y in zip(st.layer(0).views(), ref_st.layer(0).views()):
            assert torch.equal(x, y)
        got[tie] = st.layer(0).views()[0][0, 0, -1].clone()
    assert not torch.equal(got[0], got[1])  # the ties are real


@pytest.mark.parametrize("case", ["n3", "generic", "strided", "odd_group"])
def test_unfused_routes_match(case):
    if case == "n3":
        q, va, vf, ref, out, p = _both(2, 8, 2, 300, 128, 32, n=3)
    elif case == "generic":
        q, va, vf, ref, out, p = _both(2, 8, 2, 300, 128, 32, force_generic=True)
        assert p.path == 2
    elif case == "strided":
        q, va, vf, ref, out, p = _both(2, 8, 2, 300, 128, 32, strided=True)
    else:
        q, va, vf, ref, out, p = _both(2, 8, 2, 300, 70, 5)
        assert p.path == 2
    _assert_same(va, vf, ref, out)


def test_fused_append_matches_oracle():
    q, va, vf, ref, out, p = _both(2, 32, 8, 999, 128, 32, seed=21)
    exp = oracle_attention(q, *vf, n_q_heads=32, n_kv_heads=8, group_size=32)
    np.testing.assert_allclose(f32(out), exp, atol=ATOL[torch.bfloat16], rtol=0)


def test_append_attend_shape_errors():
    from kvint4 import _lib, ops
    a, f = _caches(1, 2, 10, 128, 32, torch.bfloat16, None, 0)
    q, kn, vn = _new_rows(1, 8, 2, 1, 128, torch.bfloat16, 0)
    lay = f.layer(0)
    views = (lay.k_packed_buf[:, :, :11], lay.k_scales_buf[:, :, :11],
             lay.v_packed_buf[:, :, :11], lay.v_scales_buf[:, :, :11])
    out = torch.empty_like(q)
    with pytest.raises(_lib.Kv4Error):  # wrong head count of the new rows
        ops.append_attention_into(q, kn[:, :1], vn[:, :1], *views, out, 32)
    with pytest.raises(_lib.Kv4Error):  # more new rows than the views hold
        big = kn.expand(1, 2, 12, 128)
        ops.append_attention_into(q, big, big, *views, out, 32)
    with pytest.raises(_lib.Kv4Error):  # bad tie mode
        ops.append_attention_into(q, kn, vn, *views, out, 32, False, 7)
