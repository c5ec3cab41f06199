"""Pin the CPU oracle against the golden vectors produced by the reference's
own torch functions (``tests/golden/make_golden.py``).  CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from golden_io import cases, load, to_f32
from oracle import int4_oracle as orc

Q = load("quant_cases.npz")
A = load("attn_cases.npz")


@pytest.mark.parametrize("case", cases(Q))
def test_oracle_quantize_half_even_matches_reference_torch(case):
    x = to_f32(Q[case + ".x"], str(Q[case + ".x_dtype"]))
    gs = int(Q[case + ".group_size"])
    sdt = str(Q[case + ".scale_dtype"])
    packed, scales = orc.quantize_int4(x, gs, orc.TIE_HALF_EVEN, scale_dtype=sdt)
    assert packed.shape == Q[case + ".packed"].shape
    np.testing.assert_array_equal(packed, Q[case + ".packed"])
    np.testing.assert_array_equal(scales, to_f32(Q[case + ".scales"], sdt))


@pytest.mark.parametrize("case", cases(Q))
def test_oracle_dequantize_matches_reference_torch(case):
    gs = int(Q[case + ".group_size"])
    sdt = str(Q[case + ".scale_dtype"])
    x = to_f32(Q[case + ".x"], str(Q[case + ".x_dtype"]))
    deq = orc.dequantize_int4(Q[case + ".packed"], to_f32(Q[case + ".scales"], sdt), gs,
                              x.shape[-1])
    ref = to_f32(Q[case + ".deq"], str(Q[case + ".deq_dtype"]))
    ref_dt = str(Q[case + ".deq_dtype"])
    np.testing.assert_array_equal(orc.round_to(deq, ref_dt), ref)


@pytest.mark.parametrize("case", cases(Q))
def test_oracle_half_away_differs_only_on_ties(case):
    """HALF_AWAY (Triton formula) and HALF_EVEN (torch) differ only where
    x/scale is an exact .5 tie with an even floor -- the reference's own test
    tolerates exactly this (``tests/gpt2/test_quantize.py:55-56``)."""
    x = to_f32(Q[case + ".x"], str(Q[case + ".x_dtype"]))
    gs = int(Q[case + ".group_size"])
    pa, sa = orc.quantize_int4(x, gs, orc.TIE_HALF_AWAY)
    pe, se = orc.quantize_int4(x, gs, orc.TIE_HALF_EVEN)
    np.testing.assert_array_equal(sa, se)
    ca = np.stack([pa & 15, pa >> 4], -1).reshape(pa.shape[:-1] + (-1,)).astype(int)
    ce = np.stack([pe & 15, pe >> 4], -1).reshape(pe.shape[:-1] + (-1,)).astype(int)
    diff = ca != ce
    assert np.all(np.abs(ca - ce)[diff] == 1)


def test_oracle_tie_rounding_known_answers():
    # scale = 7/7 = 1 so x/scale == x exactly
    row = np.zeros((1, 32), np.float32)
    row[0, :6] = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5]
    row[0, 31] = 7.0
    pe, _ = orc.quantize_int4(row, 32, orc.TIE_HALF_EVEN)
    pa, _ = orc.quantize_int4(row, 32, orc.TIE_HALF_AWAY)
    # half-even: 0, -0, 2, -2, 2, -2 ; +8 bias
    assert list(pe[0, :3]) == [8 | (8 << 4), 10 | (6 << 4), 10 | (6 << 4)]
    # half-away: 1, -1, 2, -2, 3, -3
    assert list(pa[0, :3]) == [9 | (7 << 4), 10 | (6 << 4), 11 | (5 << 4)]
    # the survey's torch example: [0.5, -0.5, 1.5, -1.5, 0..., 7.0] -> bytes [136, 106]
    assert list(pe[0, :2]) == [136, 106]
    assert pa[0, 0] == 121


@pytest.mark.parametrize("case", cases(A))
def test_oracle_attention_matches_reference(case):
    b, hq, hkv, sq, sk, d, gs, causal = (int(v) for v in A[case + ".meta"])
    sdt = str(A[case + ".scale_dtype"])
    q = to_f32(A[case + ".q"], str(A[case + ".q_dtype"]))
    out = orc.quantized_attention(
        q, A[case + ".k_packed"], to_f32(A[case + ".k_scales"], sdt),
        A[case + ".v_packed"], to_f32(A[case + ".v_scales"], sdt),
        n_q_heads=hq, n_kv_heads=hkv, group_size=gs, is_causal=bool(causal))
    np.testing.assert_allclose(out, A[case + ".out_ref_f32"], atol=2e-5, rtol=1e-5)
    if case + ".out_sdpa_f32" in A:
        np.testing.assert_allclose(out, A[case + ".out_sdpa_f32"], atol=2e-5, rtol=1e-5)


def test_oracle_lse_combine_equals_unsharded():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 8, 3, 64))
    k = rng.standard_normal((2, 2, 50, 64))
    v = rng.standard_normal((2, 2, 50, 64))
    full = orc.attention(q, k, v, n_q_heads=8, n_kv_heads=2, is_causal=True)
    parts = [(0, 13), (13, 31), (31, 48), (48, 50)]
    os_, ls_ = [], []
    for a, bnd in parts:
        o, l = orc.partial_attention(q, k[:, :, a:bnd], v[:, :, a:bnd], n_q_heads=8,
                                     n_kv_heads=2, is_causal=True, k_offset=a, sk_total=50)
        os_.append(o)
        ls_.append(l)
    np.testing.assert_allclose(orc.lse_combine(os_, ls_), full, atol=1e-12)
