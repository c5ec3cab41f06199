"""Quantize / append / dequantize on the GPU vs the CPU oracle: bit-exact codes
and scales (both tie modes), exact dequantization."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import cases, load, to_f32
from helpers import DT_NAME, TORCH_DT, assert_codes_near_oracle, f32, oracle_quant
from oracle import int4_oracle as orc

pytestmark = pytest.mark.gpu

Q = load("quant_cases.npz")


def _x_from_golden(case):
    dt = str(Q[case + ".x_dtype"])
    raw = Q[case + ".x"]
    if dt == "bf16":
        t = torch.from_numpy(raw.astype(np.int16)).view(torch.bfloat16)
    elif dt == "f16":
        t = torch.from_numpy(raw.view(np.float16))
    else:
        t = torch.from_numpy(raw)
    return t.cuda()


@pytest.mark.parametrize("case", cases(Q))
def test_quantize_half_even_matches_golden_bit_exact(case):
    """HALF_EVEN on the GPU reproduces the reference torch path's bytes exactly."""
    flavour = case.split(".")[0]
    if flavour == "llama3":
        from kernels.llama3.quantize import TIE_HALF_EVEN, dequantize_int4, quantize_int4
    else:
        from kernels.gpt2.quantize import TIE_HALF_EVEN, dequantize_int4, quantize_int4
    x = _x_from_golden(case)
    gs = int(Q[case + ".group_size"])
    packed, scales = quantize_int4(x, group_size=gs, tie_mode=TIE_HALF_EVEN)
    np.testing.assert_array_equal(packed.cpu().numpy(), Q[case + ".packed"])
    sdt = str(Q[case + ".scale_dtype"])
    assert DT_NAME[scales.dtype] == sdt
    np.testing.assert_array_equal(f32(scales), to_f32(Q[case + ".scales"], sdt))
    # dequantize matches the reference torch dequant (in the reference's output dtype)
    if flavour == "llama3":
        deq = dequantize_int4(packed, scales, group_size=gs, d_head=x.shape[-1],
                              out_dtype=torch.float32)
    else:
        deq = dequantize_int4(packed, scales, group_size=gs, d_head=x.shape[-1])
    ref = to_f32(Q[case + ".deq"], str(Q[case + ".deq_dtype"]))
    np.testing.assert_array_equal(f32(deq), ref)


@pytest.mark.parametrize("case", cases(Q))
def test_quantize_half_away_ieee_matches_oracle_bit_exact(case):
    """Half-away rounding with IEEE divisions vs the oracle's restatement."""
    from kernels.llama3.quantize import TIE_HALF_AWAY_IEEE, quantize_int4
    x = _x_from_golden(case)
    gs = int(Q[case + ".group_size"])
    packed, scales = quantize_int4(x, group_size=gs, tie_mode=TIE_HALF_AWAY_IEEE)
    p_ref, s_ref = oracle_quant(x, gs, orc.TIE_HALF_AWAY, x.dtype)
    np.testing.assert_array_equal(packed.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(f32(scales), s_ref)


@pytest.mark.parametrize("case", cases(Q))
def test_quantize_default_mode_near_oracle(case):
    """The default mode (the reference Triton kernel's arithmetic) differs
    from the IEEE restatement only at rounding boundaries."""
    from kernels.llama3.quantize import quantize_int4
    x = _x_from_golden(case)
    if x.numel() == 0:
        pytest.skip("empty")
    gs = int(Q[case + ".group_size"])
    packed, scales = quantize_int4(x, group_size=gs)
    assert_codes_near_oracle(x, gs, packed, scales)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("tie", [2, 1])
def test_quantize_large_random_bit_exact(dtype, gs, tie):
    from kernels.llama3.quantize import quantize_int4
    g = torch.Generator().manual_seed(gs + tie)
    x = (torch.randn(4, 8, 257, 128, generator=g) * 3).to(TORCH_DT[dtype])
    x[0, 0, 0, :] = 0  # an all-zero row -> scale 1
    packed, scales = quantize_int4(x.cuda(), group_size=gs, tie_mode=tie)
    p_ref, s_ref = oracle_quant(x, gs, orc.TIE_HALF_AWAY if tie == 2 else tie, x.dtype)
    np.testing.assert_array_equal(packed.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(f32(scales), s_ref)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_quantize_default_mode_large_random_near_oracle(dtype):
    from kernels.llama3.quantize import quantize_int4
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(8, 4, 257, 128, generator=g) * 3).to(TORCH_DT[dtype])
    packed, scales = quantize_int4(x.cuda(), group_size=32)
    assert_codes_near_oracle(x, 32, packed, scales)


def test_quantize_strided_input_and_odd_shapes():
    from functools import partial

    from kernels.llama3.quantize import TIE_HALF_AWAY_IEEE
    from kernels.llama3.quantize import quantize_int4 as q4
    quantize_int4 = partial(q4, tie_mode=TIE_HALF_AWAY_IEEE)
    g = torch.Generator().manual_seed(5)
    base = torch.randn(3, 40, 6, 128, generator=g).to(torch.bfloat16).cuda()
    x = base.transpose(1, 2)  # [3, 6, 40, 128] non-contiguous, like k_proj(...).transpose(1, 2)
    packed, scales = quantize_int4(x, group_size=32)
    p_ref, s_ref = oracle_quant(x, 32, orc.TIE_HALF_AWAY, x.dtype)
    np.testing.assert_array_equal(packed.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(f32(scales), s_ref)
    # every-other-column view: scalar (non-vector) load path
    y = torch.randn(5, 140, generator=g).cuda()[:, ::2]
    packed, scales = quantize_int4(y, group_size=32)
    p_ref, s_ref = oracle_quant(y, 32, orc.TIE_HALF_AWAY, y.dtype)
    np.testing.assert_array_equal(packed.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(f32(scales), s_ref)
    # 1-D and 5-D inputs
    z = torch.randn(96, generator=g).cuda()
    p, s = quantize_int4(z, group_size=32)
    p_ref, s_ref = oracle_quant(z, 32, orc.TIE_HALF_AWAY, z.dtype)
    np.testing.assert_array_equal(p.cpu().numpy(), p_ref)
    w = torch.randn(2, 2, 2, 3, 64, generator=g).half().cuda()
    p, s = quantize_int4(w, group_size=64)
    p_ref, s_ref = oracle_quant(w, 64, orc.TIE_HALF_AWAY, w.dtype)
    np.testing.assert_array_equal(p.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(f32(s), s_ref)


def test_quantize_empty_and_zero():
    from kernels.gpt2.quantize import dequantize_int4, quantize_int4
    x = torch.zeros(1, 2, 4, 64, dtype=torch.float16, device="cuda")
    packed, scales = quantize_int4(x, group_size=32)
    x_hat = dequantize_int4(packed, scales, group_size=32, d_head=64)
    assert torch.equal(x_hat, x)
    e = torch.zeros(0, 3, 64, device="cuda")
    p, s = quantize_int4(e, group_size=32)
    assert p.shape == (0, 3, 32) and s.shape == (0, 3, 2)


def test_cache_append_matches_one_shot_quantize():
    """Prefill + token-by-token appends into the capacity buffer give the same
    bytes as quantizing the whole sequence at once (concat invariance,
    reference tests/llama3/test_quantize_sm70.py:145-168)."""
    from kernels.llama3.quantize import quantize_int4
    from models.llama3.kv_cache import QuantizedKVCache
    g = torch.Generator().manual_seed(11)
    k = torch.randn(2, 4, 150, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(2, 4, 150, 128, generator=g).to(torch.bfloat16).cuda()
    cache = QuantizedKVCache(group_size=32)
    cache.append(k[:, :, :37], v[:, :, :37], 0)
    for t in range(37, 150):
        cache.append(k[:, :, t:t + 1], v[:, :, t:t + 1], 0)
    assert cache.get_seq_length(0) == 150
    kp, ks, vp, vs = cache.get_quantized(0)
    kp1, ks1 = quantize_int4(k, 32)
    vp1, vs1 = quantize_int4(v, 32)
    assert torch.equal(kp, kp1) and torch.equal(ks, ks1)
    assert torch.equal(vp, vp1) and torch.equal(vs, vs1)
    assert kp.shape == (2, 4, 150, 64) and ks.shape == (2, 4, 150, 4)
    assert cache.nbytes() == 2 * (kp.numel() + ks.numel() * 2)


def test_dequantize_matches_oracle_all_dtypes():
    from kernels.llama3.quantize import dequantize_int4, quantize_int4
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 3, 33, 128, generator=g).cuda()
    for gs in (32, 64, 128):
        p, s = quantize_int4(x.to(torch.bfloat16), gs)
        ref = orc.dequantize_int4(p.cpu().numpy(), f32(s), gs, 128)
        for odt in (torch.float32, torch.float16, torch.bfloat16):
            out = dequantize_int4(p, s, group_size=gs, d_head=128, out_dtype=odt)
            assert out.dtype == odt
            np.testing.assert_array_equal(f32(out), orc.round_to(ref, DT_NAME[odt]))
