"""Parity against the reference's OWN GPU kernels, run on the same B200.

The reference's Triton quantizer (``kernels/llama3/quantize.py:27-75``, the
default HALF_AWAY rounding of this library) and its fused GQA decode
attention (``kernels/llama3/attention_quant.py:24-286``), plus the GPT-2
copies, are loaded unmodified from ``oracle/_ref`` (staged by
``oracle/ref_recipe.py``) and compared with this library on identical
inputs:

* codes and scales: bit-exact (golden inputs, 10^7 random values per dtype,
  rows of exact .5 ties);
* attention: max-abs 2e-2 for bf16 outputs; 1e-3 for fp32 with the
  reference's ``tl.dot`` in IEEE fp32 (``TRITON_F32_DEFAULT=ieee``).
"""

from __future__ import annotations

import math
import os

os.environ.setdefault("TRITON_F32_DEFAULT", "ieee")  # before any reference kernel compiles

import numpy as np
import pytest
import torch

from golden_io import cases, load
from helpers import kv_inputs
from oracle import triton_ref

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not triton_ref.available(),
                       reason="reference kernels not staged (oracle/ref_recipe.py)"),
]

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


def _same_codes(ours, ref):
    (p, s), (rp, rs) = ours, ref
    assert p.shape == rp.shape and s.shape == rs.shape and s.dtype == rs.dtype
    neq = (p != rp)
    assert int(neq.sum()) == 0, f"{int(neq.sum())} packed bytes differ of {p.numel()}"
    assert torch.equal(s.view(torch.uint8) if s.dtype != torch.float32 else s.view(torch.int32),
                       rs.view(torch.uint8) if rs.dtype != torch.float32 else rs.view(torch.int32))


@pytest.mark.parametrize("case", [c for c in cases(Q) if int(Q[c + ".group_size"]) % 2 == 0])
def test_quantize_matches_triton_on_golden_inputs(case):
    flavour = case.split(".")[0]
    x = _x_from_golden(case)
    gs = int(Q[case + ".group_size"])
    if flavour == "llama3":
        from kernels.llama3.quantize import quantize_int4
        ref = triton_ref.llama3_quantize()._quantize_int4_triton
    else:
        from kernels.gpt2.quantize import quantize_int4
        ref = triton_ref.gpt2_quantize().quantize_int4
    if x.numel() == 0 or x.shape[-1] == 0:
        pytest.skip("empty input takes the reference's torch path")
    _same_codes(quantize_int4(x, group_size=gs), ref(x, gs))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_matches_triton_1e7_random(dtype, gs):
    from kernels.llama3.quantize import quantize_int4
    ref = triton_ref.llama3_quantize()._quantize_int4_triton
    g = torch.Generator(device="cuda").manual_seed(gs)
    # 10^7 values: rows of N(0,1) with per-row magnitudes over 2^-10..2^10
    x = torch.randn(78125, 128, device="cuda", generator=g)
    x = x * torch.exp2(torch.randint(-10, 11, (78125, 1), device="cuda", generator=g).float())
    x = x.to(dtype)
    _same_codes(quantize_int4(x, group_size=gs), ref(x, gs))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quantize_matches_triton_on_exact_ties(dtype):
    """Rows whose quotients x / scale land exactly on k + 0.5."""
    from kernels.llama3.quantize import quantize_int4
    ref = triton_ref.llama3_quantize()._quantize_int4_triton
    rows = []
    for e in range(-6, 7):
        s = 2.0 ** e  # scale = max/7 with max = 7 * s exact in every dtype
        half = (torch.arange(-15, 15).float() + 0.5).clamp(-7.5, 6.5)  # k + 0.5
        row = torch.cat([torch.tensor([7.0]), half[:31]]) * s
        rows.append(row)
        rows.append(-row)
    x = torch.stack(rows).to(dtype).cuda()
    _same_codes(quantize_int4(x, group_size=32), ref(x, 32))


def _cfg(b, hq, hkv, s, d=128, seed=0, qdt=torch.bfloat16, sdt=torch.bfloat16):
    from kernels.llama3.quantize import quantize_int4
    k, v = kv_inputs(b, hkv, s, d, dtype=sdt, seed=seed, device="cuda")
    g = torch.Generator().manual_seed(seed + 1)
    q = torch.randn(b, hq, 1, d, generator=g).to(qdt).cuda()
    kp, ks = quantize_int4(k, group_size=32)
    vp, vs = quantize_int4(v, group_size=32)
    return q, kp, ks, vp, vs


@pytest.mark.parametrize("shape", [
    (16, 32, 8, 4096),    # Llama-3.1-8B decode, batch 16
    (1, 32, 8, 16384),    # batch-1 long context
    (1, 32, 8, 131072),
    (4, 64, 8, 2048),     # 70B head layout (GQA 8)
])
def test_attention_matches_triton_bf16(shape):
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    b, hq, hkv, s = shape
    q, kp, ks, vp, vs = _cfg(b, hq, hkv, s)
    ours = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv)
    ref = triton_ref.llama3_attention().attention_forward_quant_gqa(
        q, kp, ks, vp, vs, n_q_heads=hq, n_kv_heads=hkv, group_size=32)
    err = (ours.float() - ref.float()).abs().max().item()
    assert err <= 2e-2, err


def test_attention_matches_triton_fp32_ieee():
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    q, kp, ks, vp, vs = _cfg(2, 32, 8, 1024, qdt=torch.float32, sdt=torch.float32)
    ours = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8)
    ref = triton_ref.llama3_attention().attention_forward_quant_gqa(
        q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8, group_size=32)
    err = (ours - ref).abs().max().item()
    assert err <= 1e-3, err


def test_attention_causal_prefill_block_matches_triton():
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from kernels.llama3.quantize import quantize_int4
    k, v = kv_inputs(2, 4, 300, 128, seed=3, device="cuda")
    g = torch.Generator().manual_seed(4)
    q = torch.randn(2, 16, 37, 128, generator=g).to(torch.bfloat16).cuda()
    kp, ks = quantize_int4(k, group_size=32)
    vp, vs = quantize_int4(v, group_size=32)
    ours = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=16, n_kv_heads=4,
                                       is_causal=True)
    ref = triton_ref.llama3_attention().attention_forward_quant_gqa(
        q, kp, ks, vp, vs, n_q_heads=16, n_kv_heads=4, group_size=32, is_causal=True)
    err = (ours.float() - ref.float()).abs().max().item()
    assert err <= 2e-2, err


def test_gpt2_config1_attention_matches_triton():
    """GPT-2-small decode: fp32 q [4, 12, 1, 64], K/V [4, 12, 1024, 64], fp16 scales."""
    from kernels.gpt2.attention_quant import attention_forward_quant
    from kernels.gpt2.quantize import quantize_int4
    g = torch.Generator().manual_seed(0)
    q = torch.randn(4, 12, 1, 64, generator=g).cuda()
    k = torch.randn(4, 12, 1024, 64, generator=g).cuda()
    v = torch.randn(4, 12, 1024, 64, generator=g).cuda()
    kp, ks = quantize_int4(k, group_size=32)
    vp, vs = quantize_int4(v, group_size=32)
    rq = triton_ref.gpt2_quantize().quantize_int4
    _same_codes((kp, ks), rq(k, 32))
    ours = attention_forward_quant(q, kp, ks, vp, vs, group_size=32)
    ref = triton_ref.gpt2_attention().attention_forward_quant(q, kp, ks, vp, vs, group_size=32)
    err = (ours - ref).abs().max().item()
    assert err <= 1e-3, err
