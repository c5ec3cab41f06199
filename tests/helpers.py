"""Test helpers: seeded inputs in the reference's distributions and the CPU
oracle results for them."""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import int4_oracle as orc

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DT_NAME = {v: k for k, v in TORCH_DT.items()}


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def kv_inputs(b, hkv, s, d, dtype=torch.bfloat16, seed=0, outliers=True, device="cpu"):
    """K, V ~ N(0,1) with every K channel scaled by a factor log-uniform in
    [0.5, 8] (the outlier channels of the Llama-3.1-8B benchmark inputs)."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(b, hkv, s, d, generator=g)
    if outliers:
        f = torch.exp(torch.empty(d).uniform_(math.log(0.5), math.log(8.0), generator=g))
        k = k * f
    v = torch.randn(b, hkv, s, d, generator=g)
    return k.to(dtype).to(device), v.to(dtype).to(device)


def oracle_quant(x: torch.Tensor, group_size: int, tie: int, scale_dtype: torch.dtype):
    p, s = orc.quantize_int4(f32(x), group_size, tie, scale_dtype=DT_NAME[scale_dtype])
    return p, s


def oracle_attention(q, kp, ks, vp, vs, *, n_q_heads, n_kv_heads, group_size, is_causal=False):
    return orc.quantized_attention(f32(q), kp.cpu().numpy(), f32(ks), vp.cpu().numpy(), f32(vs),
                                   n_q_heads=n_q_heads, n_kv_heads=n_kv_heads,
                                   group_size=group_size, is_causal=is_causal)


# output tolerance of the fused kernel against the float64 oracle, per output dtype
ATOL = {torch.float32: 1e-3, torch.float16: 5e-3, torch.bfloat16: 2e-2}


def assert_codes_near_oracle(x: torch.Tensor, group_size: int, packed, scales):
    """Library codes in the default (reference Triton) mode against the
    oracle's IEEE restatement of the same formula.  The modes differ only
    in the last bit of the two fp32 divisions (PTX div.full.f32 vs div.rn),
    so: scales equal after rounding to their dtype, or 1 ulp of that dtype
    apart; codes equal except for elements whose IEEE quotient lies within
    1e-5 of a rounding boundary k + 0.5, or whose group scale differs, and
    those differ by exactly 1.  Bit-exactness of this mode is pinned against
    the reference's own Triton kernel on the GPU."""
    xs = f32(x).reshape(-1, x.shape[-1])
    sdt = DT_NAME[scales.dtype]
    p_ref, s_ref = orc.quantize_int4(xs, group_size, orc.TIE_HALF_AWAY, scale_dtype=sdt)
    p_got = packed.cpu().numpy().reshape(p_ref.shape)
    s_got = f32(scales).reshape(s_ref.shape)
    ulp = np.spacing(np.abs(s_ref).astype(np.float16 if sdt == "f16" else np.float32))
    if sdt == "bf16":
        ulp = np.abs(s_ref) * 2.0 ** -7
    s_diff = s_got != s_ref
    assert np.all(np.abs(s_got - s_ref)[s_diff] <= 1.01 * ulp[s_diff]), "scales too far apart"
    c_ref = np.stack([p_ref & 15, p_ref >> 4], -1).reshape(p_ref.shape[0], -1).astype(int)
    c_got = np.stack([p_got & 15, p_got >> 4], -1).reshape(p_got.shape[0], -1).astype(int)
    d = x.shape[-1]
    ng = s_ref.shape[-1]
    # IEEE quotients of the real columns, per group scale
    g_of = np.arange(d) // group_size
    col = (np.arange(d) // group_size) * (c_ref.shape[1] // ng) + np.arange(d) % group_size
    mx = np.zeros((xs.shape[0], ng), np.float32)
    for gi in range(ng):
        seg = np.abs(xs[:, gi * group_size:(gi + 1) * group_size])
        mx[:, gi] = seg.max(axis=1) if seg.shape[1] else 0
    scale32 = np.where(mx > 0, (mx / np.float32(7.0)).astype(np.float32), np.float32(1.0))
    q = xs / scale32[:, g_of]
    near = np.abs(np.abs(q) - np.floor(np.abs(q)) - 0.5) < 1e-5
    group_diff = s_diff[:, g_of]
    diff = c_got[:, col] != c_ref[:, col]
    assert np.all(np.abs(c_got[:, col] - c_ref[:, col])[diff] == 1), "codes differ by more than 1"
    assert np.all((near | group_diff)[diff]), "codes differ away from rounding boundaries"
