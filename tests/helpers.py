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
    [0.5, 8] (BASELINE config 2's outlier channels)."""
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
