"""Shared implementation behind the reference-shaped ``kernels.*`` modules.

Each function here allocates the outputs with the torch caching allocator on
the input's device and hands pointers/strides to ``libkvint4.so``.  Every path
is CUDA: CPU tensors raise ``ValueError`` (there is no CPU implementation in
the product; the CPU formulation lives in the test oracle only).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _lib, ops

FLOATS = (torch.bfloat16, torch.float16, torch.float32)

# the fused kernel takes up to 8 column chunks of 8 (head, query row) pairs per
# KV head; longer query blocks use the generic kernel while small, and the
# dequantize + flash-SDPA route when large (prefill).
FUSED_MAX_COLS = 64
GENERIC_MAX_WORK = 1 << 24  # sq * sk per (b, head) below which the generic kernel is used


def _as4d(t: torch.Tensor) -> torch.Tensor:
    """View ``t`` with exactly 4 dims (leading dims merged when possible)."""
    if t.dim() <= 4:
        return t
    lead = math.prod(t.shape[:-3])
    return t.reshape(lead, *t.shape[-3:])


def _need_cuda(name: str, *ts: torch.Tensor) -> None:
    if not all(t.is_cuda for t in ts):
        raise ValueError(f"{name} expects CUDA tensors")


def quantize(x: torch.Tensor, group_size: int, scale_dtype: torch.dtype,
             tie_mode: int = _lib.TIE_HALF_AWAY, name: str = "quantize_int4"):
    _need_cuda(name, x)
    d = x.shape[-1]
    ng = math.ceil(d / group_size)
    pw = ng * ((group_size + 1) // 2)
    lead = tuple(x.shape[:-1])
    packed = torch.empty(*lead, pw, dtype=torch.uint8, device=x.device)
    scales = torch.empty(*lead, ng, dtype=scale_dtype, device=x.device)
    if x.numel() == 0 or d == 0:
        return packed, scales
    x4 = x.reshape(1, d) if x.dim() == 1 else _as4d(x)
    p4 = packed.reshape(1, pw) if x.dim() == 1 else _as4d(packed)
    s4 = scales.reshape(1, ng) if x.dim() == 1 else _as4d(scales)
    ops.quantize_into(x4, p4, s4, group_size, tie_mode)
    return packed, scales


def dequantize(packed: torch.Tensor, scales: torch.Tensor, group_size: int, d_out: int,
               out_dtype: torch.dtype, name: str = "dequantize_int4") -> torch.Tensor:
    _need_cuda(name, packed, scales)
    ng = scales.shape[-1]
    pw = packed.shape[-1]
    if ng > 0 and (2 * pw) % ng == 0 and (2 * pw) // ng < group_size:
        raise ValueError("packed has insufficient width for the provided group_size")
    if ng > 0 and (2 * pw) % ng != 0:
        raise ValueError("packed width is not a whole number of groups")
    d_out = min(d_out, ng * group_size)
    lead = tuple(packed.shape[:-1])
    out = torch.empty(*lead, d_out, dtype=out_dtype, device=packed.device)
    if out.numel() == 0:
        return out
    if packed.dim() == 1:
        ops.dequantize_into(packed.reshape(1, pw), scales.reshape(1, ng), out.reshape(1, d_out),
                            group_size)
    else:
        ops.dequantize_into(_as4d(packed), _as4d(scales), _as4d(out), group_size)
    return out


def attention(q, k_packed, k_scales, v_packed, v_scales, *, n_q_heads: int, n_kv_heads: int,
              group_size: int, is_causal: bool, out: torch.Tensor | None = None,
              **kernel_opts) -> torch.Tensor:
    """Attention over the packed cache; ``out`` may be any-strided [B, Hq, sq, d]."""
    b, hq, sq, d = q.shape
    sk = k_packed.shape[2]
    if out is None:
        out = torch.empty(b, hq, sq, d, dtype=q.dtype, device=q.device)
    if q.numel() == 0:
        return out
    ratio = n_q_heads // n_kv_heads
    if sq * ratio > FUSED_MAX_COLS and sq * sk > GENERIC_MAX_WORK and not kernel_opts:
        _prefill_sdpa(q, k_packed, k_scales, v_packed, v_scales, group_size, is_causal, out)
        return out
    ops.attention_into(q, k_packed, k_scales, v_packed, v_scales, out, group_size, is_causal,
                       **kernel_opts)
    return out


def _prefill_sdpa(q, kp, ks, vp, vs, group_size, is_causal, out):
    """Long query blocks (prefill): dequantize K/V once with the CUDA kernel,
    then flash attention with bottom-right causal alignment."""
    d = q.shape[-1]
    k = dequantize(kp, ks, group_size, d, q.dtype)
    v = dequantize(vp, vs, group_size, d, q.dtype)
    sq, sk = q.shape[2], k.shape[2]
    kw = {}
    if is_causal and sq == sk:
        kw["is_causal"] = True
    elif is_causal:
        from torch.nn.attention.bias import causal_lower_right
        kw["attn_mask"] = causal_lower_right(sq, sk)
    res = F.scaled_dot_product_attention(q, k, v, enable_gqa=q.shape[1] != k.shape[1], **kw)
    out.copy_(res)
