"""Fused attention over the INT4-packed K/V cache for GPT-2 (MHA).

Drop-in for the reference's ``kernels/gpt2/attention_quant.py``
(``attention_forward_quant`` :140-248): same signature and ``ValueError``
checks; q must be fp16/fp32 and the cache has as many heads as q.  Runs the
same sm_100a kernel as the Llama path with a GQA ratio of 1.
"""

from __future__ import annotations

import math

import torch

from kvint4 import frontend


def attention_forward_quant(
    q: torch.Tensor,
    k_packed: torch.Tensor,
    k_scales: torch.Tensor,
    v_packed: torch.Tensor,
    v_scales: torch.Tensor,
    *,
    group_size: int = 32,
    is_causal: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Scaled dot-product attention using packed INT4 K/V cache."""
    if group_size <= 0:
        raise ValueError("group_size must be > 0")
    if not q.is_cuda:
        raise ValueError("attention_forward_quant expects CUDA tensors")
    if q.dtype not in (torch.float16, torch.float32):
        raise ValueError("q must be float16 or float32")
    if k_packed.dtype != torch.uint8 or v_packed.dtype != torch.uint8:
        raise ValueError("k_packed and v_packed must be uint8")
    if k_scales.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise ValueError("k_scales must be floating point")
    if v_scales.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise ValueError("v_scales must be floating point")
    if not all(t.is_cuda for t in (k_packed, k_scales, v_packed, v_scales)):
        raise ValueError("attention_forward_quant expects CUDA tensors")
    if k_packed.shape != v_packed.shape:
        raise ValueError("k_packed and v_packed must have the same shape")
    if k_scales.shape != v_scales.shape:
        raise ValueError("k_scales and v_scales must have the same shape")
    if k_packed.shape[:-1] != k_scales.shape[:-1]:
        raise ValueError("packed/scales leading dimensions must match")
    b, h, sq, d = q.shape
    if k_packed.shape[:2] != (b, h):
        raise ValueError("batch/head dimensions must match q")
    if k_scales.shape[:2] != (b, h):
        raise ValueError("batch/head dimensions must match q")
    if k_packed.shape[-1] < math.ceil(d / 2):
        raise ValueError("packed last dimension is too small for q d_head")
    if k_scales.shape[-1] < math.ceil(d / group_size):
        raise ValueError("scales last dimension is too small for q d_head/group_size")
    if k_scales.dtype != v_scales.dtype:
        v_scales = v_scales.to(k_scales.dtype)
    return frontend.attention(q, k_packed, k_scales, v_packed, v_scales, n_q_heads=h,
                              n_kv_heads=h, group_size=group_size, is_causal=is_causal, out=out)
