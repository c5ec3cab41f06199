"""Fused GQA attention over the INT4-packed K/V cache for Llama 3.1.

Drop-in for the reference's ``kernels/llama3/attention_quant.py``
(``attention_forward_quant_gqa`` :159-286): same signature, shapes, output
dtype and ``ValueError`` checks, in the same order.

    q:        [B, n_q,  sq, d_head]        bf16/fp16/fp32
    k_packed: [B, n_kv, sk, d_head // 2]   uint8
    k_scales: [B, n_kv, sk, d_head // G]   bf16/fp16/fp32
    v_packed, v_scales: as K

Query head ``h`` reads KV head ``h // (n_q // n_kv)``; with ``is_causal`` row
``i`` sees keys ``j <= sk - sq + i``.  Unlike the reference there are no
``.contiguous()`` copies: strided inputs (e.g. the cache's capacity views)
are read in place.  Decode and short query blocks run the sm_100a
tensor-core kernel (K/V dequantized in registers, one KV read per GQA group,
sequence split across the whole GPU, log-sum-exp merge); long prefill blocks
dequantize once and use flash SDPA.
"""

from __future__ import annotations

import math

import torch

from kvint4 import frontend

_Q_DTYPES = (torch.bfloat16, torch.float16, torch.float32)
_SCALE_DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def attention_forward_quant_gqa(
    q: torch.Tensor,
    k_packed: torch.Tensor,
    k_scales: torch.Tensor,
    v_packed: torch.Tensor,
    v_scales: torch.Tensor,
    *,
    n_q_heads: int,
    n_kv_heads: int,
    group_size: int = 32,
    is_causal: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused GQA scaled-dot-product attention reading packed INT4 K/V.

    Returns ``[B, n_q_heads, sq, d_head]`` in the dtype of ``q`` (written into
    ``out`` when given; ``out`` may be any strided view of that shape).
    """
    if group_size <= 0:
        raise ValueError("group_size must be > 0")
    if n_q_heads <= 0 or n_kv_heads <= 0:
        raise ValueError("n_q_heads and n_kv_heads must be > 0")
    if n_q_heads % n_kv_heads != 0:
        raise ValueError("n_q_heads must be divisible by n_kv_heads")
    if not q.is_cuda:
        raise ValueError("attention_forward_quant_gqa expects CUDA tensors")
    if not all(t.is_cuda for t in (k_packed, k_scales, v_packed, v_scales)):
        raise ValueError("attention_forward_quant_gqa expects CUDA tensors")
    if q.dtype not in _Q_DTYPES:
        raise ValueError("q must be bf16/fp16/fp32")
    if k_packed.dtype != torch.uint8 or v_packed.dtype != torch.uint8:
        raise ValueError("k_packed and v_packed must be uint8")
    if k_scales.dtype not in _SCALE_DTYPES or v_scales.dtype not in _SCALE_DTYPES:
        raise ValueError("scales must be bf16/fp16/fp32")
    if k_packed.shape != v_packed.shape:
        raise ValueError("k_packed and v_packed must have the same shape")
    if k_scales.shape != v_scales.shape:
        raise ValueError("k_scales and v_scales must have the same shape")
    if k_packed.shape[:-1] != k_scales.shape[:-1]:
        raise ValueError("packed/scales leading dimensions must match")
    if q.dim() != 4:
        raise ValueError("q must be 4D: [B, n_q_heads, sq, d_head]")
    b, hq, sq, d = q.shape
    if hq != n_q_heads:
        raise ValueError(f"q head dim {hq} != n_q_heads {n_q_heads}")
    if k_packed.shape[0] != b or k_packed.shape[1] != n_kv_heads:
        raise ValueError("k/v leading dims must be [B, n_kv_heads, ...]")
    if k_packed.shape[-1] < math.ceil(d / 2):
        raise ValueError("packed last dimension is too small for q d_head")
    if k_scales.shape[-1] < math.ceil(d / group_size):
        raise ValueError("scales last dimension is too small for q d_head/group_size")
    if k_scales.dtype != v_scales.dtype:
        v_scales = v_scales.to(k_scales.dtype)
    return frontend.attention(q, k_packed, k_scales, v_packed, v_scales, n_q_heads=n_q_heads,
                              n_kv_heads=n_kv_heads, group_size=group_size,
                              is_causal=is_causal, out=out)
