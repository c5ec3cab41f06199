"""INT4 group-wise quantize / dequantize for the Llama 3.1 KV cache.

Drop-in for the reference's ``kernels/llama3/quantize.py``: same functions,
argument meaning, shapes, dtypes and ``ValueError`` checks
(``quantize_int4`` :189-207, ``dequantize_int4`` :274-308).  Storage format:

    x:      [..., d]                 bf16 / fp16 / fp32
    packed: [..., ceil(d/G)*ceil(G/2)] uint8, low nibble = even column
    scales: [..., ceil(d/G)]         same dtype as x, scale = max|x|/7

Codes are ``clamp(round(x/scale), -8, 7) + 8``.  The default
``TIE_HALF_AWAY`` reproduces the reference's GPU (Triton) kernel bit for bit
(:47-63: half-away rounding, and fp32 divisions as Triton lowers them, PTX
``div.full.f32``); ``tie_mode=TIE_HALF_EVEN`` reproduces its CPU torch path
(:126-148, IEEE divisions, ``torch.round``) bit for bit;
``TIE_HALF_AWAY_IEEE`` is the Triton formula in IEEE arithmetic.  All work runs in libkvint4.so on the GPU; CPU tensors raise
``ValueError``.
"""

from __future__ import annotations

import torch

from kvint4 import frontend
from kvint4._lib import TIE_HALF_AWAY, TIE_HALF_AWAY_IEEE, TIE_HALF_EVEN  # noqa: F401

_SUPPORTED_FLOATS = (torch.bfloat16, torch.float16, torch.float32)


def _validate_group_size(group_size: int) -> None:
    if group_size <= 0:
        raise ValueError("group_size must be > 0")


def quantize_int4(x: torch.Tensor, group_size: int = 32, *,
                  tie_mode: int = TIE_HALF_AWAY) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize the last dim to symmetric INT4 with per-group scales.

    Returns ``(packed_uint8, scales)``; ``scales`` keeps the dtype of ``x``.
    """
    _validate_group_size(group_size)
    if x.dtype not in _SUPPORTED_FLOATS:
        raise ValueError("quantize_int4 expects bf16/fp16/fp32 input")
    if x.dim() < 1:
        raise ValueError("quantize_int4 expects at least 1D input")
    return frontend.quantize(x, group_size, x.dtype, tie_mode)


def dequantize_int4(
    packed: torch.Tensor,
    scales: torch.Tensor,
    group_size: int = 32,
    d_head: int | None = None,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Dequantize a packed INT4 tensor back to ``out_dtype`` (default: scales dtype)."""
    _validate_group_size(group_size)
    if packed.dtype != torch.uint8:
        raise ValueError("packed must be uint8")
    if scales.dtype not in _SUPPORTED_FLOATS:
        raise ValueError("scales must be bf16/fp16/fp32")
    if packed.shape[:-1] != scales.shape[:-1]:
        raise ValueError("packed/scales leading dimensions must match")
    if packed.device != scales.device:
        raise ValueError("packed and scales must be on the same device")
    if out_dtype is None:
        out_dtype = scales.dtype
    if out_dtype not in _SUPPORTED_FLOATS:
        raise ValueError("out_dtype must be bf16/fp16/fp32")
    num_groups = scales.shape[-1]
    target_d = num_groups * group_size if d_head is None else int(d_head)
    if target_d <= 0:
        raise ValueError("d_head must be > 0 when provided")
    return frontend.dequantize(packed, scales, group_size, target_d, out_dtype)
