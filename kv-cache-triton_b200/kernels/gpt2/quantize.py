"""INT4 group-wise quantize / dequantize for the GPT-2 KV cache.

Drop-in for the reference's ``kernels/gpt2/quantize.py``
(``quantize_int4`` :174-187, ``dequantize_int4`` :190-214): identical to the
Llama variant except that scales are always stored as fp16 and dequantization
always returns fp16.  GPU only (libkvint4.so); CPU tensors raise
``ValueError``.
"""

from __future__ import annotations

import torch

from kvint4 import frontend
from kvint4._lib import TIE_HALF_AWAY, TIE_HALF_AWAY_IEEE, TIE_HALF_EVEN  # noqa: F401


def _validate_group_size(group_size: int) -> None:
    if group_size <= 0:
        raise ValueError("group_size must be > 0")


def quantize_int4(x: torch.Tensor, group_size: int = 32, *,
                  tie_mode: int = TIE_HALF_AWAY) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize last dimension to symmetric INT4 with per-group fp16 scales."""
    _validate_group_size(group_size)
    if x.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise ValueError("quantize_int4 expects float16/float32/bfloat16 input")
    if x.dim() < 1:
        raise ValueError("quantize_int4 expects at least 1D input")
    return frontend.quantize(x, group_size, torch.float16, tie_mode)


def dequantize_int4(
    packed: torch.Tensor,
    scales: torch.Tensor,
    group_size: int = 32,
    d_head: int | None = None,
) -> torch.Tensor:
    """Dequantize uint8-packed INT4 tensor back to float16."""
    _validate_group_size(group_size)
    if packed.dtype != torch.uint8:
        raise ValueError("packed must be uint8")
    if scales.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise ValueError("scales must be float16/float32/bfloat16")
    if packed.shape[:-1] != scales.shape[:-1]:
        raise ValueError("packed/scales leading dimensions must match")
    if packed.device != scales.device:
        raise ValueError("packed and scales must be on the same device")
    num_groups = scales.shape[-1]
    target_d = num_groups * group_size if d_head is None else int(d_head)
    if target_d <= 0:
        raise ValueError("d_head must be > 0 when provided")
    return frontend.dequantize(packed, scales, group_size, target_d, torch.float16)
