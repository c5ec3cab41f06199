"""CPU baseline: the reference's PyTorch formulation of one INT4-KV decode step,
restated with torch CPU ops (test/benchmark infrastructure only; imported by
``bench.py``'s CPU-baseline and reference arms and by tests).

One step, as the reference runs it on a CPU tensor:
  * quantize the new K/V token with the torch path (round half to even),
    ``kernels/llama3/quantize.py:126-148``;
  * append by ``torch.cat`` along the sequence (whole-cache copy),
    ``models/llama3/kv_cache.py:96-102``;
  * dequantize the whole cache, ``kernels/llama3/quantize.py:210-234``;
  * ``repeat_interleave`` the KV heads and run
    ``torch.nn.functional.scaled_dot_product_attention``
    (``tests/llama3/test_attention_quant_gqa.py:15-40``; the reference's
    CPU fallback path ``models/llama3/llama3_quant.py:90-143``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def quantize_int4(x: torch.Tensor, group_size: int):
    d = x.shape[-1]
    ng = math.ceil(d / group_size)
    pad = ng * group_size - d
    work = x.float()
    if pad:
        work = F.pad(work, (0, pad))
    grouped = work.view(*work.shape[:-1], ng, group_size)
    max_abs = grouped.abs().amax(dim=-1, keepdim=True)
    scales = torch.where(max_abs > 0, max_abs / 7.0, torch.ones_like(max_abs))
    q = (torch.round(grouped / scales).clamp(-8, 7).to(torch.int16) + 8).to(torch.uint8)
    if group_size % 2:
        q = F.pad(q, (0, 1))
    packed = (q[..., 0::2] | (q[..., 1::2] << 4)).contiguous().view(*x.shape[:-1], -1)
    return packed, scales.squeeze(-1).to(x.dtype)


def dequantize_int4(packed: torch.Tensor, scales: torch.Tensor, group_size: int, d_head: int,
                    out_dtype=torch.float32) -> torch.Tensor:
    ng = scales.shape[-1]
    un = torch.empty(*packed.shape[:-1], packed.shape[-1] * 2, dtype=torch.float32)
    un[..., 0::2] = (packed & 0x0F).to(torch.float32) - 8.0
    un[..., 1::2] = ((packed >> 4) & 0x0F).to(torch.float32) - 8.0
    g = un.view(*un.shape[:-1], ng, -1)[..., :group_size]
    out = (g * scales.float().unsqueeze(-1)).reshape(*un.shape[:-1], -1)
    return out[..., :d_head].to(out_dtype)


def decode_step(cache: dict, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                n_q_heads: int, n_kv_heads: int, group_size: int = 32) -> torch.Tensor:
    """One decode step on CPU tensors; ``cache`` holds kp/ks/vp/vs and grows."""
    kp, ks = quantize_int4(k_new, group_size)
    vp, vs = quantize_int4(v_new, group_size)
    cache["kp"] = torch.cat([cache["kp"], kp], dim=2)
    cache["ks"] = torch.cat([cache["ks"], ks], dim=2)
    cache["vp"] = torch.cat([cache["vp"], vp], dim=2)
    cache["vs"] = torch.cat([cache["vs"], vs], dim=2)
    d = q.shape[-1]
    # the reference's CPU route: get_dequantized(out_dtype=q.dtype), then HF
    # attention (repeat_kv + SDPA) in that dtype (models/llama3/llama3_quant.py:90-99,
    # kv_cache.py:146-157)
    k = dequantize_int4(cache["kp"], cache["ks"], group_size, d, out_dtype=q.dtype)
    v = dequantize_int4(cache["vp"], cache["vs"], group_size, d, out_dtype=q.dtype)
    rep = n_q_heads // n_kv_heads
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    return F.scaled_dot_product_attention(q, k, v)
