"""CPU oracle for the INT4 KV-cache hot path (test infrastructure only).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import it.  It restates, in numpy, the arithmetic of the reference
(johnchmura/kv-cache-triton) for the path the CUDA library accelerates:

* group-wise symmetric INT4 quantization with a fixed +8 bias
  (``kernels/llama3/quantize.py:27-75`` Triton kernel and ``:126-148`` torch
  path; the GPT-2 copy ``kernels/gpt2/quantize.py:13-61, 111-133`` differs only
  in storing fp16 scales);
* dequantization ``(nibble - 8) * scale`` (``kernels/llama3/quantize.py:78-115,
  210-234``);
* single-/multi-query GQA attention over the dequantized cache with the
  bottom-right causal alignment of ``kernels/llama3/attention_quant.py:91-124``
  (reference formula of ``tests/llama3/test_attention_quant_gqa.py:15-40`` and
  ``tests/llama3/test_attention_fused_vs_ref_sm70.py:14-51``).

Pinning: ``tests/golden/make_golden.py`` imports the reference's own torch
functions and SDPA and writes ``tests/golden/*.npz``; ``tests/test_oracle.py``
checks this module against every vector there (the HALF_EVEN tie mode is the
torch path and is pinned bit-exactly; the HALF_AWAY mode restates the Triton
kernel's ``floor(q+0.5)`` / ``ceil(q-0.5)`` rounding and is pinned on every
non-tie element plus hand-written tie cases).
"""

from __future__ import annotations

import math

import numpy as np

# Half-away rounding of the Triton kernel's formula (kernels/llama3/quantize.py:47-63)
# in IEEE arithmetic: the library's KV4_TIE_HALF_AWAY_IEEE bit for bit.  The
# library's default KV4_TIE_HALF_AWAY also takes Triton's fp32 divisions (PTX
# div.full.f32), whose last bit this restatement does not model; that mode is
# pinned against the reference's own Triton kernel on the GPU instead.
TIE_HALF_AWAY = 0
TIE_HALF_EVEN = 1  # torch CPU path (torch.round), kernels/llama3/quantize.py:139


# --------------------------------------------------------------------------
# 16-bit float helpers (numpy has no bfloat16)
# --------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bfloat16 (round-to-nearest-even), returned as uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) & 0xFFFF
    r = np.where(nan, 0x7FC0, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ('f32' | 'f16' | 'bf16') and back to float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    raise ValueError(dtype)


# --------------------------------------------------------------------------
# quantize / dequantize
# --------------------------------------------------------------------------

def packed_width(d: int, group_size: int) -> int:
    """Bytes per row of the packed tensor (reference: ``ceil(d/G)`` groups of
    ``ceil(G/2)`` bytes; odd G pads each group with one zero nibble,
    ``kernels/llama3/quantize.py:128-147``)."""
    ng = math.ceil(d / group_size)
    return ng * ((group_size + 1) // 2)


def quantize_int4(x: np.ndarray, group_size: int, tie: int = TIE_HALF_EVEN,
                  scale_dtype: str = "f32"):
    """Quantize the last dim of ``x`` (float32 values, already exact copies of
    the input dtype) to packed INT4 codes.

    Returns ``(packed uint8 [..., packed_width], scales float32 [..., ng])``.
    Scales are returned rounded to ``scale_dtype``; the codes are computed with
    the un-rounded fp32 scale exactly as the reference does
    (``kernels/llama3/quantize.py:50-60, 137-148``).
    """
    if group_size <= 0:
        raise ValueError("group_size must be > 0")
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    ng = math.ceil(d / group_size)
    lead = x.shape[:-1]
    work = np.zeros(lead + (ng * group_size,), dtype=np.float32)
    work[..., :d] = x
    grouped = work.reshape(lead + (ng, group_size))
    max_abs = np.abs(grouped).max(axis=-1, keepdims=True) if group_size > 0 else None
    scale = np.where(max_abs > 0, max_abs / np.float32(7.0), np.float32(1.0)).astype(np.float32)
    q = (grouped / scale).astype(np.float32)
    if tie == TIE_HALF_EVEN:
        r = np.rint(q)
    elif tie == TIE_HALF_AWAY:
        up = np.floor((q + np.float32(0.5)).astype(np.float32))
        dn = np.ceil((q - np.float32(0.5)).astype(np.float32))
        r = np.where(q >= 0, up, dn)
    else:
        raise ValueError("tie mode")
    codes = (np.clip(r, -8, 7).astype(np.int16) + 8).astype(np.uint8)
    if group_size % 2:
        codes = np.concatenate([codes, np.zeros(lead + (ng, 1), dtype=np.uint8)], axis=-1)
    codes = codes.reshape(lead + (-1,))
    packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)
    return packed, round_to(scale[..., 0], scale_dtype)


def dequantize_int4(packed: np.ndarray, scales: np.ndarray, group_size: int,
                    d_head: int | None = None) -> np.ndarray:
    """``(nibble - 8) * scale`` in float32 (``kernels/llama3/quantize.py:210-234``).

    ``scales`` are the stored (already rounded) scales as float32.
    """
    packed = np.asarray(packed, dtype=np.uint8)
    scales = np.asarray(scales, dtype=np.float32)
    ng = scales.shape[-1]
    unpacked = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.float32)
    unpacked[..., 0::2] = (packed & 0x0F).astype(np.float32) - 8.0
    unpacked[..., 1::2] = ((packed >> 4) & 0x0F).astype(np.float32) - 8.0
    grouped = unpacked.reshape(unpacked.shape[:-1] + (ng, -1))
    if grouped.shape[-1] < group_size:
        raise ValueError("packed has insufficient width for the provided group_size")
    out = grouped[..., :group_size] * scales[..., None]
    out = out.reshape(out.shape[:-2] + (-1,))
    d = ng * group_size if d_head is None else int(d_head)
    return out[..., :d].astype(np.float32)


# --------------------------------------------------------------------------
# attention over the dequantized cache
# --------------------------------------------------------------------------

def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, n_q_heads: int,
              n_kv_heads: int, is_causal: bool = False,
              sm_scale: float | None = None) -> np.ndarray:
    """float64 GQA attention: ``softmax(q k^T * d^-1/2) v``, query head ``h``
    reading KV head ``h // (n_q/n_kv)`` (``kernels/llama3/attention_quant.py:71``);
    causal masking is bottom-right aligned (``:91-97, :123-124``): query row
    ``i`` sees keys ``j <= sk - sq + i``.  Rows that see no key return 0.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    b, hq, sq, d = q.shape
    sk = k.shape[2]
    ratio = n_q_heads // n_kv_heads
    kk = np.repeat(k, ratio, axis=1)
    vv = np.repeat(v, ratio, axis=1)
    scale = d ** -0.5 if sm_scale is None else sm_scale
    s = np.einsum("bhqd,bhkd->bhqk", q, kk) * scale
    if is_causal:
        qi = np.arange(sq)[:, None]
        kj = np.arange(sk)[None, :]
        s = np.where(kj <= (sk - sq) + qi, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhqk,bhkd->bhqd", p, vv)
    return np.where(l > 0, o / np.where(l > 0, l, 1.0), 0.0)


def quantized_attention(q, k_packed, k_scales, v_packed, v_scales, *, n_q_heads,
                        n_kv_heads, group_size=32, is_causal=False):
    """Attention of the reference's fused kernel, stated as dequant + float64
    attention (``kernels/llama3/attention_quant.py:24-152``)."""
    d = q.shape[-1]
    kd = dequantize_int4(k_packed, k_scales, group_size, d)
    vd = dequantize_int4(v_packed, v_scales, group_size, d)
    return attention(q, kd, vd, n_q_heads=n_q_heads, n_kv_heads=n_kv_heads,
                     is_causal=is_causal)


def partial_attention(q, k, v, *, n_q_heads, n_kv_heads, is_causal=False, k_offset=0,
                      sk_total=None):
    """Per-shard softmax partials for a sequence-sharded cache: returns
    ``(o normalised within the shard, lse natural-log)``; shard tokens are
    global positions ``k_offset .. k_offset + k.shape[2]``."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    b, hq, sq, d = q.shape
    sk = k.shape[2]
    sk_total = sk if sk_total is None else sk_total
    ratio = n_q_heads // n_kv_heads
    kk = np.repeat(k, ratio, axis=1)
    vv = np.repeat(v, ratio, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q, kk) * d ** -0.5
    if is_causal:
        qi = np.arange(sq)[:, None]
        kj = k_offset + np.arange(sk)[None, :]
        s = np.where(kj <= (sk_total - sq) + qi, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    fm = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - fm)
    l = p.sum(axis=-1, keepdims=True)
    o = np.where(l > 0, np.einsum("bhqk,bhkd->bhqd", p, vv) / np.where(l > 0, l, 1.0), 0.0)
    lse = np.where(l[..., 0] > 0, fm[..., 0] + np.log(np.where(l[..., 0] > 0, l[..., 0], 1.0)), -np.inf)
    return o, lse


def lse_combine(parts_o, parts_lse):
    """Merge shard partials: ``o = sum_r o_r exp(lse_r - lse*) / sum_r exp(lse_r - lse*)``."""
    o = np.stack([np.asarray(x, dtype=np.float64) for x in parts_o])
    lse = np.stack([np.asarray(x, dtype=np.float64) for x in parts_lse])
    mx = lse.max(axis=0)
    fm = np.where(np.isfinite(mx), mx, 0.0)
    w = np.exp(lse - fm)
    den = w.sum(axis=0)
    num = (o * w[..., None]).sum(axis=0)
    return np.where(den[..., None] > 0, num / np.where(den > 0, den, 1.0)[..., None], 0.0)
