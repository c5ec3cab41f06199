"""INT4 KV-cache storage with preallocated capacity and in-place append.

Layout in HBM, per layer (one tensor each for K and V):

    packed  uint8 [B, n_kv, capacity, ceil(d/G)*ceil(G/2)]
    scales  float [B, n_kv, capacity, ceil(d/G)]

Tokens ``[0, seq_len)`` are valid; ``get_quantized`` returns strided views
``[:, :, :seq_len]`` with exactly the reference's shapes.  An append
quantizes the new K and V rows straight into rows ``[seq_len, seq_len+s)``
with ONE kernel launch (``kv4_append_kv``); the reference instead quantized
into fresh tensors and concatenated the whole cache each step
(``models/llama3/kv_cache.py:76-102``), an O(S) copy per decode step.
Capacity grows geometrically (one copy of the valid prefix) when exceeded.
Capacity is kept a multiple of 64 tokens so every (batch, head) plane starts
16-byte aligned, which the TMA loads of the decode kernel require.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, frontend, ops

CAPACITY_ALIGN = 64


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class LayerStore:
    k_packed_buf: torch.Tensor
    k_scales_buf: torch.Tensor
    v_packed_buf: torch.Tensor
    v_scales_buf: torch.Tensor
    seq_len: int
    # True while the last kernel that wrote these buffers was a fused decode
    # step (kv4_append_attention): the next fused step may then start early
    # (kv4_attn_opts.early_start), since no other kernel wrote the rows it reads
    early_ok: bool = False

    @property
    def capacity(self) -> int:
        return self.k_packed_buf.shape[2]

    def view_descs(self, n: int):
        """C-ABI descriptors of the four views ``[:, :, :n]``, built from
        descriptors of the buffers kept on the layer (no torch views)."""
        bufs = (self.k_packed_buf, self.k_scales_buf, self.v_packed_buf, self.v_scales_buf)
        cached = getattr(self, "_descs", None)
        if cached is None or cached[0] != tuple(b.data_ptr() for b in bufs):
            cached = (tuple(b.data_ptr() for b in bufs), [ops.desc(b) for b in bufs])
            self._descs = cached
        for d in cached[1]:
            d.shape[2] = n
        return cached[1]

    def views(self):
        s = self.seq_len
        return (self.k_packed_buf[:, :, :s], self.k_scales_buf[:, :, :s],
                self.v_packed_buf[:, :, :s], self.v_scales_buf[:, :, :s])


class Int4KVStore:
    """Per-layer INT4 storage shared by the Llama and GPT-2 caches."""

    def __init__(self, group_size: int = 32, *, capacity: int | None = None,
                 scale_dtype: torch.dtype | None = None, tie_mode: int = _lib.TIE_HALF_AWAY,
                 growth: float = 1.5):
        if group_size <= 0:
            raise ValueError("group_size must be > 0")
        self.group_size = int(group_size)
        self.capacity_hint = int(capacity) if capacity else 0
        self.scale_dtype = scale_dtype
        self.tie_mode = int(tie_mode)
        self.growth = float(growth)
        self._layers: dict[int, LayerStore] = {}

    # -- storage ---------------------------------------------------------
    def _alloc(self, like: torch.Tensor, b: int, h: int, cap: int, d: int) -> LayerStore:
        g = self.group_size
        ng = math.ceil(d / g)
        pw = ng * ((g + 1) // 2)
        sdt = self.scale_dtype or like.dtype
        dev = like.device
        return LayerStore(
            k_packed_buf=torch.empty(b, h, cap, pw, dtype=torch.uint8, device=dev),
            k_scales_buf=torch.empty(b, h, cap, ng, dtype=sdt, device=dev),
            v_packed_buf=torch.empty(b, h, cap, pw, dtype=torch.uint8, device=dev),
            v_scales_buf=torch.empty(b, h, cap, ng, dtype=sdt, device=dev),
            seq_len=0,
        )

    def append(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int) -> None:
        layer = self._reserve(key_states, value_states, layer_idx)
        s = key_states.shape[2]
        if s == 0:
            return
        ops.append_kv(key_states, value_states, layer.k_packed_buf, layer.k_scales_buf,
                      layer.v_packed_buf, layer.v_scales_buf, layer.seq_len, self.group_size,
                      self.tie_mode)
        layer.seq_len += s
        layer.early_ok = False

    def append_attend(self, query: torch.Tensor, key_states: torch.Tensor,
                      value_states: torch.Tensor, layer_idx: int, out: torch.Tensor, *,
                      n_q_heads: int, n_kv_heads: int, is_causal: bool = False) -> torch.Tensor:
        """``append`` followed by attention of ``query`` over the whole layer
        cache, written to ``out`` (any strides, [B, Hq, sq, d]).  A one-token
        decode step is a single launch: the attention kernel quantizes the new
        row itself (``kv4_append_attention``)."""
        layer = self._reserve(key_states, value_states, layer_idx)
        s = key_states.shape[2]
        if s != 1:
            self.append(key_states, value_states, layer_idx)
            kp, ks, vp, vs = self.layer(layer_idx).views()
            return frontend.attention(query, kp, ks, vp, vs, n_q_heads=n_q_heads,
                                      n_kv_heads=n_kv_heads, group_size=self.group_size,
                                      is_causal=is_causal, out=out)
        n = layer.seq_len + 1
        ops.append_attention_descs(query, key_states, value_states, layer.view_descs(n), out,
                                   self.group_size, is_causal, self.tie_mode,
                                   early_start=layer.early_ok)
        layer.seq_len = n
        layer.early_ok = True
        return out

    def _reserve(self, key_states: torch.Tensor, value_states: torch.Tensor,
                 layer_idx: int) -> LayerStore:
        """Check the new states and make room for them (valid rows unchanged)."""
        if key_states.shape != value_states.shape or key_states.dim() != 4:
            raise ValueError("key/value states must both be [B, n_kv, s, d_head]")
        if key_states.dtype not in frontend.FLOATS or value_states.dtype != key_states.dtype:
            raise ValueError("key/value states must be bf16/fp16/fp32 of the same dtype")
        frontend._need_cuda("QuantizedKVCache.append", key_states, value_states)
        b, h, s, d = key_states.shape
        layer = self._layers.get(layer_idx)
        need = (layer.seq_len if layer else 0) + s
        if layer is None:
            cap = _round_up(max(need, self.capacity_hint, CAPACITY_ALIGN), CAPACITY_ALIGN)
            layer = self._alloc(key_states, b, h, cap, d)
            self._layers[layer_idx] = layer
        else:
            kb = layer.k_packed_buf
            if kb.shape[0] != b or kb.shape[1] != h or kb.device != key_states.device:
                raise ValueError("batch/head/device of appended states must match the cache")
            if need > layer.capacity:
                cap = _round_up(max(need, int(layer.capacity * self.growth)), CAPACITY_ALIGN)
                grown = self._alloc(key_states, b, h, cap, d)
                grown.k_scales_buf = grown.k_scales_buf.to(layer.k_scales_buf.dtype)
                grown.v_scales_buf = grown.v_scales_buf.to(layer.v_scales_buf.dtype)
                n = layer.seq_len
                for src, dst in zip(
                        (layer.k_packed_buf, layer.k_scales_buf, layer.v_packed_buf,
                         layer.v_scales_buf),
                        (grown.k_packed_buf, grown.k_scales_buf, grown.v_packed_buf,
                         grown.v_scales_buf)):
                    dst[:, :, :n].copy_(src[:, :, :n])
                grown.seq_len = n
                layer = grown
                self._layers[layer_idx] = layer
        return layer

    def crop(self, max_length: int) -> None:
        """Keep the first ``max_length`` tokens of every layer (negative: drop
        that many from the end), as ``DynamicCache.crop``."""
        for st in self._layers.values():
            n = max_length if max_length >= 0 else st.seq_len + max_length
            st.seq_len = max(0, min(st.seq_len, n))

    def reorder(self, beam_idx: torch.Tensor) -> None:
        """Reorder the batch dimension of every layer (beam search)."""
        for st in self._layers.values():
            idx = beam_idx.to(st.k_packed_buf.device)
            for name in ("k_packed_buf", "k_scales_buf", "v_packed_buf", "v_scales_buf"):
                setattr(st, name, getattr(st, name).index_select(0, idx).contiguous())
            st.early_ok = False

    def layer(self, layer_idx: int) -> LayerStore:
        st = self._layers.get(layer_idx)
        if st is None:
            raise KeyError(f"no cache state for layer {layer_idx}")
        return st

    def dequantized(self, layer_idx: int, out_dtype: torch.dtype):
        st = self.layer(layer_idx)
        kp, ks, vp, vs = st.views()
        d_head = ks.shape[-1] * self.group_size
        k = frontend.dequantize(kp, ks, self.group_size, d_head, out_dtype)
        v = frontend.dequantize(vp, vs, self.group_size, d_head, out_dtype)
        return k, v

    def nbytes(self) -> int:
        """Logical bytes held (packed + scales over the valid tokens), like the
        reference's ``nbytes`` (``models/llama3/kv_cache.py:158-166``)."""
        total = 0
        for st in self._layers.values():
            for t in st.views():
                total += t.element_size() * t.numel()
        return total

    def capacity_nbytes(self) -> int:
        """Bytes actually reserved on the device (including headroom)."""
        total = 0
        for st in self._layers.values():
            for t in (st.k_packed_buf, st.k_scales_buf, st.v_packed_buf, st.v_scales_buf):
                total += t.element_size() * t.numel()
        return total
