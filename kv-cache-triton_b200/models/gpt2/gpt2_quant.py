"""GPT-2 attention with the INT4 KV cache and the fused sm_100a decode kernel.

Drop-in for the reference's ``models/gpt2/gpt2_quant.py``
(``GPT2AttentionQuantized`` :16-138, ``replace_gpt2_attention_with_quantized``
:141-157).  The module owns one decision only, where the cached attention
runs; everything else is Hugging Face's ``GPT2Attention``:

* self-attention with a ``QuantizedKVCache`` on CUDA, fp16/fp32 activations,
  a one-token query or no mask, and not the eager "reorder and upcast" mode
  (the reference's condition, :93-99): the projections run here, K/V are
  quantized into the cache and the fused INT4 kernel attends over the packed
  cache (a one-token step is one launch: append and attention fused);
* any other call with a ``QuantizedKVCache`` runs HF's forward against a thin
  cache view that quantizes the new K/V into the INT4 cache and hands HF the
  dequantized cache (the reference's fallback, :109-126);
* without a ``QuantizedKVCache`` (or for cross-attention) HF's forward runs
  unchanged.
"""

from __future__ import annotations

import types

import torch
from transformers.models.gpt2.modeling_gpt2 import GPT2Attention

from kernels.gpt2.attention_quant import attention_forward_quant
from models.gpt2.kv_cache import QuantizedKVCache


class _DequantizedCacheView:
    """What HF's forward sees of a ``QuantizedKVCache`` on the fallback route:
    ``update`` quantizes the new K/V into the INT4 cache and returns the whole
    layer dequantized in the activations' dtype."""

    def __init__(self, cache: QuantizedKVCache):
        self.cache = cache

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        self.cache.update(key_states, value_states, layer_idx, cache_kwargs)
        k, v = self.cache.get_dequantized(layer_idx)
        return k.to(key_states.dtype), v.to(value_states.dtype)


class GPT2AttentionQuantized(GPT2Attention):
    """Same as GPT2Attention, with quantized KV cache support for decode."""

    def __init__(self, config, is_cross_attention: bool = False, layer_idx: int | None = None,
                 group_size: int = 32):
        super().__init__(config, is_cross_attention=is_cross_attention, layer_idx=layer_idx)
        self.quant_group_size = int(group_size)

    def _fused_ok(self, hidden_states: torch.Tensor, attention_mask) -> bool:
        if not hidden_states.is_cuda or hidden_states.dtype not in (torch.float16, torch.float32):
            return False
        if self.config._attn_implementation == "eager" and self.reorder_and_upcast_attn:
            return False
        return hidden_states.shape[-2] == 1 or attention_mask is None

    def forward(self, hidden_states, past_key_values=None, attention_mask=None, **kwargs):
        cache = past_key_values if isinstance(past_key_values, QuantizedKVCache) else None
        if cache is None or kwargs.get("encoder_hidden_states") is not None:
            return super().forward(hidden_states, past_key_values=past_key_values,
                                   attention_mask=attention_mask, **kwargs)
        if not self._fused_ok(hidden_states, attention_mask):
            return super().forward(hidden_states, past_key_values=_DequantizedCacheView(cache),
                                   attention_mask=attention_mask, **kwargs)

        # [B, s, 3 * hidden] -> three [B, heads, s, head_dim] views
        q, k, v = (t.unflatten(-1, (-1, self.head_dim)).transpose(1, 2)
                   for t in self.c_attn(hidden_states).split(self.split_size, dim=2))
        b, heads, s, d = q.shape
        # the kernel writes [B, s, heads, d] directly: c_proj's input needs no copy
        out = torch.empty(b, s, heads, d, dtype=q.dtype, device=q.device)
        causal = attention_mask is None and s > 1
        if s == 1 and k.shape[-2] == 1:
            cache.append_attend(q, k, v, self.layer_idx, out.transpose(1, 2), n_q_heads=heads,
                                n_kv_heads=heads, is_causal=causal)
        else:
            cache.append(k, v, self.layer_idx)
            attention_forward_quant(q, *cache.get_quantized(self.layer_idx),
                                    group_size=self.quant_group_size, is_causal=causal,
                                    out=out.transpose(1, 2))
        y = self.resid_dropout(self.c_proj(out.flatten(-2)))
        return y, None


def _retarget(module: torch.nn.Module, cls: type, **attrs) -> None:
    """Turn ``module`` into an instance of its subclass ``cls`` in place: its
    parameters, buffers, device placement and any ``accelerate`` dispatch
    hook stay where they are; a hook's saved forward is re-bound so that it
    calls the subclass's forward."""
    module.__class__ = cls
    for name, value in attrs.items():
        setattr(module, name, value)
    if hasattr(module, "_old_forward"):  # accelerate's add_hook_to_module
        module._old_forward = types.MethodType(cls.forward, module)


def replace_gpt2_attention_with_quantized(model: torch.nn.Module, group_size: int = 32) -> None:
    """In-place: swap each GPT2Block self-attention for quantized-cache attention."""
    blocks = getattr(getattr(model, "transformer", None), "h", None)
    if blocks is None:
        raise ValueError("expected a GPT2 model with .transformer.h blocks")
    for block in blocks:
        attn = block.attn
        if type(attn) is not GPT2AttentionQuantized and not isinstance(attn, GPT2Attention):
            raise ValueError(f"unexpected attention module {type(attn).__name__}")
        _retarget(attn, GPT2AttentionQuantized, quant_group_size=int(group_size))
