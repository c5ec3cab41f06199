"""Llama 3 attention with the INT4 KV cache and the fused sm_100a decode kernel.

Drop-in for the reference's ``models/llama3/llama3_quant.py``
(``LlamaAttentionQuantized`` :36-143, ``replace_llama_attention_with_quantized``
:171-204).  The module owns one decision only, where the cached attention
runs; everything else is Hugging Face's ``LlamaAttention``:

* with a ``QuantizedKVCache``, CUDA activations and no mask (the reference's
  condition, :74): projections and RoPE run here, K/V are quantized into the
  cache and the fused INT4 kernel attends over the packed cache in place,
  writing its output in ``[B, s, n_q, d]`` order so ``o_proj`` needs no
  transpose copy (a one-token step is one launch: append and attention
  fused; longer query blocks are bottom-right causal);
* with a ``QuantizedKVCache`` and a mask (or CPU tensors), HF's forward runs
  against a thin cache view that quantizes the new K/V into the INT4 cache
  and hands HF the cache dequantized in the query's dtype (the reference's
  fallback, :90-99);
* without a ``QuantizedKVCache``, HF's forward runs unchanged.
"""

from __future__ import annotations

import types

import torch
from transformers.models.llama.modeling_llama import LlamaAttention, apply_rotary_pos_emb

from kernels.llama3.attention_quant import attention_forward_quant_gqa
from models.llama3.kv_cache import QuantizedKVCache


class _DequantizedCacheView:
    """What HF's forward sees of a ``QuantizedKVCache`` on the fallback route."""

    def __init__(self, cache: QuantizedKVCache):
        self.cache = cache

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        self.cache.append(key_states, value_states, layer_idx)
        return self.cache.get_dequantized(layer_idx, out_dtype=key_states.dtype)


class LlamaAttentionQuantized(LlamaAttention):
    """LlamaAttention subclass that routes to the fused INT4 kernel when a ``QuantizedKVCache`` is in use."""

    def __init__(self, config, layer_idx: int, group_size: int = 32):
        super().__init__(config=config, layer_idx=layer_idx)
        self.quant_group_size = int(group_size)

    def forward(self, hidden_states: torch.Tensor, position_embeddings=None,
                attention_mask: torch.Tensor | None = None, past_key_values=None, **kwargs):
        cache = past_key_values if isinstance(past_key_values, QuantizedKVCache) else None
        if cache is None:
            return super().forward(hidden_states, position_embeddings, attention_mask,
                                   past_key_values, **kwargs)
        if not (hidden_states.is_cuda and attention_mask is None):
            return super().forward(hidden_states, position_embeddings, attention_mask,
                                   _DequantizedCacheView(cache), **kwargs)

        lead = hidden_states.shape[:-1]

        def heads(proj):  # [B, s, n * d] -> [B, n, s, d]
            return proj(hidden_states).unflatten(-1, (-1, self.head_dim)).transpose(1, 2)

        q, k = apply_rotary_pos_emb(heads(self.q_proj), heads(self.k_proj), *position_embeddings)
        v = heads(self.v_proj)
        n_q, n_kv = self.config.num_attention_heads, self.config.num_key_value_heads
        s = q.shape[-2]
        out = torch.empty(*lead, n_q, self.head_dim, dtype=q.dtype, device=q.device)
        if s == 1:
            cache.append_attend(q, k, v, self.layer_idx, out.transpose(1, 2), n_q_heads=n_q,
                                n_kv_heads=n_kv)
        else:
            cache.append(k, v, self.layer_idx)
            attention_forward_quant_gqa(q, *cache.get_quantized(self.layer_idx), n_q_heads=n_q,
                                        n_kv_heads=n_kv, group_size=self.quant_group_size,
                                        is_causal=True, out=out.transpose(1, 2))
        return self.o_proj(out.flatten(-2)), None


def _retarget(module: torch.nn.Module, cls: type, **attrs) -> None:
    """Turn ``module`` into an instance of its subclass ``cls`` in place: the
    projections, their placement on devices and any ``accelerate`` dispatch
    hook (``device_map="auto"``) stay as they are; a hook's saved forward is
    re-bound so that it calls the subclass's forward."""
    module.__class__ = cls
    for name, value in attrs.items():
        setattr(module, name, value)
    if hasattr(module, "_old_forward"):  # accelerate's add_hook_to_module
        module._old_forward = types.MethodType(cls.forward, module)


def replace_llama_attention_with_quantized(model: torch.nn.Module, group_size: int = 32) -> None:
    """In-place: swap each Llama decoder-layer self-attention for the quantized variant."""
    layers = getattr(getattr(model, "model", None), "layers", None)
    if layers is None:
        raise ValueError("expected a Llama CausalLM model with .model.layers")
    for layer in layers:
        attn = layer.self_attn
        if not isinstance(attn, LlamaAttention):
            raise ValueError(f"unexpected attention module {type(attn).__name__}")
        _retarget(attn, LlamaAttentionQuantized, quant_group_size=int(group_size))
