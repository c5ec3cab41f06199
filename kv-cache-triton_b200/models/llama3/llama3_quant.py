"""Llama 3 attention with the INT4 KV cache and the fused sm_100a decode kernel.

Drop-in for the reference's ``models/llama3/llama3_quant.py``
(``LlamaAttentionQuantized`` :36-143, ``replace_llama_attention_with_quantized``
:171-204).  Routing is the reference's: with a ``QuantizedKVCache`` the new
K/V are quantized into the cache and, when ``attention_mask is None``, the
fused kernel reads the packed cache directly; with a mask the cache is
dequantized (on the GPU) and the stock HF attention function runs.  Without a
``QuantizedKVCache`` the module behaves like ``LlamaAttention``.

Differences that keep behaviour but remove copies: the fused kernel reads
q and the cache views in place (no ``.contiguous()``), and writes its output
directly in ``[B, s, n_q, d]`` order so the ``o_proj`` input needs no
transpose copy.  A one-token decode step appends and attends in one kernel
launch (``QuantizedKVCache.append_attend``).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
from transformers.models.llama.modeling_llama import (
    LlamaAttention,
    apply_rotary_pos_emb,
    eager_attention_forward,
)

from kernels.llama3.attention_quant import attention_forward_quant_gqa
from models.llama3.kv_cache import QuantizedKVCache


class LlamaAttentionQuantized(LlamaAttention):
    """LlamaAttention subclass that routes to the fused INT4 kernel when a ``QuantizedKVCache`` is in use."""

    def __init__(self, config, layer_idx: int, group_size: int = 32):
        super().__init__(config=config, layer_idx=layer_idx)
        self.quant_group_size = int(group_size)

    def forward(
        self,
        hidden_states: torch.Tensor,
        position_embeddings: tuple[torch.Tensor, torch.Tensor] | None = None,
        attention_mask: Optional[torch.Tensor] = None,
        past_key_values=None,
        cache_position: Optional[torch.LongTensor] = None,
        **kwargs,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)

        query_states = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        key_states = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        value_states = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)

        cos, sin = position_embeddings
        query_states, key_states = apply_rotary_pos_emb(query_states, key_states, cos, sin)

        quant_cache = past_key_values if isinstance(past_key_values, QuantizedKVCache) else None

        if quant_cache is not None:
            n_q = self.config.num_attention_heads
            n_kv = self.config.num_key_value_heads
            sq = query_states.shape[-2]
            is_causal = attention_mask is None and sq > 1

            if query_states.is_cuda and attention_mask is None:
                b = query_states.shape[0]
                out = torch.empty(b, sq, n_q, self.head_dim, dtype=query_states.dtype,
                                  device=query_states.device)
                if sq == 1:
                    # decode: the append is fused into the attention launch
                    quant_cache.append_attend(query_states, key_states, value_states,
                                              self.layer_idx, out.transpose(1, 2),
                                              n_q_heads=n_q, n_kv_heads=n_kv)
                else:
                    quant_cache.append(key_states, value_states, self.layer_idx)
                    k_packed, k_scales, v_packed, v_scales = quant_cache.get_quantized(
                        self.layer_idx)
                    attention_forward_quant_gqa(
                        query_states, k_packed, k_scales, v_packed, v_scales,
                        n_q_heads=n_q, n_kv_heads=n_kv, group_size=self.quant_group_size,
                        is_causal=is_causal, out=out.transpose(1, 2),
                    )
                attn_output = self.o_proj(out.view(*input_shape, -1))
                return attn_output, None

            quant_cache.append(key_states, value_states, self.layer_idx)

            k_full, v_full = quant_cache.get_dequantized(self.layer_idx,
                                                         out_dtype=query_states.dtype)
            return self._fallback_attention(query_states, k_full, v_full,
                                            attention_mask=attention_mask,
                                            input_shape=input_shape, **kwargs)

        if past_key_values is not None:
            cache_kwargs = {"sin": sin, "cos": cos, "cache_position": cache_position}
            key_states, value_states = past_key_values.update(
                key_states, value_states, self.layer_idx, cache_kwargs)

        return self._fallback_attention(query_states, key_states, value_states,
                                        attention_mask=attention_mask, input_shape=input_shape,
                                        **kwargs)

    def _fallback_attention(self, query_states, key_states, value_states, *, attention_mask,
                            input_shape, **kwargs):
        attention_interface: Callable = eager_attention_forward
        if self.config._attn_implementation != "eager":
            attention_interface = ALL_ATTENTION_FUNCTIONS[self.config._attn_implementation]
        attn_output, attn_weights = attention_interface(
            self, query_states, key_states, value_states, attention_mask,
            dropout=0.0 if not self.training else self.attention_dropout,
            scaling=self.scaling, **kwargs)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        attn_output = self.o_proj(attn_output)
        return attn_output, attn_weights


def _transplant_projection(src: torch.nn.Linear, dst: torch.nn.Linear) -> None:
    """Move weight/bias from ``src`` to ``dst`` and re-attach any ``accelerate`` hook
    (reference ``models/llama3/llama3_quant.py:146-168``)."""
    dst.weight = src.weight
    dst.bias = src.bias if getattr(src, "bias", None) is not None else None
    hook = getattr(src, "_hf_hook", None)
    if hook is not None:
        try:
            from accelerate.hooks import add_hook_to_module, remove_hook_from_module
            remove_hook_from_module(src)
            add_hook_to_module(dst, hook)
        except Exception:
            pass


def replace_llama_attention_with_quantized(model: torch.nn.Module, group_size: int = 32) -> None:
    """In-place: swap each Llama decoder-layer self-attention for the quantized variant."""
    layers = getattr(getattr(model, "model", None), "layers", None)
    if layers is None:
        raise ValueError("expected a Llama CausalLM model with .model.layers")
    try:
        from accelerate.hooks import add_hook_to_module, remove_hook_from_module
        accel = True
    except Exception:
        accel = False
    for layer in layers:
        old = layer.self_attn
        if isinstance(old, LlamaAttentionQuantized):
            old.quant_group_size = int(group_size)
            continue
        new = LlamaAttentionQuantized(old.config, layer_idx=old.layer_idx, group_size=group_size)
        for pname in ("q_proj", "k_proj", "v_proj", "o_proj"):
            _transplant_projection(getattr(old, pname), getattr(new, pname))
        old_hook = getattr(old, "_hf_hook", None)
        if accel and old_hook is not None:
            remove_hook_from_module(old)
            add_hook_to_module(new, old_hook)
        new.train(old.training)
        layer.self_attn = new
