"""GPT-2 attention with the INT4 KV cache and the fused sm_100a decode kernel.

Drop-in for the reference's ``models/gpt2/gpt2_quant.py``
(``GPT2AttentionQuantized`` :16-138, ``replace_gpt2_attention_with_quantized``
:141-157), with its routing (:93-118): the fused kernel runs for
self-attention on CUDA when the query is a single token or no mask is given
(and not in eager "reorder_and_upcast" mode); otherwise the cache is
dequantized on the GPU and the stock attention function runs.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
from transformers.cache_utils import EncoderDecoderCache
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
from transformers.models.gpt2.modeling_gpt2 import GPT2Attention, eager_attention_forward

from kernels.gpt2.attention_quant import attention_forward_quant
from models.gpt2.kv_cache import QuantizedKVCache


class GPT2AttentionQuantized(GPT2Attention):
    """Same as GPT2Attention, with quantized KV cache support for decode."""

    def __init__(self, config, is_cross_attention: bool = False, layer_idx: int | None = None,
                 group_size: int = 32):
        super().__init__(config, is_cross_attention=is_cross_attention, layer_idx=layer_idx)
        self.quant_group_size = int(group_size)

    def forward(
        self,
        hidden_states,
        past_key_values=None,
        cache_position: Optional[torch.LongTensor] = None,
        attention_mask: Optional[torch.FloatTensor] = None,
        head_mask: Optional[torch.FloatTensor] = None,
        encoder_hidden_states: Optional[torch.Tensor] = None,
        encoder_attention_mask: Optional[torch.FloatTensor] = None,
        output_attentions: Optional[bool] = False,
        **kwargs,
    ):
        is_cross_attention = encoder_hidden_states is not None
        quant_cache = past_key_values if isinstance(past_key_values, QuantizedKVCache) else None
        is_updated = False
        curr_past_key_value = None
        if past_key_values is not None and quant_cache is None:
            if isinstance(past_key_values, EncoderDecoderCache):
                is_updated = past_key_values.is_updated.get(self.layer_idx)
                curr_past_key_value = (past_key_values.cross_attention_cache if is_cross_attention
                                       else past_key_values.self_attention_cache)
            else:
                curr_past_key_value = past_key_values

        if is_cross_attention:
            if not hasattr(self, "q_attn"):
                raise ValueError(
                    "If class is used as cross attention, the weights `q_attn` have to be defined. "
                    "Please make sure to instantiate class with `GPT2Attention(..., is_cross_attention=True)`.")
            query_states = self.q_attn(hidden_states)
            attention_mask = encoder_attention_mask
            if past_key_values is not None and quant_cache is None and is_updated:
                key_states = curr_past_key_value.layers[self.layer_idx].keys
                value_states = curr_past_key_value.layers[self.layer_idx].values
            else:
                key_states, value_states = self.c_attn(encoder_hidden_states).split(
                    self.split_size, dim=2)
                shape_kv = (*key_states.shape[:-1], -1, self.head_dim)
                key_states = key_states.view(shape_kv).transpose(1, 2)
                value_states = value_states.view(shape_kv).transpose(1, 2)
        else:
            query_states, key_states, value_states = self.c_attn(hidden_states).split(
                self.split_size, dim=2)
            shape_kv = (*key_states.shape[:-1], -1, self.head_dim)
            key_states = key_states.view(shape_kv).transpose(1, 2)
            value_states = value_states.view(shape_kv).transpose(1, 2)

        shape_q = (*query_states.shape[:-1], -1, self.head_dim)
        query_states = query_states.view(shape_q).transpose(1, 2)

        # one-token decode on the fused kernel: the append happens inside the
        # attention launch (QuantizedKVCache.append_attend) below
        fuse_append = (
            quant_cache is not None
            and not is_cross_attention
            and query_states.is_cuda
            and query_states.shape[-2] == 1
            and key_states.shape[-2] == 1
            and not (self.config._attn_implementation == "eager" and self.reorder_and_upcast_attn)
            and query_states.dtype in (torch.float16, torch.float32)
        )
        if quant_cache is not None and not is_cross_attention:
            if not fuse_append:
                quant_cache.append(key_states, value_states, self.layer_idx)
        elif (past_key_values is not None and not is_cross_attention) or (
                past_key_values is not None and is_cross_attention and not is_updated):
            key_states, value_states = curr_past_key_value.update(key_states, value_states,
                                                                  self.layer_idx)
            if is_cross_attention:
                past_key_values.is_updated[self.layer_idx] = True

        is_causal = attention_mask is None and query_states.shape[-2] > 1 and not is_cross_attention
        using_eager = self.config._attn_implementation == "eager"
        attention_interface: Callable = eager_attention_forward
        if not using_eager:
            attention_interface = ALL_ATTENTION_FUNCTIONS[self.config._attn_implementation]

        use_quant_kernel = (
            quant_cache is not None
            and not is_cross_attention
            and query_states.is_cuda
            and not (using_eager and self.reorder_and_upcast_attn)
            and (query_states.shape[-2] == 1 or attention_mask is None)
            and query_states.dtype in (torch.float16, torch.float32)
        )

        if using_eager and self.reorder_and_upcast_attn:
            if quant_cache is not None and not is_cross_attention:
                key_states, value_states = quant_cache.get_dequantized(self.layer_idx)
            attn_output, attn_weights = self._upcast_and_reordered_attn(
                query_states, key_states, value_states, attention_mask, head_mask)
        elif use_quant_kernel:
            b, h, sq, d = query_states.shape
            out = torch.empty(b, sq, h, d, dtype=query_states.dtype, device=query_states.device)
            if fuse_append:
                quant_cache.append_attend(query_states, key_states, value_states, self.layer_idx,
                                          out.transpose(1, 2), n_q_heads=h, n_kv_heads=h,
                                          is_causal=is_causal)
            else:
                k_packed, k_scales, v_packed, v_scales = quant_cache.get_quantized(self.layer_idx)
                attention_forward_quant(query_states, k_packed, k_scales, v_packed, v_scales,
                                        group_size=self.quant_group_size, is_causal=is_causal,
                                        out=out.transpose(1, 2))
            attn_output = out
            attn_weights = None
        else:
            if quant_cache is not None and not is_cross_attention:
                key_states, value_states = quant_cache.get_dequantized(self.layer_idx)
                key_states = key_states.to(query_states.dtype)
                value_states = value_states.to(query_states.dtype)
            attn_output, attn_weights = attention_interface(
                self, query_states, key_states, value_states, attention_mask, head_mask=head_mask,
                dropout=self.attn_dropout.p if self.training else 0.0, is_causal=is_causal,
                **kwargs)

        attn_output = attn_output.reshape(*attn_output.shape[:-2], -1).contiguous()
        attn_output = self.c_proj(attn_output)
        attn_output = self.resid_dropout(attn_output)
        return attn_output, attn_weights


def replace_gpt2_attention_with_quantized(model: torch.nn.Module, group_size: int = 32) -> None:
    """In-place: swap each GPT2Block self-attention for quantized-cache attention."""
    blocks = getattr(getattr(model, "transformer", None), "h", None)
    if blocks is None:
        raise ValueError("expected a GPT2 model with .transformer.h blocks")
    for block in blocks:
        old = block.attn
        if isinstance(old, GPT2AttentionQuantized):
            old.quant_group_size = int(group_size)
            continue
        device = next(old.parameters()).device
        ref_dtype = next(old.parameters()).dtype
        new = GPT2AttentionQuantized(old.config, layer_idx=old.layer_idx, group_size=group_size)
        new.load_state_dict(old.state_dict())
        new.to(device=device, dtype=ref_dtype)
        new.train(old.training)
        block.attn = new
