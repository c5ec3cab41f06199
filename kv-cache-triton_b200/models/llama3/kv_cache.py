"""Quantized KV cache for Llama 3.1 decode with packed INT4 storage.

Drop-in for the reference's ``models/llama3/kv_cache.py`` (``QuantizedKVCache``
:30-166): the same duck-typed subset of the transformers ``Cache`` API
(``get_seq_length``, ``get_mask_sizes``, ``get_max_cache_shape``,
``is_initialized``, ``is_sliding``, ``__len__``, ``reset``, ``has_layer``,
``append``, ``update``, ``get_quantized``, ``get_dequantized``, ``nbytes``)
and the same tensor shapes: ``get_quantized`` returns
``[B, n_kv, S, d/2]`` packed and ``[B, n_kv, S, d/G]`` scales (scales keep
the K/V dtype).  Storage is a preallocated capacity buffer per layer that
new tokens are quantized into in place (see ``kvint4.cache``); the returned
tensors are views of it, valid until the next append to that layer.
"""

from __future__ import annotations

import torch

from kvint4._lib import TIE_HALF_AWAY
from kvint4.cache import Int4KVStore


class QuantizedKVCache:
    """Per-layer INT4-packed KV cache. Compatible with HF Llama attention."""

    def __init__(self, group_size: int = 32, *, capacity: int | None = None,
                 tie_mode: int = TIE_HALF_AWAY):
        if group_size <= 0:
            raise ValueError("group_size must be > 0")
        self.group_size = int(group_size)
        self._store = Int4KVStore(self.group_size, capacity=capacity, tie_mode=tie_mode)

    @property
    def _layers(self):
        return self._store._layers

    def get_seq_length(self, layer_idx: int = 0) -> int:
        layer = self._layers.get(layer_idx)
        return 0 if layer is None else int(layer.seq_len)

    def get_mask_sizes(self, cache_position, layer_idx: int = 0) -> tuple[int, int]:
        past_len = self.get_seq_length(layer_idx)
        if isinstance(cache_position, int):
            query_length = int(cache_position)
        elif isinstance(cache_position, torch.Tensor):
            if cache_position.dim() == 0:
                query_length = int(cache_position.item())
            else:
                query_length = int(cache_position.shape[0])
        else:
            query_length = int(cache_position)
        return past_len + query_length, 0

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return -1

    @property
    def is_initialized(self) -> bool:
        return len(self._layers) > 0

    @property
    def is_sliding(self) -> list[bool]:
        return [False for _ in self._layers]

    def __len__(self) -> int:
        return len(self._layers)

    def reset(self) -> None:
        self._layers.clear()

    # HF generate() asks these of any cache object it is given
    is_compileable = False

    def crop(self, max_length: int) -> None:
        """Drop tokens past ``max_length`` (negative: that many from the end)."""
        self._store.crop(max_length)

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        """Reorder the batch dimension for beam search."""
        self._store.reorder(beam_idx)

    def has_layer(self, layer_idx: int) -> bool:
        return layer_idx in self._layers

    def append(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int) -> None:
        """Quantize ``[B, n_kv, s, d]`` K/V (any strides) into the layer's cache."""
        self._store.append(key_states, value_states, layer_idx)

    def append_attend(self, query: torch.Tensor, key_states: torch.Tensor,
                      value_states: torch.Tensor, layer_idx: int, out: torch.Tensor, *,
                      n_q_heads: int, n_kv_heads: int, is_causal: bool = False) -> torch.Tensor:
        """``append`` then fused attention of ``query`` over the layer's cache
        into ``out`` ([B, Hq, sq, d], any strides).  One kernel launch for a
        one-token decode step (the new row is quantized inside the attention
        kernel); returns ``out``."""
        return self._store.append_attend(query, key_states, value_states, layer_idx, out,
                                         n_q_heads=n_q_heads, n_kv_heads=n_kv_heads,
                                         is_causal=is_causal)

    def update(
        self,
        key_states: torch.Tensor,
        value_states: torch.Tensor,
        layer_idx: int,
        cache_kwargs: dict | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """Quantize and append K/V, then return the full dequantized cache.

        The fused attention path reads packed tensors via ``get_quantized`` and
        never uses this; it serves stock attention modules.
        """
        del cache_kwargs
        self._store.append(key_states, value_states, layer_idx)
        return self.get_dequantized(layer_idx, out_dtype=key_states.dtype)

    def get_quantized(
        self, layer_idx: int
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        return self._store.layer(layer_idx).views()

    def get_dequantized(
        self,
        layer_idx: int,
        out_dtype: torch.dtype = torch.bfloat16,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        return self._store.dequantized(layer_idx, out_dtype)

    def nbytes(self) -> int:
        """Total bytes stored across all layers (packed + scales)."""
        return self._store.nbytes()

    def capacity_nbytes(self) -> int:
        """Device bytes reserved, including append headroom."""
        return self._store.capacity_nbytes()
