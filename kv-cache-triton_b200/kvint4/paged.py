"""Paged (block-table) INT4 KV cache for ragged batches.

The reference keeps one contiguous cache per layer in which every batch
element has the same length (``models/llama3/kv_cache.py:27``).  Here the
packed codes and scales live in fixed-size pages drawn from a pool shared by
all sequences, so sequences of different lengths can be batched.

Layout in HBM, per layer (one pool each for K and V):

    packed  uint8 [num_pages, n_kv, page_size, ceil(d/G)*ceil(G/2)]
    scales  float [num_pages, n_kv, page_size, ceil(d/G)]

The byte format inside a row is the reference's.  A sequence owns a list of
page ids (its block-table row); token ``t`` is row ``t % page_size`` of page
``blocks[t // page_size]``.  All layers share the sequence's page ids.

A decode step is planned once for all layers (``begin_step``): pages are
allocated for the new tokens, and the slot mapping, block table and new
lengths are copied to the device.  Then, per layer, ``append`` quantizes
the new K/V rows into their slots (``kv4_append_kv_paged``) and ``attend``
runs the fused decode attention over each sequence's pages
(``kv4_attention_paged``).  ``commit`` makes the new lengths current.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, ops

PAGE_SIZES = (8, 16, 32, 64, 128)


@dataclass
class PagedStep:
    """Device-side description of one step for a list of sequences."""
    seq_ids: list
    n_new: int
    slot_mapping: torch.Tensor  # int32 [B * n_new]
    block_table: torch.Tensor   # int32 [B, max_blocks] (-1 past each sequence)
    seq_lens: torch.Tensor      # int32 [B], lengths including the new tokens
    max_seq_len: int
    new_lens: list


class PagedInt4KVCache:
    """Page pools for ``n_layers`` layers plus a host-side page allocator."""

    def __init__(self, num_pages: int, page_size: int, n_kv_heads: int, head_dim: int, *,
                 group_size: int = 32, n_layers: int = 1, scale_dtype=torch.bfloat16,
                 device="cuda", tie_mode: int = _lib.TIE_HALF_AWAY):
        if page_size not in PAGE_SIZES:
            raise ValueError(f"page_size must be one of {PAGE_SIZES}")
        if num_pages <= 0 or n_layers <= 0 or group_size <= 0:
            raise ValueError("num_pages, n_layers and group_size must be > 0")
        self.page_size = int(page_size)
        self.group_size = int(group_size)
        self.n_kv_heads = int(n_kv_heads)
        self.head_dim = int(head_dim)
        self.tie_mode = int(tie_mode)
        ng = math.ceil(head_dim / group_size)
        pw = ng * ((group_size + 1) // 2)
        self.k_pages, self.k_scales, self.v_pages, self.v_scales = [], [], [], []
        for _ in range(n_layers):
            self.k_pages.append(torch.zeros(num_pages, n_kv_heads, page_size, pw,
                                            dtype=torch.uint8, device=device))
            self.v_pages.append(torch.zeros_like(self.k_pages[-1]))
            self.k_scales.append(torch.zeros(num_pages, n_kv_heads, page_size, ng,
                                             dtype=scale_dtype, device=device))
            self.v_scales.append(torch.zeros_like(self.k_scales[-1]))
        self.num_pages = int(num_pages)
        self._free = list(range(num_pages - 1, -1, -1))  # pop() hands out low ids first
        self._blocks: dict = {}
        self._lens: dict = {}

    # -- allocator ---------------------------------------------------------
    def add_sequence(self, seq_id) -> None:
        if seq_id in self._blocks:
            raise ValueError(f"sequence {seq_id!r} exists")
        self._blocks[seq_id] = []
        self._lens[seq_id] = 0

    def free_sequence(self, seq_id) -> None:
        self._free.extend(reversed(self._blocks.pop(seq_id)))
        del self._lens[seq_id]

    def seq_len(self, seq_id) -> int:
        return self._lens[seq_id]

    def blocks(self, seq_id) -> list:
        return list(self._blocks[seq_id])

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def _reserve(self, seq_id, new_len: int) -> None:
        need = -(-new_len // self.page_size) - len(self._blocks[seq_id])
        if need > len(self._free):
            raise RuntimeError(f"page pool exhausted: need {need}, {len(self._free)} free")
        for _ in range(max(0, need)):
            self._blocks[seq_id].append(self._free.pop())

    # -- steps -------------------------------------------------------------
    def begin_step(self, seq_ids, n_new: int, device=None) -> PagedStep:
        """Reserve pages for ``n_new`` tokens of every sequence in ``seq_ids``
        and describe the step on the device."""
        if n_new < 0:
            raise ValueError("n_new must be >= 0")
        device = device or (self.k_pages[0].device if self.k_pages else "cpu")
        slots, new_lens = [], []
        for sid in seq_ids:
            old = self._lens[sid]
            self._reserve(sid, old + n_new)
            blk = self._blocks[sid]
            for t in range(old, old + n_new):
                slots.append(blk[t // self.page_size] * self.page_size + t % self.page_size)
            new_lens.append(old + n_new)
        max_len = max(new_lens) if new_lens else 0
        max_blocks = max(1, -(-max_len // self.page_size))
        table = torch.full((len(seq_ids), max_blocks), -1, dtype=torch.int32)
        for i, sid in enumerate(seq_ids):
            blk = self._blocks[sid][:max_blocks]
            if blk:
                table[i, :len(blk)] = torch.tensor(blk, dtype=torch.int32)
        return PagedStep(
            seq_ids=list(seq_ids), n_new=int(n_new),
            slot_mapping=torch.tensor(slots, dtype=torch.int32).to(device, non_blocking=True),
            block_table=table.to(device, non_blocking=True),
            seq_lens=torch.tensor(new_lens, dtype=torch.int32).to(device, non_blocking=True),
            max_seq_len=max(1, max_len), new_lens=new_lens)

    def commit(self, step: PagedStep) -> None:
        for sid, n in zip(step.seq_ids, step.new_lens):
            self._lens[sid] = n

    def append(self, layer: int, step: PagedStep, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantize k, v [B, Hkv, n_new, d] into the step's slots of ``layer``."""
        if k.shape != v.shape or k.dim() != 4 or k.shape[0] != len(step.seq_ids) or \
                k.shape[2] != step.n_new:
            raise ValueError("k/v must be [len(seq_ids), n_kv, n_new, d]")
        ops.append_kv_paged(k, v, self.k_pages[layer], self.k_scales[layer],
                            self.v_pages[layer], self.v_scales[layer], step.slot_mapping,
                            self.group_size, self.tie_mode)

    def attend(self, layer: int, step: PagedStep, q: torch.Tensor, out: torch.Tensor | None = None,
               is_causal: bool = False) -> torch.Tensor:
        """Fused decode attention of q [B, Hq, sq, d] over each sequence's
        pages (lengths after the step's append)."""
        if out is None:
            out = torch.empty_like(q)
        ops.attention_paged_into(q, self.k_pages[layer], self.k_scales[layer],
                                 self.v_pages[layer], self.v_scales[layer], step.block_table,
                                 step.seq_lens, step.max_seq_len, out, self.group_size,
                                 is_causal)
        return out

    def gather(self, layer: int, seq_id):
        """Contiguous (packed K, K scales, packed V, V scales) copies of one
        sequence, [1, n_kv, len, ...] each (for checks and export)."""
        n = self._lens[seq_id]
        blk = torch.tensor(self._blocks[seq_id], dtype=torch.long,
                           device=self.k_pages[layer].device)
        res = []
        for pool in (self.k_pages[layer], self.k_scales[layer], self.v_pages[layer],
                     self.v_scales[layer]):
            x = pool.index_select(0, blk).permute(1, 0, 2, 3)
            x = x.reshape(x.shape[0], -1, x.shape[-1])[:, :n]
            res.append(x.unsqueeze(0).contiguous())
        return tuple(res)
