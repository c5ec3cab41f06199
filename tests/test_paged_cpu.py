"""Host logic of the paged cache (no GPU): page allocation, slot mapping and
block tables, freeing and exhaustion."""

from __future__ import annotations

import pytest
import torch


def _cache(num_pages=10, page=16):
    from kvint4.paged import PagedInt4KVCache
    return PagedInt4KVCache(num_pages, page, 2, 64, group_size=32, device="cpu")


def test_slots_and_block_table_follow_pages():
    c = _cache()
    c.add_sequence("a")
    c.add_sequence("b")
    st = c.begin_step(["a"], 20)          # a: pages 0, 1
    c.commit(st)
    assert c.blocks("a") == [0, 1]
    assert st.slot_mapping.tolist() == list(range(20))
    st = c.begin_step(["b", "a"], 13)     # b: page 2; a grows into page 1 then 2 -> 3
    assert c.blocks("b") == [2]
    assert c.blocks("a") == [0, 1, 3]
    assert st.slot_mapping[:13].tolist() == [2 * 16 + t for t in range(13)]
    a_slots = [(0, 1, 3)[t // 16] * 16 + t % 16 for t in range(20, 33)]
    assert st.slot_mapping[13:].tolist() == a_slots
    assert st.seq_lens.tolist() == [13, 33]
    assert st.block_table.tolist() == [[2, -1, -1], [0, 1, 3]]
    assert st.max_seq_len == 33
    assert c.seq_len("a") == 20  # not committed yet
    c.commit(st)
    assert (c.seq_len("a"), c.seq_len("b")) == (33, 13)


def test_free_returns_pages_and_exhaustion_raises():
    c = _cache(num_pages=4, page=8)
    c.add_sequence(0)
    c.commit(c.begin_step([0], 30))       # 4 pages
    assert c.free_pages == 0
    with pytest.raises(RuntimeError):
        c.begin_step([0], 3)
    c.free_sequence(0)
    assert c.free_pages == 4
    c.add_sequence(1)
    st = c.begin_step([1], 1)
    assert c.blocks(1) == [0]
    with pytest.raises(ValueError):
        c.add_sequence(1)


def test_page_size_and_shapes():
    from kvint4.paged import PagedInt4KVCache
    with pytest.raises(ValueError):
        PagedInt4KVCache(4, 12, 2, 64, device="cpu")
    c = _cache(num_pages=3, page=32)
    assert tuple(c.k_pages[0].shape) == (3, 2, 32, 32)
    assert tuple(c.k_scales[0].shape) == (3, 2, 32, 2)
    assert c.k_scales[0].dtype == torch.bfloat16


def test_paged_calls_need_cuda_tensors():
    """No CPU fallback: the attention entry refuses host tensors."""
    from kvint4 import _lib
    c = _cache()
    c.add_sequence(0)
    st = c.begin_step([0], 4)
    q = torch.zeros(1, 4, 1, 64, dtype=torch.bfloat16)
    with pytest.raises((ValueError, _lib.Kv4Error, RuntimeError)):
        c.attend(0, st, q)
