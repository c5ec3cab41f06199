"""CPU-only checks of the boundary: the C-ABI library loads and exports every
symbol ``include/kvint4.h`` declares; the reference-shaped Python functions
raise the reference's ``ValueError``s; there is no CPU fallback."""

from __future__ import annotations

import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "kvint4.h")).read()
    return sorted(set(re.findall(r"\b(kv4_[a-z_0-9]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from kvint4 import _lib
    L = _lib.lib()
    declared = _declared_symbols()
    assert len(declared) >= 11
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(_lib.EXPORTED)
    assert L.kv4_version() >= 100
    assert L.kv4_strerror(0) == b"ok"


def test_plan_reports_paths_without_gpu_calls():
    """kv4_attention_plan is host-only arithmetic; with no device it still
    answers (the fast path needs the driver entry point, so it may plan the
    generic path here)."""
    from kvint4 import ops
    q = torch.empty(2, 8, 1, 128, dtype=torch.bfloat16)
    kp = torch.empty(2, 2, 100, 64, dtype=torch.uint8)
    ks = torch.empty(2, 2, 100, 4, dtype=torch.bfloat16)
    p = ops.plan(q, kp, ks, kp, ks, q, 32)
    assert p.path in (1, 2)
    p = ops.plan(q, kp, ks, kp, ks, q, 32, force_generic=True)
    assert p.path == 2 and p.workspace_bytes == 0


def test_plan_rejects_bad_shapes():
    from kvint4 import _lib, ops
    q = torch.empty(2, 8, 1, 128, dtype=torch.bfloat16)
    kp = torch.empty(2, 3, 100, 64, dtype=torch.uint8)  # 8 % 3 != 0
    ks = torch.empty(2, 3, 100, 4, dtype=torch.bfloat16)
    with pytest.raises(_lib.Kv4Error):
        ops.plan(q, kp, ks, kp, ks, q, 32)


def test_quantize_validation_errors_match_reference():
    from kernels.llama3.quantize import dequantize_int4, quantize_int4
    with pytest.raises(ValueError):
        quantize_int4(torch.randn(4, 128), group_size=0)
    with pytest.raises(ValueError):
        quantize_int4(torch.randint(0, 5, (4, 128), dtype=torch.int32), group_size=32)
    with pytest.raises(ValueError, match="CUDA"):
        quantize_int4(torch.randn(4, 128), group_size=32)  # no CPU fallback
    p = torch.zeros(2, 64, dtype=torch.uint8)
    with pytest.raises(ValueError):
        dequantize_int4(p.float(), torch.ones(2, 4))
    with pytest.raises(ValueError):
        dequantize_int4(p, torch.ones(3, 4))
    with pytest.raises(ValueError):
        dequantize_int4(p, torch.ones(2, 4), d_head=0)


def test_attention_validation_errors_match_reference():
    from kernels.gpt2.attention_quant import attention_forward_quant
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    q = torch.randn(1, 8, 1, 128, dtype=torch.bfloat16)
    kp = torch.zeros(1, 4, 32, 64, dtype=torch.uint8)
    ks = torch.ones(1, 4, 32, 4, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        attention_forward_quant_gqa(q, kp, ks, kp, ks, n_q_heads=7, n_kv_heads=4)
    with pytest.raises(ValueError):
        attention_forward_quant_gqa(q, kp, ks, kp, ks, n_q_heads=8, n_kv_heads=3)
    with pytest.raises(ValueError, match="CUDA"):
        attention_forward_quant_gqa(q, kp, ks, kp, ks, n_q_heads=8, n_kv_heads=4)
    with pytest.raises(ValueError, match="CUDA"):
        attention_forward_quant(q.float(), kp, ks, kp, ks)


def test_cache_host_logic_validation():
    from models.gpt2.kv_cache import QuantizedKVCache as G
    from models.llama3.kv_cache import QuantizedKVCache as L
    with pytest.raises(ValueError):
        L(group_size=0)
    c = L(group_size=32)
    assert c.get_seq_length(0) == 0 and len(c) == 0 and not c.is_initialized
    assert c.get_mask_sizes(torch.arange(5), 0) == (5, 0)
    assert c.get_mask_sizes(3, 0) == (3, 0)
    assert c.get_max_cache_shape() == -1
    with pytest.raises(KeyError):
        c.get_quantized(0)
    with pytest.raises(ValueError, match="CUDA"):
        c.append(torch.randn(1, 2, 3, 64), torch.randn(1, 2, 3, 64), 0)
    g = G()
    assert g.get_max_cache_shape() is None
    with pytest.raises(KeyError):
        g.get_dequantized(1)
