"""Calls with tensors on one GPU while another GPU is current.

A model spread over several GPUs (``device_map``) calls the patched attention
for a layer on cuda:k while cuda:0 is current; the library must launch on
the tensors' device (tensor maps, occupancy and the smem attribute are per
device)."""

from __future__ import annotations

import pytest
import torch

from helpers import kv_inputs

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _run(dev):
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from kernels.llama3.quantize import quantize_int4
    k, v = kv_inputs(2, 8, 3000, 128, seed=11, device=dev)
    q = torch.randn(2, 32, 1, 128, generator=torch.Generator().manual_seed(12)).to(
        torch.bfloat16).to(dev)
    kp, ks = quantize_int4(k, group_size=32)
    vp, vs = quantize_int4(v, group_size=32)
    return kp, ks, attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8)


def test_ops_on_cuda1_while_cuda0_current():
    with torch.cuda.device(0):
        kp, ks, out = _run("cuda:1")  # the first launches on cuda:1, with cuda:0 current
        torch.cuda.synchronize("cuda:1")
    with torch.cuda.device(1):
        kp1, ks1, ref = _run("cuda:1")
        torch.cuda.synchronize()
    assert out.device.index == 1
    assert torch.equal(kp, kp1) and torch.equal(ks, ks1)
    assert torch.equal(out, ref)
