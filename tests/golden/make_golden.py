"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once in a container that has the reference checkout (read-only) and its
CPU dependencies (torch, triton for the import only):

    python tests/golden/make_golden.py --reference /path/to/kv-cache-triton

It imports the reference's own CPU functions -- nothing is copied:
  * ``kernels/llama3/quantize.py``: ``_quantize_int4_torch`` (:126-148),
    ``_dequantize_int4_torch`` (:210-234)  (scales keep the input dtype)
  * ``kernels/gpt2/quantize.py``: ``_quantize_int4_torch`` (:111-133),
    ``_dequantize_int4_torch`` (:217-235)  (scales always fp16)
  * ``tests/llama3/test_attention_fused_vs_ref_sm70.py::_gqa_ref`` (:14-51),
    the reference's looped fp32 GQA attention with bottom-right causal mask,
    and ``torch.nn.functional.scaled_dot_product_attention`` as used by
    ``tests/llama3/test_attention_quant_gqa.py:38-40``.
and writes ``quant_cases.npz`` and ``attn_cases.npz`` next to this script.
16-bit floats are stored as their raw uint16 bit patterns.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def _dtype_name(dt: torch.dtype) -> str:
    return {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[dt]


def quant_inputs():
    g = torch.Generator().manual_seed(0)
    cases = []

    def rnd(shape, dtype, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dtype)

    for dt in (torch.bfloat16, torch.float16, torch.float32):
        for gs in (32, 64, 128):
            cases.append((f"randn_{_dtype_name(dt)}_g{gs}", rnd((2, 3, 5, 128), dt), gs))
    cases.append(("d64_f16_g32", rnd((2, 3, 5, 64), torch.float16), 32))
    cases.append(("d70_f32_g32", rnd((2, 2, 3, 70), torch.float32), 32))
    cases.append(("d12_f32_g5_odd", rnd((3, 12), torch.float32), 5))
    cases.append(("d64_bf16_g128_pad", rnd((2, 4, 64), torch.bfloat16), 128))
    cases.append(("zeros_f16_g32", torch.zeros(1, 2, 4, 64, dtype=torch.float16), 32))
    cases.append(("tiny_bf16_g32", rnd((2, 4, 128), torch.bfloat16, 1e-6), 32))
    out = rnd((2, 4, 128), torch.float32)
    out[:, :, 7] *= 5000.0
    out[:, 1, 77] = -5000.0
    cases.append(("outlier_f32_g32", out, 32))
    # exact ties of x/scale at k + 0.5 (max = 7 -> scale = 1)
    ties = torch.zeros(4, 32, dtype=torch.float32)
    ties[0, :8] = torch.tensor([0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 6.5, -6.5])
    ties[0, 31] = 7.0
    ties[1, :6] = torch.tensor([3.5, -3.5, 4.5, -4.5, 5.5, -7.5])
    ties[1, 30] = -7.0
    ties[2, :] = torch.linspace(-7.0, 7.0, 32)
    ties[3, :4] = torch.tensor([0.49999997, -0.49999997, 7.0, 1e-30])
    cases.append(("ties_f32_g32", ties, 32))
    cases.append(("ties_bf16_g32", ties.to(torch.bfloat16), 32))
    # bf16 rows whose scale is not a power of two (many near-ties)
    nt = (torch.randint(-14, 15, (8, 64), generator=g).float() * 0.5).to(torch.bfloat16)
    nt[:, 0] = 7.0
    cases.append(("halfsteps_bf16_g32", nt, 32))
    return cases


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("KV4_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from kernels.gpt2 import quantize as gq  # noqa: E402
    from kernels.llama3 import quantize as lq  # noqa: E402
    from tests.llama3.test_attention_fused_vs_ref_sm70 import _gqa_ref  # noqa: E402
    import torch.nn.functional as F  # noqa: E402

    here = os.path.dirname(os.path.abspath(__file__))
    qd = {}
    for name, x, gs in quant_inputs():
        d = x.shape[-1]
        for flavour, mod in (("llama3", lq), ("gpt2", gq)):
            key = f"{flavour}.{name}"
            packed, scales = mod._quantize_int4_torch(x, gs)
            if flavour == "llama3":
                deq = mod._dequantize_int4_torch(packed, scales, group_size=gs, d_head=d,
                                                 out_dtype=torch.float32)
            else:
                deq = mod._dequantize_int4_torch(packed, scales, group_size=gs, d_head=d)
            qd[f"{key}.x"] = _bits(x)
            qd[f"{key}.x_dtype"] = np.array(_dtype_name(x.dtype))
            qd[f"{key}.group_size"] = np.array(gs)
            qd[f"{key}.packed"] = packed.numpy()
            qd[f"{key}.scales"] = _bits(scales)
            qd[f"{key}.scale_dtype"] = np.array(_dtype_name(scales.dtype))
            qd[f"{key}.deq"] = _bits(deq)
            qd[f"{key}.deq_dtype"] = np.array(_dtype_name(deq.dtype))
    np.savez_compressed(os.path.join(here, "quant_cases.npz"), **qd)

    ad = {}
    g = torch.Generator().manual_seed(1)
    attn_cases = [
        # name, b, n_q, n_kv, sq, sk, d, gs, causal, q dtype
        ("decode_gqa4_d128", 2, 8, 2, 1, 77, 128, 32, False, torch.bfloat16),
        ("decode_mha_d64", 1, 4, 4, 1, 96, 64, 32, False, torch.float16),
        ("decode_gqa8_d128_g64", 1, 8, 1, 1, 130, 128, 64, False, torch.float32),
        ("prefill_causal_square", 1, 4, 2, 16, 16, 128, 32, True, torch.bfloat16),
        ("chunk_causal_bottom_right", 1, 4, 2, 5, 37, 64, 32, True, torch.float32),
        ("multiq_noncausal", 1, 8, 2, 3, 40, 128, 128, False, torch.bfloat16),
    ]
    for (name, b, hq, hkv, sq, sk, d, gs, causal, qdt) in attn_cases:
        q = torch.randn(b, hq, sq, d, generator=g).to(qdt)
        kx = torch.randn(b, hkv, sk, d, generator=g)
        kx = kx * torch.exp(torch.empty(d).uniform_(np.log(0.5), np.log(8.0), generator=g))
        kx = kx.to(qdt)
        vx = torch.randn(b, hkv, sk, d, generator=g).to(qdt)
        kp, ks = lq._quantize_int4_torch(kx, gs)
        vp, vs = lq._quantize_int4_torch(vx, gs)
        kd = lq._dequantize_int4_torch(kp, ks, group_size=gs, d_head=d, out_dtype=torch.float32)
        vd = lq._dequantize_int4_torch(vp, vs, group_size=gs, d_head=d, out_dtype=torch.float32)
        out = _gqa_ref(q.float(), kd, vd, n_q_heads=hq, n_kv_heads=hkv, scale=d ** -0.5,
                       is_causal=causal)
        ad[f"{name}.meta"] = np.array([b, hq, hkv, sq, sk, d, gs, int(causal)])
        ad[f"{name}.q"] = _bits(q)
        ad[f"{name}.q_dtype"] = np.array(_dtype_name(qdt))
        ad[f"{name}.k_packed"] = kp.numpy()
        ad[f"{name}.k_scales"] = _bits(ks)
        ad[f"{name}.v_packed"] = vp.numpy()
        ad[f"{name}.v_scales"] = _bits(vs)
        ad[f"{name}.scale_dtype"] = np.array(_dtype_name(ks.dtype))
        ad[f"{name}.out_ref_f32"] = out.float().numpy()
        if not causal or sq == sk:
            rep = hq // hkv
            sd = F.scaled_dot_product_attention(
                q.float(), kd.repeat_interleave(rep, 1), vd.repeat_interleave(rep, 1),
                is_causal=causal)
            ad[f"{name}.out_sdpa_f32"] = sd.numpy()
    np.savez_compressed(os.path.join(here, "attn_cases.npz"), **ad)
    print("wrote", len(qd), "quant arrays and", len(ad), "attention arrays")


if __name__ == "__main__":
    main()
