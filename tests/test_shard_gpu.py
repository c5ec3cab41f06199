"""Sequence-sharded decode through NCCL on one GPU (world size 1 in a child
process) and the shard split emulated on one GPU: both equal the unsharded
fused kernel / the oracle."""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from helpers import f32, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_seq_sharded_attention_nccl_world1():
    code = textwrap.dedent(f"""
        import os, sys, socket, torch, torch.distributed as dist
        sys.path[:0] = [{os.path.join(ROOT, 'kv-cache-triton_b200')!r}, {ROOT!r},
                        {os.path.join(ROOT, 'tests')!r}]
        s = socket.socket(); s.bind(("127.0.0.1", 0)); port = s.getsockname()[1]; s.close()
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(0)
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
        from kvint4.cache import Int4KVStore
        from kvint4.shard import seq_sharded_attention
        from kernels.llama3.attention_quant import attention_forward_quant_gqa
        from helpers import kv_inputs
        k, v = kv_inputs(2, 2, 999, 128, device="cuda", seed=5)
        st = Int4KVStore(32); st.append(k, v, 0)
        kp, ks, vp, vs = st.layer(0).views()
        q = torch.randn(2, 8, 1, 128, device="cuda").to(torch.bfloat16)
        a = seq_sharded_attention(q, kp, ks, vp, vs, k_offset=0, sk_total=999)
        b = attention_forward_quant_gqa(q, kp, ks, vp, vs, n_q_heads=8, n_kv_heads=2)
        err = (a.float() - b.float()).abs().max().item()
        dist.destroy_process_group()
        assert err <= 2e-2, err
        print("ok", err)
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


def test_four_sequence_shards_on_one_gpu_match_oracle():
    """Four shards of a causal multi-query decode, each through the partial
    kernel at its own key offset, merged by the combine kernel."""
    from kvint4 import ops
    from kvint4.cache import Int4KVStore
    from kvint4.shard import shard_range
    sk = 2049
    k, v = kv_inputs(1, 8, sk, 128, device="cuda", seed=6)
    q = torch.randn(1, 32, 2, 128, device="cuda").to(torch.bfloat16)
    parts_o, parts_l = [], []
    full_store = Int4KVStore(32)
    full_store.append(k, v, 0)
    for r in range(4):
        a, e = shard_range(sk, 4, r)
        st = Int4KVStore(32)
        st.append(k[:, :, a:e], v[:, :, a:e], 0)
        po = torch.empty(1, 32, 2, 128, device="cuda")
        pl = torch.empty(1, 32, 2, device="cuda")
        ops.attention_partial_into(q, *st.layer(0).views(), po, pl, a, sk, 32, True)
        parts_o.append(po.reshape(-1, 128))
        parts_l.append(pl.reshape(-1))
    out = torch.empty(1, 32, 2, 128, device="cuda", dtype=torch.bfloat16)
    ops.lse_combine_into(torch.stack(parts_o), torch.stack(parts_l), out)
    kp, ks, vp, vs = full_store.layer(0).views()
    ref = oracle_attention(q, kp, ks, vp, vs, n_q_heads=32, n_kv_heads=8, group_size=32,
                           is_causal=True)
    np.testing.assert_allclose(f32(out), ref, atol=2e-2, rtol=0)


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run_exchange(world: int):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port",
           str(_free_port()), os.path.join(ROOT, "tests", "exchange_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_peer_exchange_world1():
    """kv4_lse_exchange with one rank (its own buffer as the only peer)."""
    _run_exchange(1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_two_gpus():
    """Sequence shards on two GPUs merged over peer memory, eagerly and from
    a CUDA graph, equal the unsharded kernel."""
    _run_exchange(2)
