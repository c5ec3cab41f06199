"""Worker for the peer-memory exchange tests (tests/test_shard_gpu.py): every
rank holds its shard of one batch-1 long-context cache, runs the partial
kernel plus kv4_lse_exchange eagerly and from a CUDA graph, and compares the
merged output with the unsharded fused kernel on the whole cache.  Launched
with torch.distributed.run; prints "ok <max error>" on rank 0."""

from __future__ import annotations

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "kv-cache-triton_b200"), ROOT, os.path.join(ROOT, "tests")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    from helpers import kv_inputs
    from kernels.llama3.attention_quant import attention_forward_quant_gqa
    from kvint4.cache import Int4KVStore
    from kvint4.shard import PeerExchange, seq_sharded_attention, shard_range

    sk = int(os.environ.get("KV4_SK", "20000"))
    k, v = kv_inputs(1, 8, sk, 128, device=dev, seed=21)  # same cache on every rank
    full = Int4KVStore(32)
    full.append(k, v, 0)
    a, e = shard_range(sk, world, rank)
    mine = Int4KVStore(32)
    mine.append(k[:, :, a:e], v[:, :, a:e], 0)
    del k, v
    views = mine.layer(0).views()
    xchg = PeerExchange(rows=32, d=128, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    worst = 0.0
    q = torch.empty(1, 32, 1, 128, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)

    def step():
        seq_sharded_attention(q, *views, k_offset=a, sk_total=sk, out=out, exchange=xchg)

    def check():
        ref = attention_forward_quant_gqa(q, *full.layer(0).views(), n_q_heads=32, n_kv_heads=8)
        return (out.float() - ref.float()).abs().max().item()

    for _ in range(5):  # eager calls: epochs 1..5, both buffer halves
        q.copy_(torch.randn(q.shape, device=dev, generator=g))
        step()
        worst = max(worst, check())
    step()  # warm the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(4):  # replays: the epoch advances on the device
        q.copy_(torch.randn(q.shape, device=dev, generator=g))
        graph.replay()
        worst = max(worst, check())
    from kvint4 import ops
    errword = ops.device_error(dev)
    t = torch.tensor([worst, float(errword)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        assert t[1].item() == 0, f"device error word {t[1].item()}"
        assert t[0].item() <= 2e-2, t[0].item()
        print("ok", t[0].item())


if __name__ == "__main__":
    main()
