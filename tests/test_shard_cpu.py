"""Host logic of the multi-GPU layer on CPU: shard ranges, KV-head ownership,
and the sequence-shard exchange (gather of (o, lse) partials) over a real
2-rank gloo process group, merged and checked against unsharded attention
(the oracle stands in for the GPU partial kernel here)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import int4_oracle as orc


def test_shard_range_covers_and_balances():
    from kvint4.shard import shard_range
    for n in (0, 1, 7, 4096, 131073):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_head_shard():
    from kvint4.shard import head_shard
    assert head_shard(32, 8, 8, 3) == ((3, 4), (12, 16))
    assert head_shard(64, 8, 2, 1) == ((4, 8), (32, 64))
    with pytest.raises(ValueError):
        head_shard(32, 8, 3, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, k, v, sk, causal, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kvint4.shard import gather_partials, shard_range
        a, e = shard_range(sk, world, rank)
        o, lse = orc.partial_attention(q, k[:, :, a:e], v[:, :, a:e], n_q_heads=q.shape[1],
                                       n_kv_heads=k.shape[1], is_causal=causal, k_offset=a,
                                       sk_total=sk)
        all_o, all_lse = gather_partials(torch.from_numpy(o).float(),
                                         torch.from_numpy(lse).float())
        merged = orc.lse_combine(list(all_o.double().numpy()), list(all_lse.double().numpy()))
        results[rank] = merged.reshape(q.shape)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,causal", [(2, False), (2, True), (3, True)])
def test_sequence_shard_exchange_gloo(world, causal):
    rng = np.random.default_rng(world)
    q = rng.standard_normal((1, 8, 2, 64))
    k = rng.standard_normal((1, 2, 301, 64))
    v = rng.standard_normal((1, 2, 301, 64))
    full = orc.attention(q, k, v, n_q_heads=8, n_kv_heads=2, is_causal=causal)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, q, k, v, 301, causal, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        for r in range(world):
            np.testing.assert_allclose(results[r], full, atol=1e-5)


def _dropout_worker(rank, world, port, results):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the exchange
    from kvint4.shard import gather_partials
    try:
        gather_partials(torch.zeros(1, 2, 1, 8), torch.zeros(1, 2, 1))
        results[rank] = "no error"
    except Exception as e:  # the survivor learns of the loss on the host
        results[rank] = type(e).__name__


def test_rank_loss_surfaces_as_host_error():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert results.get(0) not in (None, "no error")
