"""Multi-GPU sharding of the INT4 decode (one process per GPU).

The reference has no multi-GPU layer of its own (it places whole layers on
GPUs through accelerate, ``benchmarks/llama3/run_llama3_benchmark.py:115-121``).
Two ways to split one decode step over ranks:

* KV-head (or batch) sharding: rank r owns KV heads
  ``[r*Hkv/P, (r+1)*Hkv/P)`` and their q heads.  Attention per KV group is
  independent, so there is no collective on the data path; outputs stay
  head-sharded, as a tensor-parallel output projection consumes them.
* Sequence sharding (batch-1 long context): rank r owns key positions
  ``shard_range(S, P, r)``.  Each rank computes softmax partials over its
  tokens (``kv4_attention_partial``: o normalised within the shard plus its
  log-sum-exp), then either pushed into every rank's buffer over NVLink
  and merged in one kernel (``PeerExchange``, ``kv4_lse_exchange``) or
  all-gathered in one collective and merged with ``kv4_lse_combine``:
  ``o = sum_r o_r exp(lse_r - lse*) / sum_r exp(lse_r - lse*)``.
  The payload is tiny (B*Hq*sq*(d+1) floats per rank), so the exchange is
  latency-bound; the new token is appended on the rank that owns its
  position (the last rank).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [start, end) of ``n`` items owned by ``rank``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def head_shard(n_q_heads: int, n_kv_heads: int, world: int, rank: int):
    """KV heads and q heads owned by ``rank`` under KV-head sharding."""
    if n_kv_heads % world:
        raise ValueError("n_kv_heads must be divisible by the world size")
    if n_q_heads % n_kv_heads:
        raise ValueError("n_q_heads must be divisible by n_kv_heads")
    per = n_kv_heads // world
    ratio = n_q_heads // n_kv_heads
    kv = (rank * per, (rank + 1) * per)
    return kv, (kv[0] * ratio, kv[1] * ratio)


def gather_partials(part_o: torch.Tensor, part_lse: torch.Tensor, group=None):
    """All-gather every rank's (o, lse) partial in ONE collective (o and lse
    packed into one float32 row of d + 1 values): returns contiguous
    ``[P, rows, d]`` and ``[P, rows]`` float32 tensors."""
    world = dist.get_world_size(group)
    rows = part_lse.numel()
    d = part_o.shape[-1]
    packed = torch.cat([part_o.reshape(rows, d).float(), part_lse.reshape(rows, 1).float()], 1)
    if dist.get_backend(group) == "nccl":
        allp = torch.empty(world, rows, d + 1, dtype=torch.float32, device=packed.device)
        dist.all_gather_into_tensor(allp, packed, group=group)
    else:
        parts = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(parts, packed, group=group)
        allp = torch.stack(parts)
    return allp[..., :d].contiguous(), allp[..., d].contiguous()


class PeerExchange:
    """Exchange of sequence-shard partials over peer memory (NVLink): one
    ``kv4_lse_exchange`` launch per step pushes this rank's (o, lse) into
    every rank's buffer, waits (bounded) for the others and merges, with no
    collective library and no host in the loop, so a step can sit in a CUDA
    graph.  The buffers are torch symmetric memory (``rows`` = B*Hq*sq rows
    of ``d`` values); every rank must make the same calls in the same order."""

    def __init__(self, rows: int, d: int, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        from ._lib import lib
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.rows, self.d = int(rows), int(d)
        nbytes = int(lib().kv4_lse_exchange_bytes(self.rows, self.d, self.world))
        if nbytes <= 0:
            raise ValueError("bad exchange geometry")
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64,
                                  device=device)
        self.state = torch.zeros(2, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)  # every buffer is zero before anyone writes

    def combine(self, part_o: torch.Tensor, part_lse: torch.Tensor, out: torch.Tensor) -> None:
        import ctypes

        from ._lib import check, lib
        if part_o.dtype != torch.float32 or part_lse.dtype != torch.float32:
            raise ValueError("partials must be float32")
        po, pl = part_o.contiguous(), part_lse.contiguous()
        d = ops.desc(out)
        check("kv4_lse_exchange",
              lib().kv4_lse_exchange(po.data_ptr(), pl.data_ptr(), self.rows, self.d,
                                     self.peers.data_ptr(), self.world, self.rank,
                                     self.state.data_ptr(), ctypes.byref(d),
                                     ops._stream(out.device)))


def seq_sharded_attention(q: torch.Tensor, k_packed, k_scales, v_packed, v_scales, *,
                          k_offset: int, sk_total: int, group_size: int = 32,
                          is_causal: bool = False, group=None,
                          out: torch.Tensor | None = None,
                          exchange: PeerExchange | None = None) -> torch.Tensor:
    """Attention of ``q`` over a sequence whose keys are spread over the ranks
    of ``group``; this rank holds keys ``[k_offset, k_offset + sk_local)``.
    Every rank returns the full result.  With ``exchange`` the partials
    travel over peer memory in one kernel; otherwise by one all-gather and
    ``kv4_lse_combine``."""
    b, hq, sq, d = q.shape
    part_o = torch.empty(b, hq, sq, d, dtype=torch.float32, device=q.device)
    part_lse = torch.empty(b, hq, sq, dtype=torch.float32, device=q.device)
    ops.attention_partial_into(q, k_packed, k_scales, v_packed, v_scales, part_o, part_lse,
                               k_offset, sk_total, group_size, is_causal)
    if out is None:
        out = torch.empty(b, hq, sq, d, dtype=q.dtype, device=q.device)
    if exchange is not None:
        exchange.combine(part_o, part_lse, out)
        return out
    all_o, all_lse = gather_partials(part_o, part_lse, group)
    ops.lse_combine_into(all_o, all_lse, out)
    return out
