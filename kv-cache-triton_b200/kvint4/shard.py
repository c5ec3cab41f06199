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
  log-sum-exp), the partials are all-gathered (NCCL over NVLink on B200) and
  merged with ``kv4_lse_combine``:
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
    """All-gather every rank's (o, lse) partial: returns contiguous
    ``[P, rows, d]`` and ``[P, rows]`` float32 tensors."""
    world = dist.get_world_size(group)
    rows = part_lse.numel()
    d = part_o.shape[-1]
    o = part_o.reshape(rows, d).contiguous()
    lse = part_lse.reshape(rows).contiguous()
    if dist.get_backend(group) == "nccl":
        all_o = torch.empty(world, rows, d, dtype=o.dtype, device=o.device)
        all_lse = torch.empty(world, rows, dtype=lse.dtype, device=lse.device)
        dist.all_gather_into_tensor(all_o, o, group=group)
        dist.all_gather_into_tensor(all_lse, lse, group=group)
        return all_o, all_lse
    lo = [torch.empty_like(o) for _ in range(world)]
    ll = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(lo, o, group=group)
    dist.all_gather(ll, lse, group=group)
    return torch.stack(lo), torch.stack(ll)


def seq_sharded_attention(q: torch.Tensor, k_packed, k_scales, v_packed, v_scales, *,
                          k_offset: int, sk_total: int, group_size: int = 32,
                          is_causal: bool = False, group=None,
                          out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of ``q`` over a sequence whose keys are spread over the ranks
    of ``group``; this rank holds keys ``[k_offset, k_offset + sk_local)``.
    Every rank returns the full result."""
    b, hq, sq, d = q.shape
    part_o = torch.empty(b, hq, sq, d, dtype=torch.float32, device=q.device)
    part_lse = torch.empty(b, hq, sq, dtype=torch.float32, device=q.device)
    ops.attention_partial_into(q, k_packed, k_scales, v_packed, v_scales, part_o, part_lse,
                               k_offset, sk_total, group_size, is_causal)
    all_o, all_lse = gather_partials(part_o, part_lse, group)
    if out is None:
        out = torch.empty(b, hq, sq, d, dtype=q.dtype, device=q.device)
    ops.lse_combine_into(all_o, all_lse, out)
    return out
