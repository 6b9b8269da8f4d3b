"""Multi-GPU layouts of the MLA decode layer (one process per GPU).

* Batch sharding (`batch_shard`): sequences are independent, so each rank owns
  a contiguous slice of the batch and its KV cache; no collective on the data
  path.
* Key sharding (`key_shard`, `sk_sharded_attention`): for long contexts with
  few sequences every rank owns a contiguous slice of each sequence's keys,
  runs the attention on it (mla_attention_partial), all-gathers the partial
  outputs and their log-sum-exp over NCCL, and merges them with lse_combine.
  The merge is exact; the message per rank is B*Sq*H*(V + 1) values.

The reference implementation is single-GPU; this module has no counterpart there.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def _split(n: int, rank: int, world: int) -> Tuple[int, int]:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def batch_shard(batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) of the sequences owned by `rank`."""
    return _split(batch, rank, world)


def key_shard(sk: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) of the keys owned by `rank` (sizes differ by at most one)."""
    return _split(sk, rank, world)


def gather_partials(out: torch.Tensor, lse: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's partial (out, lse) into [world, ...] tensors (rank order)."""
    world = dist.get_world_size(group)
    outs = [torch.empty_like(out) for _ in range(world)]
    lses = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(outs, out.contiguous(), group=group)
    dist.all_gather(lses, lse.contiguous(), group=group)
    return torch.stack(outs), torch.stack(lses)


def sk_sharded_attention(q_absorbed, q_rope, c_kv_local, pe_local, W_uv, scale: float, group=None,
                         precision: Optional[str] = None) -> torch.Tensor:
    """Attention over keys sharded across the ranks of `group`: every rank passes
    the same queries and its own key shard; every rank gets the full output."""
    import mla_custom_cuda as mcc
    out, lse = mcc.mla_attention_partial(q_absorbed, q_rope, c_kv_local, pe_local, W_uv, scale,
                                         precision=precision)
    outs, lses = gather_partials(out, lse, group)
    merged, _ = mcc.lse_combine(outs, lses)
    return merged
