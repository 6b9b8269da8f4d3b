"""Multi-GPU layouts of the MLA decode layer (one process per GPU).

* Batch sharding (`batch_shard`): sequences are independent, so each rank owns
  a contiguous slice of the batch and its KV cache; no collective on the data
  path.
* Key sharding (`key_shard`, `sk_sharded_attention`): for long contexts with
  few sequences every rank owns a contiguous slice of each sequence's keys,
  runs the attention on it (mla_attention_partial), all-gathers the partial
  outputs and their log-sum-exp over NCCL, and merges them with lse_combine.
  The merge is exact; the message per rank is B*Sq*H*(V + 1) values.
* Head-sharded Q-prep (`head_shard`, `shard_q_weights`, `head_sharded_q_absorbed`)
  for the key-sharded layout: Q-prep streams its weights on every GPU whatever
  the key shard, so at long context and small batch it caps the scaling. Each
  rank keeps only its heads' slices of W_q_b and W_uk, computes q for those
  heads (2a1 and the RMSNorm are repeated on every rank) and the ranks
  all-gather q (B*Sq*H*(kv_rank + rope) values) before the attention.

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


def head_shard(heads: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) of the heads whose queries `rank` computes."""
    return _split(heads, rank, world)


def shard_q_weights(W_q_b: torch.Tensor, W_uk: torch.Tensor, nope_dim: int, rope_dim: int, rank: int,
                    world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """This rank's heads of W_q_b [q_lora, H*(nope+rope)] and W_uk [H, nope, kv_rank],
    as contiguous tensors (done once, at weight-load time)."""
    heads = W_uk.shape[0]
    if heads % world:
        raise ValueError(f"{heads} heads do not split evenly over {world} ranks")
    h0, h1 = head_shard(heads, rank, world)
    qk = nope_dim + rope_dim
    return W_q_b[:, h0 * qk:h1 * qk].contiguous(), W_uk[h0:h1].contiguous()


def gather_heads(q_locals, group=None):
    """All-gather per-rank [B, Sq, H/world, d_i] tensors into [B, Sq, H, d_i] (heads
    in rank order), all of them in one collective."""
    world = dist.get_world_size(group)
    flat = torch.cat([q.reshape(-1) for q in q_locals])
    out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    if world == 1:
        out.copy_(flat)
    else:
        dist.all_gather_into_tensor(out, flat, group=group)
    out = out.view(world, -1)
    res, off = [], 0
    for q in q_locals:
        n = q.numel()
        B, Sq, Hl, d = q.shape
        part = out[:, off:off + n].view(world, B, Sq, Hl, d)          # [rank, B, Sq, Hl, d]
        res.append(part.permute(1, 2, 0, 3, 4).reshape(B, Sq, world * Hl, d))
        off += n
    return res


def head_sharded_q_absorbed(x, W_q_a, q_norm_w, W_q_b_local, W_uk_local, positions, nope_dim: int, rope_dim: int,
                            eps: float, group=None, precision: Optional[str] = None):
    """q_absorbed / q_rope of all heads from each rank's head slices of the weights
    (shard_q_weights): local Q-prep for H/world heads, then one all-gather of q."""
    import mla_custom_cuda as mcc
    qa, qr = mcc.q_absorbed_ex(x, W_q_a, q_norm_w, W_q_b_local, W_uk_local, positions, nope_dim, rope_dim, eps,
                               precision=precision)
    qa_all, qr_all = gather_heads([qa, qr], group)
    return qa_all, qr_all


def gather_partials(out: torch.Tensor, lse: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's partial (out, lse) into [world, ...] tensors (rank
    order), both in one collective (lse travels in out's dtype when that is fp32 or fp64)."""
    world = dist.get_world_size(group)
    if out.dtype != lse.dtype:   # 16-bit outputs: two collectives keep lse in fp32
        outs = torch.empty(world * out.numel(), dtype=out.dtype, device=out.device)
        lses = torch.empty(world * lse.numel(), dtype=lse.dtype, device=lse.device)
        dist.all_gather_into_tensor(outs, out.contiguous().reshape(-1), group=group)
        dist.all_gather_into_tensor(lses, lse.contiguous().reshape(-1), group=group)
        return outs.view((world,) + tuple(out.shape)), lses.view((world,) + tuple(lse.shape))
    flat = torch.cat([out.reshape(-1), lse.reshape(-1)])
    buf = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(buf, flat, group=group)
    buf = buf.view(world, -1)
    n = out.numel()
    return buf[:, :n].reshape((world,) + tuple(out.shape)), buf[:, n:].reshape((world,) + tuple(lse.shape))


def sk_sharded_attention(q_absorbed, q_rope, c_kv_local, pe_local, W_uv, scale: float, group=None,
                         precision: Optional[str] = None) -> torch.Tensor:
    """Attention over keys sharded across the ranks of `group`: every rank passes
    the same queries and its own key shard; every rank gets the full output.

    fp64 is rejected before any work: the shards' log-sum-exp travel in fp32,
    which would cap an fp64 merge at fp32 accuracy (mla_lse_combine has no fp64
    variant for that reason)."""
    if q_absorbed.dtype == torch.float64:
        raise RuntimeError("sk_sharded_attention: fp64 is not supported (the merge weights are fp32); "
                           "run fp64 attention unsharded")
    import mla_custom_cuda as mcc
    out, lse = mcc.mla_attention_partial(q_absorbed, q_rope, c_kv_local, pe_local, W_uv, scale,
                                         precision=precision)
    outs, lses = gather_partials(out, lse, group)
    merged, _ = mcc.lse_combine(outs, lses)
    return merged
