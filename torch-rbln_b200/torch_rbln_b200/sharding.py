"""KV-head sharding of paged decode across the GPUs of one node.

The reference has no model-parallel attention of its own: its only
collective is an all-gather through ProcessGroupRBLN
(torch_rbln/csrc/distributed/c10d/rbln/ProcessGroupRBLN.cpp:754-830), used
by tests that shard tensors by hand (test/distributed/test_tp_pp.py:268).
Here one process drives one GPU: rank r owns a contiguous slice of the KV
heads (its slice of the paged KV pool and the matching query heads), runs
rbln_custom_ops.paged_causal_attn_decode on it, and one all-gather of the
per-rank head outputs rebuilds [B, Hkv, G, 1, D] on every rank. The block
table and sequence lengths are replicated. That all-gather is the only
exchange (NCCL over NVLink / NVSwitch on GPUs, gloo on CPU).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [h0, h1) slice of KV heads owned by `rank`."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def shard_heads(t: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    """The rank's slice of a [.., Hkv, ..] tensor along `dim` (a view)."""
    h0, h1 = kv_head_range(t.shape[dim], rank, world)
    return t.narrow(dim, h0, h1 - h0)


def all_gather_heads(out_local: torch.Tensor, world: int, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """[B, Hkv/world, G, S, D] per rank -> [B, Hkv, G, S, D] on every rank,
    heads in rank order."""
    if world == 1:
        return out_local
    x = out_local.contiguous()
    buf = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, x, group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), x, group=group)
    B, h, G, S, D = x.shape
    return buf.permute(1, 0, 2, 3, 4, 5).reshape(B, world * h, G, S, D)


def head_sharded_paged_decode(q, k, v, kcache_local, vcache_local, seq, scale, block_table, block_size,
                              mask=None, *, rank: int, world: int, group=None):
    """paged_causal_attn_decode with the KV heads split over `world` ranks.

    q, k, v hold all heads ([B, Hkv, G|1, 1, D], replicated); the caches hold
    only this rank's heads. Returns the full [B, Hkv, G, 1, D] output on
    every rank (one all-gather)."""
    ql, kl, vl = (shard_heads(t, rank, world) for t in (q, k, v))
    out_local = torch.ops.rbln_custom_ops.paged_causal_attn_decode(
        ql.contiguous(), kl.contiguous(), vl.contiguous(), kcache_local, vcache_local, seq, scale, block_table,
        block_size, mask)
    return all_gather_heads(out_local, world, group)
