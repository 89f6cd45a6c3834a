"""KV-head-sharded paged decode across GPUs.

Sequence sharding needs no collective (every rank owns whole sequences).  The
alternative for a batch that must stay on every rank is to shard the KV heads:
rank r keeps kv heads [r*H/N, (r+1)*H/N) of every sequence (and serves the
query heads of those groups), runs the paged GQA decode on its slice, and the
per-layer outputs — disjoint head ranges, so no reduction — are all-gathered:
``B x Hq x D`` elements per layer (1 MiB at B = 128, Hq = 32, D = 128, bf16).

The collective is ``torch.distributed.all_gather_into_tensor`` (NCCL over
NVLink on GPUs; gloo works for the host-side tests), followed by one reorder
of the gathered ``[N, B, Hq/N, D]`` into ``[B, Hq, D]``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_range(n_heads: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the heads rank ``rank`` owns; heads split evenly."""
    if n_heads % world != 0:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    per = n_heads // world
    return rank * per, (rank + 1) * per


def shard_query(q: torch.Tensor, n_kv_heads: int, world: int, rank: int) -> torch.Tensor:
    """The query heads of this rank's kv heads: q [B, Hq, D] -> [B, Hq/N, D] (a view)."""
    n_q = q.shape[1]
    group = n_q // n_kv_heads
    lo, hi = head_range(n_kv_heads, world, rank)
    return q[:, lo * group: hi * group]


def gather_heads(local_out: torch.Tensor, world: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather the per-rank head slices [B, Hq/N, D] into [B, Hq, D]."""
    b, hl, d = local_out.shape
    gathered = torch.empty((world, b, hl, d), dtype=local_out.dtype, device=local_out.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local_out.contiguous(), group=group)
    else:  # gloo (host-side tests) has only the list form
        dist.all_gather(list(gathered.unbind(0)), local_out.contiguous(), group=group)
    if out is None:
        out = torch.empty((b, world * hl, d), dtype=local_out.dtype, device=local_out.device)
    out.view(b, world, hl, d).copy_(gathered.permute(1, 0, 2, 3))
    return out


class HeadShardedDecode:
    """Paged GQA decode over a PagedKVPool that holds this rank's kv-head slice."""

    def __init__(self, pool, n_q_heads: int, world: int, rank: int, group=None):
        self.pool, self.world, self.rank, self.group = pool, world, rank, group
        self.n_q_heads = n_q_heads
        self.n_kv_total = pool.n_kv_heads * world
        if n_q_heads % self.n_kv_total != 0:
            raise ValueError("query heads must be a multiple of the kv heads")

    def decode(self, layer: int, q: torch.Tensor, out: torch.Tensor | None = None, **kw) -> torch.Tensor:
        """q [B, Hq, D] (all heads) -> out [B, Hq, D] (all heads, on every rank)."""
        q_local = shard_query(q, self.n_kv_total, self.world, self.rank)
        local = self.pool.decode(layer, q_local, **kw)
        return gather_heads(local, self.world, self.group, out)
