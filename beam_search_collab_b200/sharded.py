"""Index sharding across GPUs, one process per GPU.

For an index too large for one GPU the base is cut into contiguous row
ranges, one per rank, and each rank builds its own graph over its own rows
(the reference `build_graph` run on the shard's vectors) and its own index.
Every query is searched on every shard; each shard returns its K best
(distance, shard-local id) entries, the shards' lists are all-gathered over
NCCL (NVLink) and merged on the GPU into the K best (distance, global id)
entries -- the one exchange on the path (bs_merge_shards).

The reference searches one index on one GPU and has no counterpart; the
per-shard search is bs_search unchanged (same semantics, same results as the
reference CPU search on that shard's graph).

The collective and the id bookkeeping are written against torch.distributed
only, so they run under NCCL on GPUs and under gloo on CPU (the tests).
"""
from __future__ import annotations

from typing import Sequence


def shard_bounds(n: int, shards: int, shard: int) -> tuple[int, int]:
    """Rows [lo, hi) of `shard` when n rows are cut into `shards` contiguous
    ranges whose sizes differ by at most one."""
    if not 0 <= shard < shards:
        raise ValueError(f"shard {shard} outside 0..{shards - 1}")
    base, extra = divmod(n, shards)
    lo = shard * base + min(shard, extra)
    return lo, lo + base + (1 if shard < extra else 0)


def shard_offsets(n_local: int, group=None) -> list[int]:
    """Global id of every rank's first row: the exclusive prefix sum of the
    ranks' shard sizes (one small all-gather)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dev = _collective_device(group)
    mine = torch.tensor([n_local], dtype=torch.int64, device=dev)
    sizes = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(sizes, mine, group=group)
    out, acc = [], 0
    for s in sizes:
        out.append(acc)
        acc += int(s.item())
    if acc >= 0xFFFFFFFF:
        raise ValueError("global ids must stay below 0xffffffff")
    return out


def gather_shard_results(ids, dists, group=None):
    """All-gathers every rank's [nq, K] result lists (int32 shard-local ids,
    -1 = none; float32 distances) in one collective.  Returns ids and dists
    of shape [world, nq, K], rank r's lists at index r, on the inputs' device."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    nq, K = ids.shape
    # one message per rank: id and distance bits side by side
    packed = torch.stack([ids.to(torch.int32), dists.to(torch.float32).view(torch.int32)], dim=-1).contiguous()
    out = torch.empty((world * nq, K, 2), dtype=torch.int32, device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)
    out = out.view(world, nq, K, 2)
    return out[..., 0].contiguous(), out[..., 1].contiguous().view(torch.float32)


def _collective_device(group):
    import torch
    import torch.distributed as dist
    backend = dist.get_backend(group)
    return torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")


class ShardedIndex:
    """This rank's shard of a sharded index (`index`, a beam_search_collab_b200
    Index over rows [offset, offset + n_local) of the global base)."""

    def __init__(self, index, n_local: int, group=None):
        self.index = index
        self.group = group
        self.offsets: Sequence[int] = shard_offsets(n_local, group)

    @classmethod
    def from_arrays(cls, vectors, edges, device: int = 0, group=None) -> "ShardedIndex":
        """`vectors` [n_local, dim] and `edges` [n_local, degree] of this
        rank's shard (edges in shard-local ids)."""
        from . import Index
        return cls(Index.from_arrays(vectors, edges, device=device), len(vectors), group)

    def search(self, queries, K_out: int | None = None, **params):
        """Searches the same queries (a CUDA tensor on this rank's device,
        identical on every rank) on this shard, exchanges the shards' lists and
        returns the merged (ids [nq, K_out] int32 global ids, dists) on every
        rank.  `params` are bs_search's (mode, K, topk_size, ...)."""
        from . import merge_shards
        ids, dists, _ = self.index.search(queries, **params)
        ids_all, dists_all = gather_shard_results(ids, dists, self.group)
        K = ids.shape[1]
        return merge_shards(dists_all, ids_all, self.offsets, K_out or K)
