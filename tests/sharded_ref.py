"""Test-side restatement of the shard merge (numpy), and the seeded sharded
data set shared by the CPU (gloo) and GPU tests."""
import numpy as np

import oracle as O
from beam_search_collab_b200.sharded import shard_bounds

NO = 0xFFFFFFFF


def merge_ref(ids_all, dists_all, offsets, K_out):
    """K_out smallest (distance, global id) over the shards' lists; ids are
    shard-local u32 (0xffffffff = none)."""
    S, nq, K = ids_all.shape
    out_i = np.full((nq, K_out), NO, dtype=np.uint32)
    out_d = np.full((nq, K_out), np.finfo(np.float32).max, dtype=np.float32)
    for q in range(nq):
        gid, d = [], []
        for s in range(S):
            keep = ids_all[s, q] != NO
            gid.append(ids_all[s, q][keep].astype(np.uint64) + offsets[s])
            d.append(dists_all[s, q][keep])
        gid = np.concatenate(gid)
        d = np.concatenate(d)
        order = np.lexsort((gid, d))[:K_out]
        out_i[q, :len(order)] = gid[order]
        out_d[q, :len(order)] = d[order]
    return out_i, out_d


def dataset(n=3000, dim=24, deg=12, nq=64, seed=7):
    """Seeded float base with a random graph per shard built later."""
    rng = np.random.default_rng(seed)
    base = (rng.standard_normal((n, dim)) * 3).astype(np.float32)
    queries = (rng.standard_normal((nq, dim)) * 3).astype(np.float32)
    return base, queries


def shard(base, shards, s, deg=12, seed=11):
    """Rows and a random degree-`deg` graph (shard-local ids) of shard s."""
    lo, hi = shard_bounds(len(base), shards, s)
    rng = np.random.default_rng(seed + s)
    m = hi - lo
    edges = rng.integers(0, m, size=(m, deg), dtype=np.uint32)
    return lo, base[lo:hi], edges


def oracle_shard_search(vecs, edges, queries, K, topk):
    r = O.search(vecs, edges, queries, K=K, topk_size=topk, entry=O.entry_point(vecs))
    return r.ids.astype(np.uint32), r.dists.astype(np.float32)
