"""Index sharding, host side: row ranges, global id offsets and the
all-gather of the shards' result lists, run as two gloo ranks on CPU (each
rank searches its shard with the oracle; the product's collective exchanges
the lists; the merge is checked against merging the shards' oracle results
directly)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sharded_ref as R
from beam_search_collab_b200.sharded import gather_shard_results, shard_bounds, shard_offsets


@pytest.mark.parametrize("n,shards", [(10, 3), (1000, 8), (7, 7), (5, 8)])
def test_shard_bounds_cover_the_rows_once(n, shards):
    spans = [shard_bounds(n, shards, s) for s in range(shards)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(n, shards, shards)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, K, topk, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        base, queries = R.dataset()
        lo, vecs, edges = R.shard(base, world, rank)
        ids, dists = R.oracle_shard_search(vecs, edges, queries, K, topk)
        offsets = shard_offsets(len(vecs))
        ids_all, dists_all = gather_shard_results(torch.from_numpy(ids.view(np.int32)), torch.from_numpy(dists))
        out[rank] = (offsets, lo, ids_all.numpy().view(np.uint32).copy(), dists_all.numpy().copy())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_exchange_and_merge_shard_results():
    world, K, topk = 2, 10, 32
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.start_processes(_rank, args=(world, port, K, topk, out), nprocs=world, start_method="spawn")
        res = dict(out)
    base, queries = R.dataset()
    expect_ids, expect_d = [], []
    for s in range(world):
        lo, vecs, edges = R.shard(base, world, s)
        i, d = R.oracle_shard_search(vecs, edges, queries, K, topk)
        expect_ids.append(i)
        expect_d.append(d)
    expect_ids, expect_d = np.stack(expect_ids), np.stack(expect_d)
    offsets = [R.shard(base, world, s)[0] for s in range(world)]
    for r in range(world):
        got_off, lo, ids_all, dists_all = res[r]
        assert list(got_off) == offsets and lo == offsets[r]
        assert np.array_equal(ids_all, expect_ids)              # rank s's lists at index s
        assert np.array_equal(dists_all.view(np.uint32), expect_d.view(np.uint32))
    merged_i, merged_d = R.merge_ref(ids_all, dists_all, offsets, K)
    # every merged id is a true global row whose distance matches
    for q in range(len(queries)):
        for i, d in zip(merged_i[q], merged_d[q]):
            if i != R.NO:
                diff = base[i].astype(np.float64) - queries[q]
                assert abs(float((diff * diff).sum()) - float(d)) <= 1e-4 * max(1.0, float(d))
        assert np.all(np.diff(merged_d[q]) >= 0)
