"""Index sharding on the GPU: the shard merge kernel (bs_merge_shards) against
the numpy restatement, on shards searched by bs_search (each shard's lists
checked against the oracle first); and, with two GPUs, the full
ShardedIndex path over NCCL."""
import os
import socket

import numpy as np
import pytest
import torch

import beam_search_collab_b200 as B
import sharded_ref as R

pytestmark = pytest.mark.gpu


def _shard_results(shards, K, topk):
    base, queries = R.dataset()
    qd = torch.from_numpy(queries).cuda()
    ids_l, d_l, offs = [], [], []
    for s in range(shards):
        lo, vecs, edges = R.shard(base, shards, s)
        ix = B.Index.from_arrays(vecs, edges)
        try:
            ids, d, st = ix.search(qd, mode="warp4", K=K, topk_size=topk)
            torch.cuda.synchronize()
        finally:
            ix.close()
        ref_i, ref_d = R.oracle_shard_search(vecs, edges, queries, K, topk)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_i)
        assert np.array_equal(d.cpu().numpy().view(np.uint32), ref_d.view(np.uint32))
        ids_l.append(ids)
        d_l.append(d)
        offs.append(lo)
    return torch.stack(ids_l).contiguous(), torch.stack(d_l).contiguous(), offs


@pytest.mark.parametrize("shards,K,topk,K_out", [(2, 10, 32, 10), (3, 10, 32, 30), (4, 40, 32, 40), (8, 5, 16, 17)])
def test_merge_of_shard_results_matches_reference_merge(shards, K, topk, K_out):
    ids_all, d_all, offs = _shard_results(shards, K, topk)
    gi, gd = B.merge_shards(d_all, ids_all, offs, K_out)
    torch.cuda.synchronize()
    ref_i, ref_d = R.merge_ref(ids_all.cpu().numpy().view(np.uint32), d_all.cpu().numpy(), offs, K_out)
    assert np.array_equal(gi.cpu().numpy().view(np.uint32), ref_i)
    assert np.array_equal(gd.cpu().numpy().view(np.uint32), ref_d.view(np.uint32))


def test_merge_rejects_bad_arguments():
    ids_all, d_all, offs = _shard_results(2, 10, 32)
    with pytest.raises(B.BSearchError):
        B.merge_shards(d_all, ids_all, offs, 21)          # K_out > shards * K
    with pytest.raises(B.BSearchError):
        B.merge_shards(d_all.cpu(), ids_all.cpu(), offs, 10)   # host pointers


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    from beam_search_collab_b200.sharded import ShardedIndex
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        base, queries = R.dataset()
        lo, vecs, edges = R.shard(base, world, rank)
        sx = ShardedIndex.from_arrays(vecs, edges, device=rank)
        gi, gd = sx.search(torch.from_numpy(queries).cuda(rank), mode="warp4", K=10, topk_size=32)
        torch.cuda.synchronize()
        out[rank] = (list(sx.offsets), gi.cpu().numpy().view(np.uint32).copy(), gd.cpu().numpy().copy())
        sx.index.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_index_over_nccl_matches_reference_merge():
    import torch.multiprocessing as mp
    world = 2
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.start_processes(_nccl_rank, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
        res = dict(out)
    base, queries = R.dataset()
    ids_l, d_l, offs = [], [], []
    for s in range(world):
        lo, vecs, edges = R.shard(base, world, s)
        i, d = R.oracle_shard_search(vecs, edges, queries, 10, 32)
        ids_l.append(i)
        d_l.append(d)
        offs.append(lo)
    ref_i, ref_d = R.merge_ref(np.stack(ids_l), np.stack(d_l), offs, 10)
    for r in range(world):
        got_off, gi, gd = res[r]
        assert got_off == offs
        assert np.array_equal(gi, ref_i)
        assert np.array_equal(gd.view(np.uint32), ref_d.view(np.uint32))
