"""GPU exact ground truth (bs_ground_truth) against a numpy brute force with
the same distances: squared differences in float32 summed left to right
(np.cumsum, a sequential sum: the reference's order,
include/cpu_search_base.hpp:29-37), ordered by (distance, id).  Ids must match
row for row and distances bit for bit, for float rows, byte rows with integer
queries (the integer-exact path) and byte rows with fractional queries."""
import numpy as np
import pytest

import beam_search_collab_b200 as B
import golden_sets as G

pytestmark = pytest.mark.gpu


def _brute(base, queries, k):
    ids = np.empty((len(queries), k), dtype=np.uint32)
    dists = np.empty((len(queries), k), dtype=np.float32)
    for i, q in enumerate(queries):
        t = (q[None, :] - base).astype(np.float32)
        d = np.cumsum(t * t, axis=1, dtype=np.float32)[:, -1]
        o = np.lexsort((np.arange(len(base)), d))[:k]
        ids[i], dists[i] = o, d[o]
    return ids, dists


@pytest.mark.parametrize("name,k", [("f48", 10), ("f48", 100), ("i128", 100), ("s96d64", 37)])
def test_ground_truth_matches_brute_force(name, k):
    g = G.load(name)
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        ids, d = ix.ground_truth(g.queries, k)
        ref_i, ref_d = _brute(g.base, g.queries, k)
        assert np.array_equal(ids, ref_i)
        assert np.array_equal(d.view(np.uint32), ref_d.view(np.uint32))
        if name == "i128":
            # the reference's own recall file agrees (ties by id)
            assert np.array_equal(ids[:, :10].astype(np.int64), g.gt[:, :10])
    finally:
        ix.close()


def test_ground_truth_fractional_queries_on_byte_rows_and_device_buffers():
    torch = pytest.importorskip("torch")
    g = G.load("i128")
    q = g.queries.copy()
    q[1::2] += np.float32(0.25)
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        ids, d = ix.ground_truth(torch.from_numpy(q).cuda(), 20)
        torch.cuda.synchronize()
        ref_i, ref_d = _brute(g.base, q, 20)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_i)
        assert np.array_equal(d.cpu().numpy().view(np.uint32), ref_d.view(np.uint32))
        with pytest.raises(B.BSearchError):
            ix.ground_truth(q, 300)
    finally:
        ix.close()
