"""GPU parity of the RaBitQ search over node blocks (one bulk copy of
[adjacency | codes | factors | own row] per expansion, a bitmap visited set per
warp cleared through a log of the ids each query set).

Every variant must return the reference CPU search's rows (the golden ids
recorded from CPURabitqSearch) and the oracle's distance bits, with the
oracle's expansion and estimate counts: the default block kernel, the gather
kernel (BSEARCH_LAYOUT=gather), the nibble-table estimator, the whole-bitmap
clearing path (a log too small for any query), and byte-valued rows (the
integer-exact own-row distance), with a codebook built by the GPU builder,
which is byte-identical to the reference build_rabitq.
"""
import os

import numpy as np
import pytest

import beam_search_collab_b200 as B
from beam_search_collab_b200 import datasets as ds
import golden_sets as G
import oracle as O

pytestmark = pytest.mark.gpu

CASES = [("f48", 10, 64), ("f48", 20, 200), ("s96d64", 10, 128)]


def _index(g, monkeypatch=None, **env):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    ix = B.Index.from_arrays(g.base, g.edges)
    ix.load_codebook(g.codebook_path)
    for k in env:
        monkeypatch.delenv(k)
    return ix


def _check(g, ix, K, topk, block=True, queries=None):
    q = g.queries if queries is None else queries
    ids, dists, st = ix.search(q, mode="rabitq", K=K, topk_size=topk)
    if queries is None:
        exp, _ = g.expected("rabitq", K, topk)
        same = (ids == exp).all(axis=1)
        assert same.all(), f"{g.name} K={K} T={topk}: {np.count_nonzero(~same)} rows differ"
    entry = ix.rabitq_entry()
    ref = O.search(g.base, g.edges, q, K=K, topk_size=topk, entry=entry, mode="rabitq", codebook=g.codebook())
    assert np.array_equal(ids, ref.ids)
    assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))
    assert st.expansions == ref.stats.expansions
    assert st.estimates == ref.stats.estimates
    assert st.error_flags == 0
    assert (st.block_bytes > 0) == block
    return ids


@pytest.mark.parametrize("name,K,topk", CASES)
def test_block_kernel_matches_reference_golden(name, K, topk):
    g = G.load(name)
    if not g.codebook_path:
        pytest.skip("codebook not available")
    ix = _index(g)
    try:
        _check(g, ix, K, topk)
        _check(g, ix, K, topk)            # the visited arena is clean after a call
        assert ix.take_errors() == 0
    finally:
        ix.close()


@pytest.mark.parametrize("name,K,topk", CASES)
def test_gather_kernel_and_estimator_variants_agree(name, K, topk, monkeypatch):
    g = G.load(name)
    if not g.codebook_path:
        pytest.skip("codebook not available")
    ix = _index(g, monkeypatch, BSEARCH_LAYOUT="gather")
    try:
        _check(g, ix, K, topk, block=False)
    finally:
        ix.close()
    ix = _index(g)
    try:
        monkeypatch.setenv("BSEARCH_RQ_ESTIMATOR", "lut")
        _check(g, ix, K, topk)
        monkeypatch.delenv("BSEARCH_RQ_ESTIMATOR")
    finally:
        ix.close()


def test_whole_bitmap_clearing_path(monkeypatch):
    """A log of 4 ids: every query overflows it and its end clears the whole
    bitmap.  Repeated batches (several queries per warp) must stay exact."""
    g = G.load("s96d64")
    if not g.codebook_path:
        pytest.skip("codebook not available")
    ix = _index(g, monkeypatch, BSEARCH_RQ_LOG_CAP="4")
    try:
        q = np.ascontiguousarray(np.tile(g.queries, (20, 1)))
        ids = _check(g, ix, 10, 128, queries=q)
        exp, _ = g.expected("rabitq", 10, 128)
        assert (ids[:len(exp)] == exp).all()
        assert (ids.reshape(20, len(exp), 10) == exp[None]).all()
    finally:
        ix.close()


def test_byte_rows_with_gpu_built_codebook(tmp_path):
    """i128 rows are integers in [0,255] (stored as bytes): the own-row
    distance is the integer-exact __dp4a path.  Codebook from the GPU builder
    (seed 12345), read back for the oracle; fractional queries take the
    sequential byte fold."""
    g = G.load("i128")
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        cb_path = os.path.join(tmp_path, "cb.bin")
        entry = ix.build_codebook(12345, cb_path)
        cb = ds.read_codebook(cb_path, g.base.shape[0], g.base.shape[1], g.edges.shape[1])
        q_frac = g.queries.copy()
        q_frac[1::2] += np.float32(0.5)
        for q in (g.queries, q_frac):
            for K, topk in ((10, 64), (10, 160)):
                ids, dists, st = ix.search(q, mode="rabitq", K=K, topk_size=topk)
                assert st.block_bytes > 0
                ref = O.search(g.base, g.edges, q, K=K, topk_size=topk, entry=entry, mode="rabitq", codebook=cb)
                assert np.array_equal(ids, ref.ids)
                assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))
                assert st.expansions == ref.stats.expansions and st.estimates == ref.stats.estimates
        assert ix.take_errors() == 0
    finally:
        ix.close()
