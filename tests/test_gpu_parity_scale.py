"""Parity beyond the golden sets: a 60,000-row slice of the C2 distribution
(integer values 0..255: byte rows, the integer-exact path) and a 40,000-row
float set (the sequential fold), with graphs made by the GPU graph builder
(the reference build_graph's algorithm and settings) and the RaBitQ codebook
by the GPU codebook builder (the reference build_rabitq's), searched in every
kind of mode; rows, distance bits and counters against the CPU oracle (the
reference CPU search restated, itself pinned to the reference's own golden
rows)."""
import os
import tempfile

import numpy as np
import pytest

import beam_search_collab_b200 as B
import oracle as O
from beam_search_collab_b200 import datasets as ds

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c2_slice():
    s = ds.gen_c2(n=60_000, nq=300)
    ix = B.Index.from_vectors(s.base, 32)
    edges = ix.build_graph(beam_width=128, alpha=2.0, seed=1234)
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "codebook.bin")
        rq_entry = ix.build_codebook(12345, path)
        cb = ds.read_codebook(path, s.base.shape[0], s.base.shape[1], edges.shape[1])
    yield s, ix, edges, cb, rq_entry
    ix.close()


@pytest.fixture(scope="module")
def float_set():
    s = ds.gen_c1(n=40_000, nq=200, dim=64)
    ix = B.Index.from_vectors(s.base, 24)
    edges = ix.build_graph(beam_width=96, alpha=1.5, seed=7)
    yield s, ix, edges
    ix.close()


def _check(ids, dists, st, ref):
    same = (ids == ref.ids).all(axis=1)
    assert same.all(), f"{np.count_nonzero(~same)} of {len(same)} rows differ"
    assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))
    assert st.expansions == ref.stats.expansions
    assert st.error_flags == 0


def test_entry_point_on_the_slice(c2_slice):
    s, ix, _, _, _ = c2_slice
    assert ix.entry_point() == O.entry_point(s.base)


@pytest.mark.parametrize("mode,topk", [("warp4", 56), ("warp1", 128), ("base", 56), ("base", 200), ("warp8", 16)])
def test_exact_modes_on_the_slice(c2_slice, mode, topk):
    s, ix, edges, _, _ = c2_slice
    entry = ix.entry_point()
    ids, dists, st = ix.search(s.queries, mode=mode, K=10, topk_size=topk)
    assert st.integer_exact == 1
    _check(ids, dists, st, O.search(s.base, edges, s.queries, K=10, topk_size=topk, entry=entry))


def test_bloom_mode_on_the_slice(c2_slice):
    s, ix, edges, _, _ = c2_slice
    entry = ix.entry_point()
    ids, dists, st = ix.search(s.queries, mode="bwarp2", K=10, topk_size=64, filter_capacity=4096,
                               reset_interval=16)
    ref = O.search(s.base, edges, s.queries, K=10, topk_size=64, entry=entry, mode="bloom", filter_bits=4096,
                   reset_interval=16)
    assert np.array_equal(ids, ref.ids)
    assert st.distances == ref.stats.distances


@pytest.mark.parametrize("topk", [64, 192])
def test_rabitq_on_the_slice(c2_slice, topk):
    s, ix, edges, cb, rq_entry = c2_slice
    ids, dists, st = ix.search(s.queries, mode="rabitq", K=10, topk_size=topk)
    ref = O.search(s.base, edges, s.queries, K=10, topk_size=topk, entry=rq_entry, mode="rabitq", codebook=cb)
    _check(ids, dists, st, ref)
    assert st.estimates == ref.stats.estimates


@pytest.mark.parametrize("mode,topk", [("warp4", 64), ("base", 100)])
def test_float_rows_on_a_larger_set(float_set, mode, topk):
    s, ix, edges = float_set
    entry = ix.entry_point()
    assert entry == O.entry_point(s.base)
    ids, dists, st = ix.search(s.queries, mode=mode, K=20, topk_size=topk)
    _check(ids, dists, st, O.search(s.base, edges, s.queries, K=20, topk_size=topk, entry=entry))
