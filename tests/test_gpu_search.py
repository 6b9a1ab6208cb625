"""GPU parity: the CUDA search (through the C ABI) against the oracle and the
reference's own golden results.  Integer ids must be identical row for row;
distances are compared bit for bit (both distance paths reproduce the
reference's fp32 sums exactly)."""
import os

import numpy as np
import pytest

import beam_search_collab_b200 as B
import oracle as O
import golden_sets as G

pytestmark = pytest.mark.gpu

EXACT_MODES = ("base", "warp1", "warp2", "warp4", "warp8")


@pytest.fixture(scope="module")
def indexes():
    out = {}
    for name in G.NAMES:
        g = G.load(name)
        ix = B.Index.from_arrays(g.base, g.edges)
        if g.codebook_path:
            ix.load_codebook(g.codebook_path)
        out[name] = (g, ix)
    yield out
    for _, ix in out.values():
        ix.close()


@pytest.mark.parametrize("name", G.NAMES)
def test_entry_point_matches_reference(indexes, name):
    g, ix = indexes[name]
    assert ix.entry_point() == g.entry


@pytest.mark.parametrize("name", G.NAMES)
@pytest.mark.parametrize("mode", EXACT_MODES)
def test_exact_modes_match_reference_golden(indexes, name, mode):
    g, ix = indexes[name]
    for m, K, topk in g.runs("base"):
        exp, run = g.expected(m, K, topk)
        ids, dists, st = ix.search(g.queries, mode=mode, K=K, topk_size=topk)
        same = (ids == exp).all(axis=1)
        assert same.all(), f"{name} {mode} K={K} T={topk}: {np.count_nonzero(~same)}/{len(same)} rows differ"
        ref = O.search(g.base, g.edges, g.queries, K=K, topk_size=topk, entry=g.entry)
        assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))
        assert st.expansions == ref.stats.expansions
        assert st.error_flags == 0


@pytest.mark.parametrize("name", G.NAMES)
def test_small_filter_forces_resets_and_stays_exact(indexes, name):
    g, ix = indexes[name]
    exp, _ = g.expected("base", 10, 64)
    ids, _, st = ix.search(g.queries, mode="warp2", K=10, topk_size=64, filter_capacity=32)
    assert (ids == exp).all()


@pytest.mark.parametrize("name", G.NAMES)
def test_distance_counter_matches_oracle_when_filter_never_resets(indexes, name, monkeypatch):
    """Gather layout with a visited table large enough never to reset: every
    pushed node is scored exactly once, as in the reference CPU search.  (The
    block layout sizes its table to the beam and may score a forgotten node
    again; its counter is then larger, its results the same.)"""
    g, _ = indexes[name]
    monkeypatch.setenv("BSEARCH_LAYOUT", "gather")
    ix = B.Index.from_arrays(g.base, g.edges)
    monkeypatch.delenv("BSEARCH_LAYOUT")
    try:
        ref = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry)
        _, _, st = ix.search(g.queries, mode="warp1", K=10, topk_size=64, filter_capacity=1 << 14)
        assert st.expansions == ref.stats.expansions
        assert st.distances == ref.stats.distances
    finally:
        ix.close()


@pytest.mark.parametrize("name", ["f48", "s96d64"])
def test_rabitq_matches_reference_golden(indexes, name):
    g, ix = indexes[name]
    if not g.codebook_path:
        pytest.skip("codebook not available")
    cb = g.codebook()
    for m, K, topk in g.runs("rabitq"):
        exp, run = g.expected(m, K, topk)
        ids, dists, st = ix.search(g.queries, mode="rabitq", K=K, topk_size=topk)
        same = (ids == exp).all(axis=1)
        assert same.all(), f"{name} rabitq K={K} T={topk}: {np.count_nonzero(~same)} rows differ"
        ref = O.search(g.base, g.edges, g.queries, K=K, topk_size=topk, entry=run["search_entry"],
                       mode="rabitq", codebook=cb)
        assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))
        assert st.expansions == ref.stats.expansions
        assert st.estimates == ref.stats.estimates


@pytest.mark.parametrize("cap", [64, 1024, 1 << 13])
def test_rabitq_visited_set_spill_stays_exact(indexes, cap):
    g, ix = indexes["s96d64"]
    if not g.codebook_path:
        pytest.skip("codebook not available")
    exp, _ = g.expected("rabitq", 10, 128)
    ids, _, st = ix.search(g.queries, mode="rabitq", K=10, topk_size=128, filter_capacity=cap)
    assert (ids == exp).all()
    assert st.error_flags == 0


@pytest.mark.parametrize("bits,reset", [(256, 16), (1024, 16), (4096, 32), (1 << 16, 0)])
@pytest.mark.parametrize("mode", ["bwarp1", "bwarp4"])
def test_bloom_modes_match_bloom_oracle(indexes, bits, reset, mode):
    g, ix = indexes["f48"]
    ids, dists, st = ix.search(g.queries, mode=mode, K=10, topk_size=64, filter_capacity=bits,
                               reset_interval=reset)
    ref = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry, mode="bloom",
                   filter_bits=bits, reset_interval=reset)
    assert np.array_equal(ids, ref.ids)
    assert st.distances == ref.stats.distances


def test_integer_path_and_sequential_path_agree(indexes, monkeypatch):
    g, ix = indexes["i128"]
    ids_t, d_t, st_t = ix.search(g.queries, mode="warp4", K=100, topk_size=256)
    assert st_t.integer_exact == 1
    monkeypatch.setenv("BSEARCH_FORCE_SEQ", "1")
    ids_s, d_s, st_s = ix.search(g.queries, mode="warp4", K=100, topk_size=256)
    assert st_s.integer_exact == 0
    assert np.array_equal(ids_t, ids_s)
    assert np.array_equal(d_t.view(np.uint32), d_s.view(np.uint32))


@pytest.mark.parametrize("name", G.NAMES)
def test_gather_layout_and_block_layout_agree(indexes, name, monkeypatch):
    """The default index keeps neighbourhood blocks (one bulk copy per
    expansion); BSEARCH_LAYOUT=gather builds the plain layout.  Both run the
    same search and must agree bit for bit, in exact and Bloom modes."""
    g, ix_blocks = indexes[name]
    monkeypatch.setenv("BSEARCH_LAYOUT", "gather")
    ix_gather = B.Index.from_arrays(g.base, g.edges)
    monkeypatch.delenv("BSEARCH_LAYOUT")
    try:
        for mode, K, topk in (("warp4", 10, 64), ("base", 50, 160), ("bwarp2", 10, 64)):
            a = ix_blocks.search(g.queries, mode=mode, K=K, topk_size=topk)
            b = ix_gather.search(g.queries, mode=mode, K=K, topk_size=topk)
            assert np.array_equal(a[0], b[0])
            assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
            assert a[2].expansions == b[2].expansions
            assert a[2].distances >= b[2].distances   # the block layout may re-score forgotten nodes
    finally:
        ix_gather.close()


def test_byte_storage_and_float_storage_agree(indexes, monkeypatch):
    """i128 values are integers in [0,255]: the index keeps an exact u8 copy.
    Forcing f32 rows must give the same ids and distance bits, for integer
    queries, out-of-byte-range integer queries and fractional queries."""
    g, ix_u8 = indexes["i128"]
    monkeypatch.setenv("BSEARCH_STORAGE", "f32")
    ix_f32 = B.Index.from_arrays(g.base, g.edges)
    monkeypatch.delenv("BSEARCH_STORAGE")
    try:
        q_big = g.queries.copy()
        q_big[::3, 5] = 300.0            # integer, outside the byte range
        q_frac = g.queries.copy()
        q_frac[1::2] += np.float32(0.5)
        for q in (g.queries, q_big, q_frac):
            a = ix_u8.search(q, mode="warp4", K=10, topk_size=64)
            b = ix_f32.search(q, mode="warp4", K=10, topk_size=64)
            ref = O.search(g.base, g.edges, q, K=10, topk_size=64, entry=g.entry)
            assert np.array_equal(a[0], ref.ids) and np.array_equal(b[0], ref.ids)
            assert np.array_equal(a[1].view(np.uint32), ref.dists.view(np.uint32))
            assert np.array_equal(b[1].view(np.uint32), ref.dists.view(np.uint32))
    finally:
        ix_f32.close()


def test_fractional_queries_leave_the_integer_path_and_stay_exact(indexes):
    g, ix = indexes["i128"]
    q = g.queries.copy()
    q[::2] += np.float32(0.25)          # half of the queries are not integers
    ids, dists, st = ix.search(q, mode="warp2", K=10, topk_size=64)
    assert st.integer_exact == 0
    ref = O.search(g.base, g.edges, q, K=10, topk_size=64, entry=g.entry)
    assert np.array_equal(ids, ref.ids)
    assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))


def test_device_and_host_buffers_agree(indexes):
    torch = pytest.importorskip("torch")
    g, ix = indexes["f48"]
    ids_h, d_h, _ = ix.search(g.queries, mode="warp4", K=10, topk_size=64)
    qd = torch.from_numpy(g.queries).cuda()
    ids_d, d_d, _ = ix.search(qd, mode="warp4", K=10, topk_size=64)
    torch.cuda.synchronize()
    assert np.array_equal(ids_d.cpu().numpy().view(np.uint32), ids_h)
    assert np.array_equal(d_d.cpu().numpy(), d_h)


@pytest.mark.parametrize("name,mode,topk", [("i128", "warp4", 64), ("f48", "bwarp2", 64), ("s96d64", "rabitq", 128)])
@pytest.mark.parametrize("host", ["pageable", "pinned"])
def test_large_host_batch_matches_device_batch_and_golden_rows(indexes, name, mode, topk, host):
    """Host buffers reach the kernels two ways: pageable memory through device
    staging and whole-batch copies, page-locked memory in place (each warp
    reads its query over the bus and writes its result row back).  Both must
    give the device-buffer result row for row.  The batch repeats the golden
    queries, so each copy of a query returns the same row, the first the
    golden one."""
    torch = pytest.importorskip("torch")
    g, ix = indexes[name]
    if mode == "rabitq" and not g.codebook_path:
        pytest.skip("codebook not available")
    reps = -(-9000 // len(g.queries))
    q = np.ascontiguousarray(np.tile(g.queries, (reps, 1))[:9000])
    kw = dict(mode=mode, K=10, topk_size=topk)
    if host == "pageable":
        ids_h, d_h, st_h = ix.search(q, **kw)
    else:
        hq = torch.from_numpy(q).pin_memory()
        hid = torch.full((len(q), 10), 7, dtype=torch.int32).pin_memory()
        hd = torch.zeros((len(q), 10), dtype=torch.float32).pin_memory()
        st_h = B.Stats()
        ix.search_raw(hq.data_ptr(), len(q), hid.data_ptr(), hd.data_ptr(), B.SearchParams(**kw), stats=st_h)
        ids_h, d_h = hid.numpy().view(np.uint32), hd.numpy()
    ids_d, d_d, st_d = ix.search(torch.from_numpy(q).cuda(), **kw)
    torch.cuda.synchronize()
    assert np.array_equal(ids_d.cpu().numpy().view(np.uint32), ids_h)
    assert np.array_equal(d_d.cpu().numpy().view(np.uint32), d_h.view(np.uint32))
    assert st_h.expansions == st_d.expansions and st_h.distances == st_d.distances
    assert st_h.error_flags == 0
    nq0 = len(g.queries)
    for r in range(1, reps):
        n = min(nq0, len(q) - r * nq0)
        assert np.array_equal(ids_h[r * nq0:r * nq0 + n], ids_h[:n])
    if mode != "bwarp2":
        exp, _ = g.expected("rabitq" if mode == "rabitq" else "base", 10, topk)
        assert (ids_h[:nq0] == exp).all()


@pytest.mark.parametrize("deg", [24, 48])
def test_wide_rows_stream_through_the_chunk_ring_and_stay_exact(monkeypatch, deg):
    """Float rows wider than 1 KB in the gather layout are folded chunk by
    chunk through a shared-memory ring; every distance must still equal the
    reference's sequential order bit for bit (dim 300: a partial last chunk;
    degree 48: two groups of rows per expansion)."""
    rng = np.random.default_rng(5 + deg)
    n, dim = 4000, 300
    base = (rng.standard_normal((n, dim)) * 2).astype(np.float32)
    q = (rng.standard_normal((40, dim)) * 2).astype(np.float32)
    edges = rng.integers(0, n, size=(n, deg), dtype=np.uint32)
    monkeypatch.setenv("BSEARCH_LAYOUT", "gather")
    ix = B.Index.from_arrays(base, edges)
    monkeypatch.delenv("BSEARCH_LAYOUT")
    try:
        entry = O.entry_point(base)
        for mode, K, topk in (("warp4", 10, 64), ("base", 32, 128)):
            ids, d, st = ix.search(q, mode=mode, K=K, topk_size=topk)
            ref = O.search(base, edges, q, K=K, topk_size=topk, entry=entry)
            assert np.array_equal(ids, ref.ids)
            assert np.array_equal(d.view(np.uint32), ref.dists.view(np.uint32))
            assert st.distances == ref.stats.distances or st.distances > ref.stats.distances
    finally:
        ix.close()


def test_k_larger_than_beam_pads_with_no_node(indexes):
    g, ix = indexes["f48"]
    ids, dists, _ = ix.search(g.queries[:8], mode="warp1", K=80, topk_size=32)
    ref = O.search(g.base, g.edges, g.queries[:8], K=80, topk_size=32, entry=g.entry)
    assert np.array_equal(ids, ref.ids)
    assert (ids[:, 32:] == B.NO_NODE).all()
    assert (dists[:, 32:] == np.finfo(np.float32).max).all()


def test_max_iterations_zero_and_empty_batch(indexes):
    g, ix = indexes["f48"]
    ids, _, st = ix.search(g.queries[:4], mode="warp1", K=3, topk_size=64, max_iterations=0)
    assert (ids[:, 0] == g.entry).all() and (ids[:, 1:] == B.NO_NODE).all()
    assert st.expansions == 0
    ids, _, st = ix.search(g.queries[:0], mode="warp1", K=3, topk_size=64)
    assert ids.shape == (0, 3)


def test_explicit_entry_point(indexes):
    g, ix = indexes["f48"]
    ids, _, st = ix.search(g.queries[:16], mode="warp4", K=10, topk_size=64, entry_point=5)
    ref = O.search(g.base, g.edges, g.queries[:16], K=10, topk_size=64, entry=5)
    assert st.entry_point == 5
    assert np.array_equal(ids, ref.ids)


def test_graph_with_padding_duplicates_and_missing_neighbours():
    g = G.load("f48")
    edges = g.edges.copy()
    edges[:, 20:24] = 0                  # build_graph pads short lists with node 0
    edges[::3, 30] = 0xFFFFFFFF          # empty slot
    edges[::5, 31] = g.base.shape[0] + 7  # out-of-range id
    ix = B.Index.from_arrays(g.base, edges)
    try:
        for mode in ("warp1", "bwarp2"):
            ids, dists, _ = ix.search(g.queries, mode=mode, K=10, topk_size=64)
            om = "base" if mode == "warp1" else "bloom"
            ref = O.search(g.base, edges, g.queries, K=10, topk_size=64, entry=g.entry, mode=om)
            assert np.array_equal(ids, ref.ids)
            for row in ids:
                v = row[row != B.NO_NODE]
                assert len(set(v.tolist())) == len(v)
    finally:
        ix.close()


def test_invalid_configurations_are_rejected(indexes):
    g, ix = indexes["f48"]
    with pytest.raises(B.BSearchError) as e:
        ix.search(g.queries[:2], mode="warp3", K=10, topk_size=64)
    assert "Unknown mode: warp3" in str(e.value)
    with pytest.raises(B.BSearchError) as e:
        ix.search(g.queries[:2], mode="warp1", K=10, topk_size=1024)
    assert e.value.status == 2
    with pytest.raises(B.BSearchError):
        ix.search(g.queries[:2], mode="warp1", K=10, topk_size=64, entry_point=10 ** 6)
    gi, ixi = indexes["i128"]
    with pytest.raises(B.BSearchError) as e:
        ixi.search(gi.queries[:2], mode="rabitq", K=10, topk_size=64)
    assert "codebook" in str(e.value)
