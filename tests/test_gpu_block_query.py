"""Mode base: one thread block per query over the neighbourhood blocks
(csrc/bs_search_bq.cu).  Its rows must equal the reference's golden rows and
the oracle's distance bits, with 2 and 4 warps per query, on every distance
path (byte rows split over the block's threads, float rows folded one row per
thread), degrees 32 and 64, wide beams, host buffers used in place, and
batches larger than the resident blocks (blocks take several queries each,
and the next-block guesses carry over from one query to the next)."""
import numpy as np
import pytest

import beam_search_collab_b200 as B
import oracle as O
import golden_sets as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def indexes():
    out = {}
    for name in G.NAMES:
        g = G.load(name)
        out[name] = (g, B.Index.from_arrays(g.base, g.edges))
    yield out
    for _, ix in out.values():
        ix.close()


@pytest.mark.parametrize("warps", ["2", "4"])
@pytest.mark.parametrize("name", G.NAMES)
def test_block_per_query_matches_golden_rows_and_oracle_bits(indexes, name, warps, monkeypatch):
    g, ix = indexes[name]
    monkeypatch.setenv("BSEARCH_BQ_WARPS", warps)
    for m, K, topk in g.runs("base"):
        exp, _ = g.expected(m, K, topk)
        ids, dists, st = ix.search(g.queries, mode="base", K=K, topk_size=topk)
        assert st.warps_per_query == int(warps)
        assert st.block_bytes > 0
        same = (ids == exp).all(axis=1)
        assert same.all(), f"{name} K={K} T={topk}: {np.count_nonzero(~same)}/{len(same)} rows differ"
        ref = O.search(g.base, g.edges, g.queries, K=K, topk_size=topk, entry=g.entry)
        assert np.array_equal(dists.view(np.uint32), ref.dists.view(np.uint32))
        assert st.expansions == ref.stats.expansions
        assert st.error_flags == 0


@pytest.mark.parametrize("name", G.NAMES)
@pytest.mark.parametrize("topk", [16, 100, 512])
def test_block_per_query_equals_warp_per_query(indexes, name, topk):
    """Every beam width (one to sixteen registers of keys per lane) gives the
    warp kernel's rows, distance bits and expansion count."""
    g, ix = indexes[name]
    a = ix.search(g.queries, mode="base", K=10, topk_size=topk)
    b = ix.search(g.queries, mode="warp4", K=10, topk_size=topk)
    assert a[2].warps_per_query in (2, 4) and b[2].warps_per_query == 1
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    assert a[2].expansions == b[2].expansions
    assert a[2].error_flags == 0


def test_integer_and_sequential_paths_in_the_block_kernel(indexes, monkeypatch):
    """i128 (byte rows): integer queries split each row over the block's
    threads; fractional queries fall back to one thread per row in the
    reference's order; BSEARCH_FORCE_SEQ forces the sequential fold for all.
    All three equal the oracle bit for bit."""
    g, ix = indexes["i128"]
    q_frac = g.queries.copy()
    q_frac[1::2] += np.float32(0.5)
    for q in (g.queries, q_frac):
        ids, d, st = ix.search(q, mode="base", K=10, topk_size=64)
        ref = O.search(g.base, g.edges, q, K=10, topk_size=64, entry=g.entry)
        assert np.array_equal(ids, ref.ids)
        assert np.array_equal(d.view(np.uint32), ref.dists.view(np.uint32))
    monkeypatch.setenv("BSEARCH_FORCE_SEQ", "1")
    ids, d, st = ix.search(g.queries, mode="base", K=10, topk_size=64)
    assert st.integer_exact == 0
    ref = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry)
    assert np.array_equal(ids, ref.ids)
    assert np.array_equal(d.view(np.uint32), ref.dists.view(np.uint32))


@pytest.mark.parametrize("host", ["pageable", "pinned", "device"])
def test_block_per_query_large_batch_and_host_buffers(indexes, host, monkeypatch):
    """9,000 queries with 2 warps per query: more queries than resident
    blocks, so every block searches many queries in turn; each copy of a
    golden query returns its golden row, whichever buffer kind."""
    torch = pytest.importorskip("torch")
    g, ix = indexes["i128"]
    monkeypatch.setenv("BSEARCH_BQ_WARPS", "2")
    reps = -(-9000 // len(g.queries))
    q = np.ascontiguousarray(np.tile(g.queries, (reps, 1))[:9000])
    kw = dict(mode="base", K=10, topk_size=64)
    if host == "pageable":
        ids, _, st = ix.search(q, **kw)
    elif host == "pinned":
        hq = torch.from_numpy(q).pin_memory()
        hid = torch.full((len(q), 10), 7, dtype=torch.int32).pin_memory()
        hd = torch.zeros((len(q), 10), dtype=torch.float32).pin_memory()
        st = B.Stats()
        ix.search_raw(hq.data_ptr(), len(q), hid.data_ptr(), hd.data_ptr(), B.SearchParams(**kw), stats=st)
        ids = hid.numpy().view(np.uint32)
    else:
        ids_d, _, st = ix.search(torch.from_numpy(q).cuda(), **kw)
        torch.cuda.synchronize()
        ids = ids_d.cpu().numpy().view(np.uint32)
    assert st.error_flags == 0 and st.warps_per_query == 2
    exp, _ = g.expected("base", 10, 64)
    nq0 = len(g.queries)
    for r in range(reps):
        n = min(nq0, len(q) - r * nq0)
        assert np.array_equal(ids[r * nq0:r * nq0 + n], exp[:n])


def test_base_without_blocks_uses_the_warp_kernels(indexes, monkeypatch):
    """The gather layout (no neighbourhood blocks): base runs warp per query
    and gives the same rows."""
    g, ix = indexes["f48"]
    monkeypatch.setenv("BSEARCH_LAYOUT", "gather")
    gx = B.Index.from_arrays(g.base, g.edges)
    monkeypatch.delenv("BSEARCH_LAYOUT")
    try:
        a = gx.search(g.queries, mode="base", K=10, topk_size=64)
        b = ix.search(g.queries, mode="base", K=10, topk_size=64)
        assert a[2].warps_per_query == 1 and a[2].block_bytes == 0
        assert b[2].warps_per_query == 4
        assert np.array_equal(a[0], b[0])
        assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    finally:
        gx.close()


def test_block_per_query_wait_bound_reports_an_error(monkeypatch):
    """BSEARCH_WAIT_POLLS=0: every first wait gives up at once; warp 0 waits
    (bounded again) for the copies in flight, the block reports the error
    bit and leaves.  The call fails with BS_ERR_KERNEL, the index's error word
    holds the bit, and the next search returns the golden rows."""
    g = G.load("i128")
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        exp, _ = g.expected("base", 10, 64)
        monkeypatch.setenv("BSEARCH_WAIT_POLLS", "0")
        with pytest.raises(B.BSearchError) as e:
            ix.search(g.queries, mode="base", K=10, topk_size=64)
        assert e.value.status == 6 and "0x4" in str(e.value)
        assert ix.take_errors() == 4
        monkeypatch.delenv("BSEARCH_WAIT_POLLS")
        ids, _, st = ix.search(g.queries, mode="base", K=10, topk_size=64)
        assert st.error_flags == 0 and st.warps_per_query == 4
        assert (ids == exp).all()
        assert ix.take_errors() == 0
    finally:
        ix.close()
