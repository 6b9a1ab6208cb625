"""GPU: bs_search_no_alloc, the search entry point for callers that cannot
allocate device memory while they run (a process that reserves the GPU's
memory up front and forbids later allocations, or a loop that cannot accept an
allocation's blocking or failure).  Its kernel scratch lives in a fixed
file-scope device array instead of per-call allocations.

Checked through the C ABI against the regular entry point bs_search, on two
calls in a row (the fixed array keeps the previous call's contents, so the
second call shows that everything that must start at zero is cleared), with
the same exact-equality tolerance as the other parity tests.  This file is
named so that pytest collects it last; it also runs alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import beam_search_collab_b200 as B
import golden_sets as G

pytestmark = pytest.mark.gpu


def _call_no_alloc(ix, params, q, ids, dists):
    c = params._c()
    return B.lib().bs_search_no_alloc(ix._h, ctypes.byref(c), ctypes.c_void_p(q.data_ptr()), q.shape[0],
                                      ctypes.c_void_p(ids.data_ptr()),
                                      ctypes.c_void_p(dists.data_ptr() if dists is not None else None), None)


@pytest.mark.parametrize("name,mode,K,topk", [("f48", "warp4", 10, 64), ("i128", "warp2", 100, 256),
                                              ("s96d64", "bwarp1", 10, 64), ("f48", "base", 16, 96)])
def test_no_alloc_matches_bs_search_on_two_calls(name, mode, K, topk):
    torch = pytest.importorskip("torch")
    g = G.load(name)
    ix = B.Index.from_arrays(g.base, g.edges)   # fresh index: the first call computes the entry point
    try:
        q = torch.from_numpy(g.queries).cuda()
        nq = q.shape[0]
        params = B.SearchParams(mode=mode, K=K, topk_size=topk)
        outs = []
        for _ in range(2):
            ids = torch.full((nq, K), -7, dtype=torch.int32, device="cuda")
            dists = torch.full((nq, K), float("nan"), dtype=torch.float32, device="cuda")
            rc = _call_no_alloc(ix, params, q, ids, dists)
            assert rc == 0, B.lib().bs_last_error().decode()
            torch.cuda.synchronize()
            outs.append((ids, dists))
            # the first call computed the entry point in the fixed array: it
            # must be the reference's (cpu_cli's printed entry)
            assert ix.entry_point() == g.entry
        assert ix.take_errors() == 0                  # no kernel error bits
        ref_ids, ref_d, st = ix.search(q, params)     # the regular entry point
        torch.cuda.synchronize()
        assert st.error_flags == 0
        for ids, dists in outs:
            assert torch.equal(ids, ref_ids)
            assert np.array_equal(dists.cpu().numpy().view(np.uint32), ref_d.cpu().numpy().view(np.uint32))
    finally:
        ix.close()


def test_no_alloc_rejects_what_needs_allocation():
    torch = pytest.importorskip("torch")
    g = G.load("f48")
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        q = torch.from_numpy(g.queries).cuda()
        ids = torch.empty((q.shape[0], 10), dtype=torch.int32, device="cuda")
        rq = B.SearchParams(mode="rabitq", K=10, topk_size=64)
        assert _call_no_alloc(ix, rq, q, ids, None) == 2
        assert "fixed scratch" in B.lib().bs_last_error().decode()
        host_q = torch.from_numpy(g.queries)
        assert _call_no_alloc(ix, B.SearchParams(mode="warp1", K=10, topk_size=64), host_q, ids, None) == 1
        assert "device pointers only" in B.lib().bs_last_error().decode()
    finally:
        ix.close()
