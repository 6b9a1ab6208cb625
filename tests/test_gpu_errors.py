"""GPU: how kernel-side errors reach the caller, and buffers on the wrong GPU.

A block copy's wait is bounded: when it gives up, the warp waits (bounded
again) for the copy in flight, sets an error bit and leaves its query.  The
test drives that path without any fault: BSEARCH_WAIT_POLLS=0 makes the first
wait of every expansion give up at once, the copy still lands, and the
library must report BS_ERR_KERNEL (synchronous calls) or leave the bit in the
index's error word (asynchronous calls, read by bs_index_take_errors).  The
context stays usable: the next search returns the golden rows.
"""
import numpy as np
import pytest

import beam_search_collab_b200 as B
import golden_sets as G

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 4


@pytest.fixture
def f48():
    g = G.load("f48")
    ix = B.Index.from_arrays(g.base, g.edges)
    yield g, ix
    ix.close()


def test_wait_timeout_is_reported_and_the_index_stays_usable(f48, monkeypatch):
    torch = pytest.importorskip("torch")
    g, ix = f48
    exp, _ = g.expected("base", 10, 64)
    _, _, st = ix.search(g.queries, mode="warp4", K=10, topk_size=64)
    assert st.block_bytes > 0, "the golden index should use neighbourhood blocks"
    assert ix.take_errors() == 0

    monkeypatch.setenv("BSEARCH_WAIT_POLLS", "0")
    with pytest.raises(B.BSearchError) as e:
        ix.search(g.queries, mode="warp4", K=10, topk_size=64)       # stats: synchronous
    assert e.value.status == 6
    assert "0x4" in str(e.value)
    assert ix.take_errors() == WAIT_TIMEOUT                            # the word saw it too
    assert ix.take_errors() == 0                                       # and was cleared

    q = torch.from_numpy(g.queries).cuda()
    ids = torch.empty((q.shape[0], 10), dtype=torch.int32, device="cuda")
    ix.search_raw(q.data_ptr(), q.shape[0], ids.data_ptr(), 0, B.SearchParams(mode="warp4", K=10, topk_size=64))
    assert ix.take_errors() == WAIT_TIMEOUT                            # asynchronous call

    monkeypatch.delenv("BSEARCH_WAIT_POLLS")
    ids2, _, st2 = ix.search(g.queries, mode="warp4", K=10, topk_size=64)
    assert st2.error_flags == 0
    assert (ids2 == exp).all()
    assert ix.take_errors() == 0


def test_buffers_on_another_gpu_are_refused():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    g = G.load("f48")
    ix = B.Index.from_arrays(g.base, g.edges, device=0)
    try:
        q1 = torch.from_numpy(g.queries).to("cuda:1")
        ids1 = torch.full((q1.shape[0], 10), -3, dtype=torch.int32, device="cuda:1")
        with pytest.raises(B.BSearchError) as e:
            ix.search_raw(q1.data_ptr(), q1.shape[0], ids1.data_ptr(), 0, B.SearchParams(mode="warp4", K=10, topk_size=64))
        assert e.value.status == 1 and "another GPU" in str(e.value)
        torch.cuda.synchronize("cuda:1")
        assert (ids1 == -3).all()                                      # nothing was launched
    finally:
        ix.close()
