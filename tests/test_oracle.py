"""CPU: the oracle restatement (oracle/bs_oracle.c) is pinned against the
reference's own search classes and cpu_cli (golden fixtures), and its pieces
against independent numpy restatements and hand-computed answers."""
import numpy as np
import pytest

import oracle as O
import golden_sets as G


@pytest.mark.parametrize("name", G.NAMES)
def test_oracle_matches_reference_golden(name):
    g = G.load(name)
    cb = g.codebook()
    for mode, K, topk in g.runs():
        if mode == "rabitq" and cb is None:
            pytest.skip("codebook needs oracle/_ref/build_rabitq")
        exp, run = g.expected(mode, K, topk)
        r = O.search(g.base, g.edges, g.queries, K=K, topk_size=topk, entry=run["search_entry"],
                     mode=mode, codebook=cb)
        same = (r.ids == exp).all(axis=1)
        assert same.all(), f"{name} {mode} K={K} T={topk}: {np.count_nonzero(~same)} rows differ"


@pytest.mark.parametrize("name", G.NAMES)
def test_entry_point_matches_cpu_cli(name):
    g = G.load(name)
    assert O.entry_point(g.base) == g.entry


@pytest.mark.parametrize("name", G.NAMES)
def test_recall_definition_matches_cpu_cli(name):
    g = G.load(name)
    for mode, K, topk in g.runs():
        exp, run = g.expected(mode, K, topk)
        r = O.recall_cpu(exp, g.gt, K)
        # cpu_cli prints a float with 6 significant digits
        assert float(f"{np.float32(r):.6g}") == pytest.approx(run["cpu_cli_recall"], abs=1e-6)


def test_recall_gpu_definition_counts_duplicates_and_missing():
    gt = np.array([[1, 2, 3, 4]], dtype=np.int32)
    pred = np.array([[1, 1, 0xFFFFFFFF, 4, 9]], dtype=np.uint32)
    r, dups = O.recall_gpu(pred, gt, 5)
    assert dups == 1
    assert r == pytest.approx(2 / 4)              # divides by min(K, gt_k)
    assert O.recall_cpu(pred, gt, 5) == pytest.approx(2 / 5)


def _np_quantize(q, signs, pdim):
    """Independent float32 restatement of include/cpu_search_rabitq.hpp:34-57."""
    dim = q.shape[0]
    r = np.zeros(pdim, dtype=np.float32)
    r[:dim] = q.astype(np.float32) * signs[:dim].astype(np.float32)
    n = 1
    while n < pdim:
        for i in range(0, pdim, 2 * n):
            u = r[i:i + n].copy()
            v = r[i + n:i + 2 * n].copy()
            r[i:i + n] = u + v
            r[i + n:i + 2 * n] = u - v
        n <<= 1
    lo, hi = r.min(), r.max()
    w = np.float32(hi - lo) / np.float32(63)
    inv = np.float32(1) / w
    t = (r - lo) * inv + np.float32(0.5)
    qv = np.floor(t.astype(np.float64) + 0.5)   # lroundf (half away from zero) on positive values
    return qv.astype(np.uint8), lo, w


def test_quantizer_known_answer():
    # q=[1,2,3,4], signs 0.5: rotated [0.5,1,1.5,2] -> WHT [5,-1,-2,0],
    # low -2, w = 7/63, values lroundf((x+2)*9 + 0.5) = [64, 10, 1, 19]
    q, lo, w, s = O.quantize(np.array([1, 2, 3, 4], np.float32), np.full(4, 0.5, np.float32), 4)
    assert lo == -2.0
    assert w == pytest.approx(7 / 63)
    assert list(q) == [64, 10, 1, 19]
    assert s == 94


def test_quantizer_matches_numpy_restatement():
    rng = np.random.default_rng(7)
    for dim in (32, 48, 96, 128, 200):
        pdim = 1 << (dim - 1).bit_length()
        signs = (rng.integers(0, 2, pdim) * 2 - 1).astype(np.float32) / np.float32(np.sqrt(pdim))
        for _ in range(20):
            qv = rng.standard_normal(dim).astype(np.float32)
            q, lo, w, s = O.quantize(qv, signs, pdim)
            nq, nlo, nw = _np_quantize(qv, signs, pdim)
            assert lo == nlo and np.float32(w) == nw
            assert np.array_equal(q, nq)
            assert s == int(q.astype(np.int64).sum())
            assert q.min() >= 1 and q.max() <= 64


def test_raw_estimator_matches_popcount():
    rng = np.random.default_rng(3)
    for pdim in (32, 64, 128, 1024):
        quant = rng.integers(1, 65, pdim).astype(np.uint8)
        code = rng.integers(0, 2 ** 32, pdim // 32, dtype=np.uint64).astype(np.uint32)
        bits = np.unpackbits(code.view(np.uint8), bitorder="little")[:pdim]
        exp = int((bits.astype(np.int64) * quant).sum())
        assert O.lib().orc_rabitq_raw(quant.ctypes.data_as(O._u8p), code.ctypes.data_as(O._u32p), pdim) == exp


def test_bloom_without_false_positives_equals_exact():
    g = G.load("f48")
    a = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry, mode="base")
    b = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry, mode="bloom",
                 filter_bits=1 << 26, reset_interval=0)
    assert np.array_equal(a.ids, b.ids)


def test_bloom_small_filter_loses_some_recall():
    g = G.load("f48")
    a = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry, mode="base")
    b = O.search(g.base, g.edges, g.queries, K=10, topk_size=64, entry=g.entry, mode="bloom",
                 filter_bits=256, reset_interval=16)
    assert O.recall_cpu(b.ids, g.gt, 10) <= O.recall_cpu(a.ids, g.gt, 10)
    assert b.stats.distances <= a.stats.distances


def test_stats_counts():
    g = G.load("f48")
    r = O.search(g.base, g.edges, g.queries[:1], K=10, topk_size=64, entry=g.entry, mode="base")
    assert 1 <= r.stats.expansions <= 1024
    assert r.stats.distances >= r.stats.expansions


def test_max_iterations_zero_returns_entry_only():
    g = G.load("f48")
    r = O.search(g.base, g.edges, g.queries[:3], K=5, topk_size=64, entry=g.entry, max_iterations=0)
    assert (r.ids[:, 0] == g.entry).all()
    assert (r.ids[:, 1:] == 0xFFFFFFFF).all()
