"""CPU checks of the benchmark's host-side logic (no GPU): the query split of
the multi-GPU modes, the recall definition, the parity summary against the
reference search's rows, and the parsing of a gpu_cli-style report (a stub
CLI stands in for the binaries)."""
import os
import stat
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_query_share_covers_the_batch(world):
    # weak: every rank its own NQ_PER_GPU queries, disjoint and contiguous
    weak = [bench.query_share(r, world, False) for r in range(world)]
    assert weak[0][0] == 0 and all(b - a == bench.NQ_PER_GPU for a, b in weak)
    assert all(weak[i][1] == weak[i + 1][0] for i in range(world - 1))
    # strong: the one batch split into contiguous ranges that cover it once
    strong = [bench.query_share(r, world, True) for r in range(world)]
    assert strong[0][0] == 0 and strong[-1][1] == bench.NQ_PER_GPU
    assert all(strong[i][1] == strong[i + 1][0] for i in range(world - 1))
    sizes = [b - a for a, b in strong]
    assert max(sizes) - min(sizes) <= 1


def test_recall_counts_ids_found_in_the_truth_rows():
    gt = np.array([[1, 2, 3], [4, 5, 6]])
    pred = np.array([[3, 2, 9], [6, 5, 4]])
    assert bench.recall_at_k(pred, gt, k=3) == pytest.approx(5 / 6)
    # recall@k compares the first k of each row with the first k of the truth
    assert bench.recall_at_k(pred, gt, k=1) == 0.0
    assert bench.recall_at_k(np.array([[1, 7, 7], [9, 4, 4]]), gt, k=2) == pytest.approx(1 / 2)


def test_parity_summary_against_reference_rows():
    rng = np.random.default_rng(0)
    base = rng.integers(0, 10, size=(50, 4)).astype(np.float32)
    queries = rng.integers(0, 10, size=(3, 4)).astype(np.float32)
    d = ((queries[:, None, :].astype(np.float64) - base[None]) ** 2).sum(-1)
    order = np.argsort(d, axis=1, kind="stable")[:, :10]
    ref = order.astype(np.uint32)
    ours = ref.copy()
    ours[2, 9] = ref[2, 8]          # one id differs in one row
    dists = np.take_along_axis(d, order, 1).astype(np.float32)
    out = bench.parity_vs_reference(ref, ours, dists, base, queries, order.astype(np.int64))
    assert out["queries"] == 3
    assert out["identical_rows"] == pytest.approx(2 / 3, abs=1e-6)
    assert out["ids_match_frac"] == pytest.approx(29 / 30, abs=1e-6)
    assert out["max_rel_dist_err"] == 0.0
    assert out["recall@10_reference"] == 1.0


def test_cli_report_is_parsed(tmp_path):
    cli = tmp_path / "fake_cli"
    cli.write_text("#!/bin/sh\ncat > /dev/null\n"
                   "echo '  time: 0.625 ms  qps: 16000000.0'\n"
                   "echo 'recall@10: 0.9533'\n")
    cli.chmod(cli.stat().st_mode | stat.S_IEXEC)
    r = bench.run_cli(str(cli), {"graph": "g", "base": "b", "query": "q", "gt": "t"}, "warp4", 56, k=10)
    assert r["rc"] == 0 and r["ms"] == 0.625 and r["qps"] == 16000000.0 and r["recall@10"] == 0.9533
    assert r["mode"] == "warp4" and r["topk_size"] == 56


def test_cli_failure_keeps_its_last_error_line(tmp_path):
    cli = tmp_path / "bad_cli"
    cli.write_text("#!/bin/sh\ncat > /dev/null\necho 'first' >&2\necho 'Unknown mode: x' >&2\nexit 1\n")
    cli.chmod(cli.stat().st_mode | stat.S_IEXEC)
    r = bench.run_cli(str(cli), {}, "x", 8, k=10)
    assert r["rc"] == 1 and r["qps"] is None and r["stderr"] == "Unknown mode: x"
