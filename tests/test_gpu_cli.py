"""GPU: the drop-in CLI bin/gpu_cli end to end on the golden sets.

The reference gpu_cli reads one JSON object on stdin and prints
"data: N points, dim=D, degree=G, queries=Q, entry=E", "search: mode=M K=K",
"  time: X ms  qps: Y" and "recall@K: R" (reference src/gpu_cli.cu:398-401,
416, 163-164, 483), its recall computed by the GPU-side definition
(src/gpu_cli.cu:28-51).  The CLI here must print the same lines, and the ids
it returns (written through its optional "results" key) must be the
reference's own rows; the printed recall must then be the reference
definition applied to those rows.
"""
import os
import re

import numpy as np
import pytest

import beam_search_collab_b200 as B
import golden_sets as G
import oracle as O

pytestmark = pytest.mark.gpu

CASES = [("f48", "warp4", 10, 64), ("i128", "base", 100, 256), ("f48", "bwarp2", 10, 64),
         ("f48", "rabitq", 10, 64), ("s96d64", "rabitq", 10, 128), ("s96d64", "warp8", 50, 160)]


def _expected(g, mode, K, topk):
    if mode == "bwarp2":
        return O.search(g.base, g.edges, g.queries, K=K, topk_size=topk, entry=g.entry, mode="bloom",
                        filter_bits=1024, reset_interval=16).ids
    if mode == "rabitq":
        return g.expected("rabitq", K, topk)[0]
    try:
        return g.expected("base", K, topk)[0]
    except KeyError:
        return O.search(g.base, g.edges, g.queries, K=K, topk_size=topk, entry=g.entry).ids


@pytest.mark.parametrize("name,mode,K,topk", CASES)
def test_cli_lines_ids_and_recall(tmp_path, name, mode, K, topk):
    g = G.load(name)
    if mode == "rabitq" and not g.codebook_path:
        pytest.skip("codebook not available")
    out = os.path.join(tmp_path, "ids.u32")
    data = {"graph": g.files["graph"], "base": g.files["base"], "query": g.files["query"], "gt": g.files["gt"],
            "results": out}
    if mode == "rabitq":
        data["codebook"] = g.codebook_path
    cfg = {"data": data, "search": {"mode": mode, "K": K, "topk_size": topk, "filter_capacity": 1024,
                                    "max_iterations": 1024, "reset_interval": 16}}
    r = B.run_cli(cfg, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    n, dim, deg = g.base.shape[0], g.base.shape[1], g.edges.shape[1]
    data_line = [ln for ln in lines if ln.startswith("data: ")]
    assert len(data_line) == 1
    m = re.fullmatch(r"data: (\d+) points, dim=(\d+), degree=(\d+), queries=(\d+), entry=(\d+)", data_line[0])
    assert m and tuple(int(x) for x in m.groups()) == (n, dim, deg, len(g.queries), g.entry)
    assert f"search: mode={mode} K={K}" in lines
    assert any(re.fullmatch(r"  time: [0-9.e+-]+ ms  qps: [0-9.e+-]+", ln) for ln in lines)

    ids = np.fromfile(out, dtype=np.uint32).reshape(len(g.queries), K)
    exp = _expected(g, mode, K, topk)
    assert np.array_equal(ids, exp)

    rec = [ln for ln in lines if ln.startswith(f"recall@{K}: ")]
    assert len(rec) == 1
    want, _ = O.recall_gpu(exp, g.gt, K)
    assert abs(float(rec[0].split(": ")[1]) - want) < 2e-5


def test_cli_rejects_like_the_reference(tmp_path):
    g = G.load("f48")
    data = {"graph": g.files["graph"], "base": g.files["base"], "query": g.files["query"], "gt": g.files["gt"]}
    r = B.run_cli({"data": data, "search": {"mode": "warp3", "K": 10, "topk_size": 64}})
    assert r.returncode == 1 and "Unknown mode: warp3" in r.stderr
    r = B.run_cli({"data": data, "search": {"mode": "warp1", "K": 100, "topk_size": 64}})
    assert r.returncode == 1 and "topk_size (64) must be >= K (100)" in r.stderr
    r = B.run_cli({"data": data, "search": {"mode": "rabitq", "K": 10, "topk_size": 64}})
    assert r.returncode == 1 and "requires \"codebook\"" in r.stderr
