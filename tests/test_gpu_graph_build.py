"""GPU graph builder (bs_index_build_graph, bin/build_graph) against the
reference Vamana builder build_graph (src/build_graph.cpp).

The golden graph.bin files were written by the reference tool itself
(--beam-width 128 --alpha 2.0 --seed 1234); the GPU build must reproduce
them edge for edge, in every row's order.  Other parameters (degree, beam
width, alpha, seed, float and integer rows) are checked against the reference
tool run here (oracle/_ref/build_graph, the CPU binary built from the
reference's source).
"""
import os
import subprocess

import numpy as np
import pytest

import beam_search_collab_b200 as B
from beam_search_collab_b200 import datasets as ds
import golden_sets as G
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", G.NAMES)
def test_gpu_build_reproduces_reference_golden_graph(name):
    g = G.load(name)
    ix = B.Index.from_vectors(g.base, g.edges.shape[1])
    try:
        edges = ix.build_graph(beam_width=128, alpha=2.0, seed=1234)
        same = (edges == g.edges).all(axis=1)
        assert same.all(), f"{name}: {np.count_nonzero(~same)} of {len(same)} rows differ"
        # the built index searches like one loaded from the reference's file
        exp, _ = g.expected("base", *g.runs("base")[0][1:])
        ids, _, _ = ix.search(g.queries, mode="warp4", K=exp.shape[1], topk_size=g.runs("base")[0][2])
        assert (ids == exp).all()
    finally:
        ix.close()


def _reference_graph(base, tmp_path, degree, beam, alpha, seed):
    tool = O.ref_tool("build_graph")
    if tool is None:
        pytest.skip("oracle/_ref/build_graph not built")
    bp, gp = os.path.join(tmp_path, "b.fvecs"), os.path.join(tmp_path, "g.bin")
    ds.write_fvecs(bp, base)
    subprocess.run([tool, "--base", bp, "--graph", gp, "--degree", str(degree), "--beam-width", str(beam),
                    "--alpha", str(alpha), "--seed", str(seed)], check=True, capture_output=True)
    return ds.read_graph(gp)


@pytest.mark.parametrize("kind,n,dim,degree,beam,alpha,seed", [
    ("float", 1500, 40, 16, 64, 1.2, 7),
    ("int", 1800, 64, 24, 96, 2.0, 99),
    ("float", 900, 300, 32, 128, 1.5, 1),
    ("int_wide", 1200, 32, 40, 200, 2.0, 3),
])
def test_gpu_build_matches_reference_tool(tmp_path, kind, n, dim, degree, beam, alpha, seed):
    rng = np.random.default_rng(seed + n)
    if kind == "float":
        base = (rng.standard_normal((n, dim)) * 3).astype(np.float32)
    elif kind == "int":
        base = np.clip(np.rint(rng.normal(100, 40, size=(n, dim))), 0, 255).astype(np.float32)
    else:   # integers beyond the byte range
        base = np.rint(rng.normal(0, 300, size=(n, dim))).astype(np.float32)
    ref = _reference_graph(base, tmp_path, degree, beam, alpha, seed)
    ix = B.Index.from_vectors(base, degree)
    try:
        edges = ix.build_graph(beam_width=beam, alpha=alpha, seed=seed)
    finally:
        ix.close()
    same = (edges == ref).all(axis=1)
    assert same.all(), f"{np.count_nonzero(~same)} of {n} rows differ"


def test_build_graph_cli_writes_the_reference_file(tmp_path):
    g = G.load("f48")
    out = os.path.join(tmp_path, "graph.bin")
    cli = os.path.join(os.path.dirname(B.CLI_PATH), "build_graph")
    r = subprocess.run([cli, "--base", g.files["base"], "--graph", out, "--degree", "32", "--beam-width", "128",
                        "--alpha", "2.0", "--seed", "1234"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "Building Vamana graph: n=2000 dim=48 degree=32 beam_width=128 alpha=2 metric=l2" in r.stdout
    assert f"Wrote graph to {out}" in r.stdout
    with open(out, "rb") as a, open(g.files["graph"], "rb") as b:
        assert a.read() == b.read()
    r = subprocess.run([cli, "--base", g.files["base"], "--graph", out, "--metric", "cosine"],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "Unsupported metric: cosine" in r.stderr


def test_large_reverse_prunes_take_the_second_launch(tmp_path, monkeypatch):
    """A node that receives more reverse edges in one batch than the first
    reverse-prune launch holds (4,096 candidates; here 64 through
    BSEARCH_GB_REV_PRUNE_CAP) is pruned by a second launch with a larger
    candidate array: the graph stays identical, edge for edge, to the default
    build and to the reference tool's."""
    rng = np.random.default_rng(2024)
    centres = rng.normal(size=(20, 32)).astype(np.float32) * 4
    base = (centres[rng.integers(0, 20, 20000)] + rng.normal(size=(20000, 32))).astype(np.float32)
    ix = B.Index.from_vectors(base, 32)
    try:
        default = ix.build_graph(beam_width=64, alpha=1.2, seed=5)
    finally:
        ix.close()
    monkeypatch.setenv("BSEARCH_GB_REV_PRUNE_CAP", "64")
    ix = B.Index.from_vectors(base, 32)
    try:
        small = ix.build_graph(beam_width=64, alpha=1.2, seed=5)
    finally:
        ix.close()
    assert np.array_equal(small, default)
    ref = _reference_graph(base, tmp_path, 32, 64, 1.2, 5)
    assert np.array_equal(default, ref)
