"""GPU parity of the codebook builder (bs_index_build_codebook, bin/build_rabitq)
against the reference build_rabitq: the file it writes must be byte-identical
to the reference tool's (pinned by the sha256 the golden fixtures recorded
from it, and by the reference tool itself where oracle/_ref holds it), for
f32 and byte row storage, graphs with missing neighbours included; and a
search on the built codebook must return the golden rabitq results."""
import hashlib
import os
import subprocess

import numpy as np
import pytest

import beam_search_collab_b200 as B
from beam_search_collab_b200 import datasets as ds
import golden_sets as G
import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "beam_search_collab_b200", "bin", "build_rabitq")


def _sha(path):
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


def _ref_codebook(base_path, graph_path, out, seed=12345):
    tool = O.ref_tool("build_rabitq")
    if tool is None:
        pytest.skip("reference build_rabitq not built")
    subprocess.run([tool, "-base", base_path, "-graph", graph_path, "-out", out, "-seed", str(seed)],
                   check=True, capture_output=True)
    return out


@pytest.mark.parametrize("name", ["f48", "s96d64"])
def test_codebook_file_matches_reference_hash(name, tmp_path):
    g = G.load(name)
    out = str(tmp_path / "cb.bin")
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        entry = ix.build_codebook(12345, out)
        assert ix.rabitq_entry() == entry
    finally:
        ix.close()
    assert _sha(out) == g.meta["codebook_sha256"]


@pytest.mark.parametrize("name", ["f48", "s96d64"])
def test_search_on_built_codebook_matches_golden(name):
    g = G.load(name)
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        ix.build_codebook(12345)
        for m, K, topk in g.runs("rabitq"):
            exp, run = g.expected(m, K, topk)
            ids, _, st = ix.search(g.queries, mode="rabitq", K=K, topk_size=topk)
            assert ix.rabitq_entry() == run["search_entry"]
            assert (ids == exp).all()
            assert st.error_flags == 0
    finally:
        ix.close()


@pytest.mark.parametrize("storage", ["u8", "f32"])
@pytest.mark.parametrize("seed", [12345, 7])
def test_byte_valued_rows_match_reference_tool(storage, seed, tmp_path, monkeypatch):
    """i128 rows are integers in [0, 255]: the index keeps a byte copy unless
    f32 storage is forced; both must give the reference tool's file.  The
    base holds -0.0 values (rounded negatives), which the byte copy drops and
    the writer restores from the positions the index kept."""
    g = G.load("i128")
    ref = _ref_codebook(g.files["base"], g.files["graph"], str(tmp_path / "ref.bin"), seed)
    if storage == "f32":
        monkeypatch.setenv("BSEARCH_STORAGE", "f32")
    ix = B.Index.from_arrays(g.base, g.edges)
    try:
        out = str(tmp_path / "ours.bin")
        ix.build_codebook(seed, out)
    finally:
        ix.close()
    assert open(out, "rb").read() == open(ref, "rb").read()


def test_missing_neighbours_and_duplicate_rows_match_reference_tool(tmp_path):
    """Edges set to UINT32_MAX (no neighbour: triple_x = FLT_MAX) and
    neighbours whose row equals the node's own (zero residual: the factors'
    infinities and NaN) go through the same formulas as the reference tool."""
    rng = np.random.default_rng(5)
    n, dim, deg = 700, 40, 16
    base = rng.standard_normal((n, dim)).astype(np.float32)
    base[100:110] = base[99]                    # duplicate rows
    edges = rng.integers(0, n, size=(n, deg)).astype(np.uint32)
    edges[::7, -3:] = 0xFFFFFFFF                # missing neighbours
    edges[100:110, 0] = 99                      # edges to an identical row
    bpath, gpath = str(tmp_path / "b.fvecs"), str(tmp_path / "g.bin")
    ds.write_fvecs(bpath, base)
    ds.write_graph(gpath, edges)
    ref = _ref_codebook(bpath, gpath, str(tmp_path / "ref.bin"))
    ix = B.Index.from_arrays(base, edges)
    try:
        out = str(tmp_path / "ours.bin")
        ix.build_codebook(12345, out)
    finally:
        ix.close()
    a, b = open(out, "rb").read(), open(ref, "rb").read()
    assert len(a) == len(b)
    if a != b:
        x, y = np.frombuffer(a, np.uint32), np.frombuffer(b, np.uint32)
        bad = np.nonzero(x != y)[0]
        pytest.fail(f"{bad.size} words differ, first at {bad[:8]}: {x[bad[:8]]} vs {y[bad[:8]]}")


def test_cli_writes_the_reference_file(tmp_path):
    g = G.load("s96d64")
    out = str(tmp_path / "cli.bin")
    r = subprocess.run([CLI, "-base", g.files["base"], "-graph", g.files["graph"], "-out", out, "-seed", "12345"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "Entry point (medoid): " in r.stdout
    assert _sha(out) == g.meta["codebook_sha256"]


def test_cli_usage_error():
    r = subprocess.run([CLI, "-base", "x"], capture_output=True, text=True)
    assert r.returncode == 1 and "Usage:" in r.stderr
