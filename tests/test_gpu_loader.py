"""GPU: the file loaders (bs_index_load, bs_index_load_codebook) stream the
reference's files to the device through page-locked staging buffers and take
them apart on the GPU (fvecs row headers, the value scan that picks the exact
byte copy, codebook rows into codes and factors).  An index loaded from the
files must be the index built from the host arrays: the same storage choice,
entry point, search rows and distance bits, RaBitQ results, and a codebook it
writes must be the reference build_rabitq's file byte for byte (byte rows keep
the -0.0 positions the scan found)."""
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


@pytest.mark.parametrize("name", G.NAMES)
def test_loaded_index_equals_index_from_arrays(name):
    g = G.load(name)
    a = B.Index.from_arrays(g.base, g.edges)
    b = B.Index.load(g.files["graph"], g.files["base"])
    try:
        assert a.info() == b.info()
        assert a.entry_point() == b.entry_point() == g.entry
        for mode, K, topk in (("warp4", 10, 64), ("bwarp2", 10, 64)):
            ra = a.search(g.queries, mode=mode, K=K, topk_size=topk)
            rb = b.search(g.queries, mode=mode, K=K, topk_size=topk)
            assert np.array_equal(ra[0], rb[0])
            assert np.array_equal(ra[1].view(np.uint32), rb[1].view(np.uint32))
            assert ra[2].row_bytes == rb[2].row_bytes and ra[2].integer_exact == rb[2].integer_exact
        if g.codebook_path:
            a.load_codebook(g.codebook_path)
            b.load_codebook(g.codebook_path)
            assert a.rabitq_entry() == b.rabitq_entry()
            for m, K, topk in g.runs("rabitq"):
                exp, _ = g.expected(m, K, topk)
                ids, d, st = b.search(g.queries, mode="rabitq", K=K, topk_size=topk)
                assert (ids == exp).all()
                ra = a.search(g.queries, mode="rabitq", K=K, topk_size=topk)
                assert np.array_equal(ra[1].view(np.uint32), d.view(np.uint32))
    finally:
        a.close()
        b.close()


def test_codebook_from_loaded_byte_rows_matches_reference_tool(tmp_path):
    """C2-style rows: integers 0..255 with some -0.0 values (rounding), stored
    as bytes; the codebook written back must carry the -0.0 bit patterns."""
    tool = O.ref_tool("build_rabitq")
    if tool is None:
        pytest.skip("reference build_rabitq not built")
    g = G.load("i128")
    assert np.count_nonzero(np.signbit(g.base) & (g.base == 0)) > 0
    ours, ref = os.path.join(tmp_path, "ours.bin"), os.path.join(tmp_path, "ref.bin")
    ix = B.Index.load(g.files["graph"], g.files["base"])
    try:
        _, _, st = ix.search(g.queries[:4], mode="warp1", K=5, topk_size=32)
        assert st.row_bytes == 128          # byte storage
        ix.build_codebook(12345, ours)
    finally:
        ix.close()
    subprocess.run([tool, "-base", g.files["base"], "-graph", g.files["graph"], "-out", ref, "-seed", "12345"],
                   check=True, capture_output=True)
    with open(ours, "rb") as a, open(ref, "rb") as b:
        assert a.read() == b.read()


def test_loader_rejects_bad_files(tmp_path):
    g = G.load("f48")
    bad = os.path.join(tmp_path, "bad.fvecs")
    with open(g.files["base"], "rb") as f:
        data = bytearray(f.read())
    data[4 * 49 * 7: 4 * 49 * 7 + 4] = np.int32(47).tobytes()      # row 7 claims 47 dimensions
    with open(bad, "wb") as f:
        f.write(data)
    with pytest.raises(B.BSearchError) as e:
        B.Index.load(g.files["graph"], bad)
    assert e.value.status == 3 and "Inconsistent row dimension" in str(e.value)
    short = os.path.join(tmp_path, "short.bin")
    with open(g.files["graph"], "rb") as f:
        with open(short, "wb") as o:
            o.write(f.read()[:-4])
    with pytest.raises(B.BSearchError) as e:
        B.Index.load(short, g.files["base"])
    assert "Truncated graph file" in str(e.value)
