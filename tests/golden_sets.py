"""Loads the golden fixtures of tests/golden/ (see make_golden.py).

Vectors are regenerated from the seeded generators and checked against the
recorded sha256; codebooks are rebuilt with the reference's build_rabitq
(oracle/_ref) into a cache and checked the same way."""
from __future__ import annotations

import functools
import hashlib
import json
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

from beam_search_collab_b200 import datasets as ds
import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
NAMES = ("f48", "i128", "s96d64")


def _sha(b) -> str:
    return hashlib.sha256(b).hexdigest()


@dataclass
class GoldenSet:
    name: str
    base: np.ndarray
    queries: np.ndarray
    edges: np.ndarray
    gt: np.ndarray
    meta: dict
    dir: str
    codebook_path: str | None = None
    files: dict = field(default_factory=dict)

    def expected(self, mode, K, topk):
        for r in self.meta["runs"]:
            if (r["mode"], r["K"], r["topk_size"]) == (mode, K, topk):
                ids = np.fromfile(os.path.join(self.dir, r["file"]), dtype=np.uint32)
                return ids.reshape(self.queries.shape[0], K), r
        raise KeyError((mode, K, topk))

    def runs(self, mode=None):
        return [(r["mode"], r["K"], r["topk_size"]) for r in self.meta["runs"] if mode in (None, r["mode"])]

    @property
    def entry(self) -> int:
        return self.meta["runs"][0]["cpu_cli_entry"]

    def codebook(self):
        if self.codebook_path is None:
            return None
        return ds.read_codebook(self.codebook_path, self.base.shape[0], self.base.shape[1], self.edges.shape[1])


def _cache_dir():
    d = os.path.join(ds.cache_dir(), "golden_cache")
    os.makedirs(d, exist_ok=True)
    return d


@functools.lru_cache(maxsize=None)
def load(name: str) -> GoldenSet:
    d = os.path.join(GOLDEN, name)
    with open(os.path.join(d, "meta.json")) as f:
        meta = json.load(f)
    s = ds.GENERATORS[meta["generator"]](**meta["kwargs"])
    assert _sha(s.base.tobytes()) == meta["base_sha256"], "base generator drifted"
    assert _sha(s.queries.tobytes()) == meta["query_sha256"], "query generator drifted"
    edges = ds.read_graph(os.path.join(d, "graph.bin"))
    gt = ds.ground_truth(s.base, s.queries, 100)
    g = GoldenSet(name, s.base, s.queries, edges, gt, meta, d)
    cache = _cache_dir()
    g.files["base"] = os.path.join(cache, f"{name}_base.fvecs")
    g.files["query"] = os.path.join(cache, f"{name}_query.fvecs")
    g.files["gt"] = os.path.join(cache, f"{name}_gt.ivecs")
    g.files["graph"] = os.path.join(d, "graph.bin")
    ds.write_fvecs(g.files["base"], s.base)
    ds.write_fvecs(g.files["query"], s.queries)
    ds.write_ivecs(g.files["gt"], gt)
    if "codebook_sha256" in meta:
        cb = os.path.join(cache, f"{name}_codebook.bin")
        ok = os.path.exists(cb) and _sha(open(cb, "rb").read()) == meta["codebook_sha256"]
        if not ok and O.ref_tool("build_rabitq"):
            subprocess.run([O.ref_tool("build_rabitq"), "-base", g.files["base"], "-graph", g.files["graph"],
                            "-out", cb, "-seed", "12345"], check=True, capture_output=True)
            ok = _sha(open(cb, "rb").read()) == meta["codebook_sha256"]
        if ok:
            g.codebook_path = cb
            g.files["codebook"] = cb
    return g
