"""Regenerates the golden fixtures under tests/golden/ from the reference's own
tools (compiled into oracle/_ref/ by `make -C oracle REF=<reference tree>`):

* base / query vectors: the seeded generators of beam_search_collab_b200.datasets
  (not stored; regenerated bit-identically by the tests)
* graph.bin            : oracle/_ref/build_graph  (--degree D --beam-width 128 --alpha 2.0 --seed 1234)
* codebook             : oracle/_ref/build_rabitq (-seed 12345); stored as its sha256 only,
                         the tests rebuild it with the same tool
* expected ids         : oracle/_ref/ref_search_omp, i.e. the reference's CPUBaseSearch /
                         CPURabitqSearch classes, one file per (mode, K, topk_size)
* cpu_cli report       : the reference cpu_cli as shipped (entry point, printed recall)

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from beam_search_collab_b200 import datasets as ds  # noqa: E402
import oracle as O  # noqa: E402

# name -> (generator, kwargs, degree, with codebook, [(mode, K, topk)])
SETS = {
    "f48": ("c1", dict(n=2000, nq=200, dim=48), 32, True,
            [("base", 10, 64), ("base", 100, 128), ("base", 16, 96), ("base", 10, 32),
             ("rabitq", 10, 64), ("rabitq", 20, 200)]),
    "i128": ("c2", dict(n=2000, nq=200), 32, False,
             [("base", 10, 64), ("base", 100, 256), ("base", 10, 512)]),
    "s96d64": ("c3", dict(n=1500, nq=150), 64, True,
               [("base", 10, 64), ("base", 50, 160), ("rabitq", 10, 128)]),
}


def sha(path_or_bytes) -> str:
    h = hashlib.sha256()
    if isinstance(path_or_bytes, (bytes, bytearray, memoryview)):
        h.update(path_or_bytes)
    else:
        with open(path_or_bytes, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def make_set(name, gen, kw, degree, with_cb, runs, tmp):
    out = os.path.join(HERE, name)
    os.makedirs(out, exist_ok=True)
    s = ds.GENERATORS[gen](**kw)
    base_p, query_p, gt_p = (os.path.join(tmp, f"{name}_{x}") for x in ("base.fvecs", "query.fvecs", "gt.ivecs"))
    ds.write_fvecs(base_p, s.base)
    ds.write_fvecs(query_p, s.queries)
    gt = ds.ground_truth(s.base, s.queries, 100)
    ds.write_ivecs(gt_p, gt)
    graph_p = os.path.join(out, "graph.bin")
    subprocess.run([O.ref_tool("build_graph"), "--base", base_p, "--graph", graph_p, "--degree", str(degree),
                    "--beam-width", "128", "--alpha", "2.0", "--seed", "1234"], check=True,
                   capture_output=True)
    meta = {"generator": gen, "kwargs": kw, "degree": degree,
            "base_sha256": sha(s.base.tobytes()), "query_sha256": sha(s.queries.tobytes()),
            "gt_sha256": sha(gt.tobytes()), "graph_sha256": sha(graph_p), "runs": []}
    cb_p = None
    if with_cb:
        cb_p = os.path.join(tmp, f"{name}_codebook.bin")
        subprocess.run([O.ref_tool("build_rabitq"), "-base", base_p, "-graph", graph_p, "-out", cb_p,
                        "-seed", "12345"], check=True, capture_output=True)
        meta["codebook_sha256"] = sha(cb_p)
    for mode, K, topk in runs:
        ids_p = os.path.join(out, f"expected_{mode}_K{K}_T{topk}.u32")
        info, ids = O.run_ref_search(graph_p, base_p, query_p, K=K, topk=topk, mode=mode,
                                     codebook=cb_p, out=ids_p)
        cfg = {"data": {"graph": graph_p, "base": base_p, "query": query_p, "gt": gt_p},
               "search": {"mode": mode, "K": K, "topk_size": topk, "max_iterations": 1024}}
        if cb_p:
            cfg["data"]["codebook"] = cb_p
        rep = O.run_cpu_cli(cfg)
        entry = int(re.search(r"entry=(\d+)", rep).group(1))
        recall = float(re.search(r"recall@\d+: ([0-9.eE+-]+)", rep).group(1))
        meta["runs"].append({"mode": mode, "K": K, "topk_size": topk, "file": os.path.basename(ids_p),
                             "search_entry": info["entry"], "cpu_cli_entry": entry,
                             "cpu_cli_recall": recall, "ids_sha256": sha(ids.tobytes())})
        print(name, mode, K, topk, "entry", info["entry"], "cpu_cli recall", recall)
    with open(os.path.join(out, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1)


def main():
    if O.ref_tool("build_graph") is None:
        raise SystemExit("oracle/_ref tools missing: run `make -C oracle REF=<reference tree>`")
    with tempfile.TemporaryDirectory() as tmp:
        for name, (gen, kw, degree, with_cb, runs) in SETS.items():
            make_set(name, gen, kw, degree, with_cb, runs, tmp)


if __name__ == "__main__":
    main()
