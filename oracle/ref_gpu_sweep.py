"""BASELINE INFRASTRUCTURE ONLY: the reference's own GPU search (its gpu_cli,
compiled for sm_100a into oracle/_ref/gpu_cli by `make -C oracle gpu
REF=<reference tree>`) timed on the C2 workload, next to this build's drop-in
CLI (bin/gpu_cli) run with the same JSON configurations on the same files.

Both CLIs load the files, upload the index, run 5 back-to-back searches of all
queries and print "  time: X ms  qps: Y" (wall clock, mean of the 5 launches,
queries already on the device; reference src/gpu_cli.cu:153-165) and
"recall@10: R".  The ground-truth file holds exactly the 10 nearest ids per
query (ties by id), so the printed recall -- the reference definition,
src/gpu_cli.cu:28-51, which counts returned ids found anywhere in the file's
row -- is the standard recall@10.

    python oracle/ref_gpu_sweep.py [--out results.jsonl] [--modes ...] [--topks ...]

Prints one JSON line per run and a summary line: the best configuration of
each implementation whose recall@10 is >= 0.95, and their ratio.  The
reference gpu_cli is only run with K <= graph degree: with K above the degree
its final flush writes K distances into a degree-sized shared-memory buffer
(include/gpu_search_warp.cuh:237 and include/gpu_search_base.cuh:246 write
into the cand_dist_ buffer sized at :84-88 / :95-99), past the end of the
block's shared memory -- the illegal memory access it raised on the 960-d
workload at K=100.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)

REF_CLI = os.path.join(HERE, "_ref", "gpu_cli")
OUR_CLI = os.path.join(ROOT, "beam_search_collab_b200", "bin", "gpu_cli")
REF_MODES = ("base", "warp1", "warp2", "warp4", "bwarp1", "bwarp2", "bwarp4")
OUR_MODES = ("warp4", "warp1", "bwarp2")
TOPKS = (32, 48, 56, 64, 96, 128)
K = 10


def parse(stdout: str):
    m = re.search(r"time: ([0-9.eE+-]+) ms\s+qps: ([0-9.eE+-]+)", stdout)
    r = re.search(r"recall@\d+: ([0-9.eE+-]+)", stdout)
    return (float(m.group(1)) if m else None, float(m.group(2)) if m else None,
            float(r.group(1)) if r else None)


def run(cli, data, mode, topk):
    cfg = {"data": data, "search": {"mode": mode, "K": K, "topk_size": topk, "filter_capacity": 1024,
                                    "max_iterations": 1024, "reset_interval": 16}}
    p = subprocess.run([cli], input=json.dumps(cfg), capture_output=True, text=True, timeout=600)
    ms, qps, rec = parse(p.stdout)
    return {"rc": p.returncode, "ms": ms, "qps": qps, "recall@10": rec,
            "stderr": p.stderr.strip().splitlines()[-1] if p.returncode and p.stderr.strip() else None}


def main():
    import torch
    from beam_search_collab_b200 import datasets as ds
    import bench

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--modes", nargs="*", default=list(REF_MODES))
    ap.add_argument("--our-modes", nargs="*", default=list(OUR_MODES))
    ap.add_argument("--topks", nargs="*", type=int, default=list(TOPKS))
    ap.add_argument("--codebook", default=None, help="codebook.bin of the C2 graph (rabitq runs)")
    a = ap.parse_args()
    if not os.access(REF_CLI, os.X_OK):
        raise SystemExit("oracle/_ref/gpu_cli is not built (make -C oracle gpu REF=<reference tree>)")
    graph = os.path.join(ROOT, "bench_data", "c2", "graph.bin")
    s = ds.gen_c2(n=1_000_000, nq=10_000)
    base_t = torch.from_numpy(s.base).cuda()
    gt = bench.gpu_ground_truth(base_t, torch.from_numpy(s.queries).cuda(), K).astype(np.int32)
    del base_t
    torch.cuda.empty_cache()
    rows = []
    out = open(a.out, "w") if a.out else None
    with tempfile.TemporaryDirectory() as tmp:
        data = {"graph": graph, "base": os.path.join(tmp, "base.fvecs"), "query": os.path.join(tmp, "query.fvecs"),
                "gt": os.path.join(tmp, "gt.ivecs")}
        ds.write_fvecs(data["base"], s.base)
        ds.write_fvecs(data["query"], s.queries)
        ds.write_ivecs(data["gt"], gt)
        if a.codebook:
            if not os.path.exists(a.codebook):
                # the reference builder, seed 12345 (as the benchmark's C2+RaBitQ workload)
                subprocess.run([os.path.join(HERE, "_ref", "build_rabitq"), "-base", data["base"], "-graph", graph,
                                "-out", a.codebook, "-seed", "12345"], check=True, stdout=subprocess.DEVNULL)
            data["codebook"] = a.codebook
        plan = [("reference", REF_CLI, m) for m in a.modes] + [("ours", OUR_CLI, m) for m in a.our_modes]
        for impl, cli, mode in plan:
            for t in a.topks:
                if t < K:
                    continue
                r = {"impl": impl, "mode": mode, "topk_size": t, **run(cli, data, mode, t)}
                rows.append(r)
                line = json.dumps(r)
                print(line, flush=True)
                if out:
                    out.write(line + "\n")
                    out.flush()
    best = {}
    for impl in ("reference", "ours"):
        ok = [r for r in rows if r["impl"] == impl and r["rc"] == 0 and r["qps"] and (r["recall@10"] or 0) >= 0.95]
        best[impl] = max(ok, key=lambda r: r["qps"]) if ok else None
    summ = {"summary": True, "best_reference": best["reference"], "best_ours": best["ours"],
            "ratio": (best["ours"]["qps"] / best["reference"]["qps"]) if best["ours"] and best["reference"] else None}
    print(json.dumps(summ), flush=True)
    if out:
        out.write(json.dumps(summ) + "\n")
        out.close()


if __name__ == "__main__":
    main()
