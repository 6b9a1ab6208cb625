"""Benchmark: QPS at recall@10 >= 0.95 on the C2 workload.

C2 = 1,000,000 x 128 integer-valued [0,255] base vectors (seeded mixture of
1,024 Gaussians, ~30% zeros), 10,000 queries per GPU, degree-32 Vamana graph
(beam 128, alpha 2.0, seed 1234 -- the reference build_graph settings),
K = 10.  The operating point is the smallest beam (topk_size) whose
recall@10 against the exact top-10 is >= 0.95; a "step" is one search of all
of a GPU's queries at that point.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c3|c4] [--measure search|codebook]

--config selects another BASELINE.json workload for measurement (default and
the driver's line: c2): c3 = RaBitQ search (1M x 96 unit vectors, degree 64,
the reference build_rabitq codebook), c4 = 960-d exact search (1k queries,
K 100, topk 256).  Their graphs and codebooks live in bench_data/<config>/.

Arms
  ours       : the CUDA search through the C ABI (lib/libbsearch_b200.so).
               value = device-resident queries / results (kernel + counter
               reset per step), L2 flushed by a 256 MiB write before every
               timed step (outside the timed window).  e2e = the same search
               through the same public call with pinned host buffers, H2D of
               the queries and D2H of ids+dists inside the timed window.
  reference  : the reference's own CPU search (CPUBaseSearch through
               oracle/_ref/ref_search_omp, all host cores), same data, K and
               topk; each step a bounded sample of the queries.

--measure codebook times the GPU RaBitQ codebook builder on the workload's
base and graph instead (one JSON line, edges/s; the reference build_rabitq on
all host threads as the CPU baseline, and the two codebook files compared).
--measure graph times the GPU graph builder on the workload's base (nodes/s)
and compares its graph.bin with the reference build_graph's.

Multi-GPU (torchrun, one rank per GPU): query sharding over a replicated
index, no collective on the data path.  --scaling weak (default): every rank
searches its own 10,000 queries; --scaling strong: the workload's 10,000
queries are split over the ranks.  value = all ranks' queries / max-over-ranks
time.

Checks carried in the line: `parity` compares our rows with the reference CPU
search's rows for the CPU-baseline sample (identical rows, distances, recall);
`config.kernel_errors` holds the kernels' error bits from the timed launches
(a non-zero value aborts the run).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DATA_DIR = os.path.join(ROOT, "bench_data")
GRAPH_C2 = os.path.join(DATA_DIR, "c2", "graph.bin")
TOPK_SWEEP = (16, 24, 32, 40, 48, 52, 56, 60, 64, 72, 80, 96, 128, 192, 256)
TARGET_RECALL = 0.95
K = 10
NQ_PER_GPU = 10_000
FLUSH_BYTES = 256 << 20
# topk_size at which the C2 search first reaches recall@10 >= 0.95 (the sweep
# of the GPU arm finds it; the CPU reference arm, which cannot afford the
# ground truth, searches at the same point)
C2_OPERATING_TOPK = 56

# Workloads.  The driver's bench line is C2; C3 and
# C4 measure the RaBitQ path and the 960-d gather path with --config.
CONFIGS = {
    "c2": dict(gen="gen_c2", nq=10_000, mode="warp4", K=10, sweep=TOPK_SWEEP, codebook=False,
               operating_topk=C2_OPERATING_TOPK,
               workload="C2: 1M x 128 int-valued base, 10k queries per GPU, degree-32 Vamana, K=10",
               data="synthetic: seeded C2 mixture (1,024 Gaussians, ints 0..255), graph from the "
                    "reference build_graph settings"),
    "c3": dict(gen="gen_c3", nq=10_000, mode="rabitq", K=10, sweep=(128, 160, 192, 256, 384, 512), codebook=True,
               workload="C3: 1M x 96 unit-norm base, 10k queries per GPU, degree-64 Vamana, RaBitQ codebook "
                        "(build_rabitq seed 12345), K=10, exact rerank",
               data="synthetic: seeded C3 mixture (256 clusters on the unit sphere, concentration 20), graph "
                    "and codebook from the reference build_graph / build_rabitq"),
    # C2 with a RaBitQ codebook (dim 128 = padded_dim, so the codes cover every
    # rotated component; the reference build_rabitq, seed 12345, makes it on
    # first use): a RaBitQ workload with a real recall/QPS curve
    "c2rq": dict(gen="gen_c2", nq=10_000, mode="rabitq", K=10, sweep=(32, 48, 64, 96, 128, 192, 256, 384, 512),
                 codebook=True, data_dir="c2",
                 workload="C2 + RaBitQ: 1M x 128 int-valued base, 10k queries per GPU, degree-32 Vamana, "
                          "RaBitQ codebook (build_rabitq seed 12345), K=10, exact rerank",
                 data="synthetic: seeded C2 mixture (1,024 Gaussians, ints 0..255), graph and codebook from the "
                      "reference build_graph / build_rabitq"),
    # a 200,000-row slice of the C2 distribution with its own graph and
    # codebook (reference tools): small enough for full ncu captures of the
    # search kernels (a few hundred MB on the device), rows still beyond L2
    "c2s": dict(gen="gen_c2", gen_kwargs={"n": 200_000}, nq=10_000, mode="rabitq", K=10,
                sweep=(32, 48, 56, 64, 96, 128, 192, 256), codebook=True,
                workload="C2 slice for profiling: 200k x 128 int-valued base, 10k queries, degree-32 Vamana, "
                         "RaBitQ codebook (build_rabitq seed 12345), K=10",
                data="synthetic: seeded C2 mixture (1,024 Gaussians, ints 0..255) at 200k rows, graph and "
                     "codebook from the reference build_graph / build_rabitq"),
    "c4": dict(gen="gen_c4", nq=1_000, mode="base", K=100, sweep=(256,), codebook=False,
               workload="C4: 1M x 960 non-negative base, 1k queries per GPU, degree-32 Vamana, K=100, topk 256",
               data="synthetic: seeded C4 (|N(0,1)| * 0.1 * per-dimension log-uniform scale), graph from the "
                    "reference build_graph settings"),
}
CFG_NAME = "c2"


def build_missing_graph(base, graph):
    """A workload's graph.bin when it is not in bench_data/ yet: the reference
    settings (degree 32, beam 128, alpha 2.0, seed 1234) through the GPU graph
    builder, whose file equals the reference build_graph's edge for edge
    (tests/test_gpu_graph_build.py; all 1,000,000 rows of the C2 graph)."""
    import beam_search_collab_b200 as B
    log(f"building {graph} on the GPU (reference build_graph settings)")
    os.makedirs(os.path.dirname(graph), exist_ok=True)
    ix = B.Index.from_vectors(base, 32)
    try:
        edges = ix.build_graph(beam_width=128, alpha=2.0, seed=1234)
    finally:
        ix.close()
    tmp = graph + ".tmp"
    with open(tmp, "wb") as f:
        np.array([base.shape[0], 32], dtype=np.int32).tofile(f)
        np.ascontiguousarray(edges, dtype=np.uint32).tofile(f)
    os.replace(tmp, graph)


def config_data(name: str, nq_total: int):
    """Base, queries, graph edges and codebook path (or None) of a workload;
    graphs and codebooks are built once with the reference tools into
    bench_data/<config>/ (git-ignored, shipped to the GPU box)."""
    from beam_search_collab_b200 import datasets as ds
    cfg = CONFIGS[name]
    s = getattr(ds, cfg["gen"])(nq=nq_total, **cfg.get("gen_kwargs", {}))
    ddir = os.path.join(DATA_DIR, cfg.get("data_dir", name))
    graph = os.path.join(ddir, "graph.bin")
    if not os.path.exists(graph):
        build_missing_graph(s.base, graph)
    cb = os.path.join(ddir, "codebook.bin") if cfg["codebook"] else None
    if cb and not os.path.exists(cb):
        # too large to ship (2.4 GB for C3): the reference build_rabitq makes it here
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        tool = O.ref_tool("build_rabitq")
        if tool is None:
            raise SystemExit(f"missing {cb}: build it with the reference build_rabitq (-seed 12345)")
        with tempfile.TemporaryDirectory() as tmp:
            bp = os.path.join(tmp, "base.fvecs")
            ds.write_fvecs(bp, s.base)
            subprocess.run([tool, "-base", bp, "-graph", graph, "-out", cb, "-seed", "12345"], check=True,
                           stdout=subprocess.DEVNULL)
    return s.base, s.queries, ds.read_graph(graph), cb


# ------------------------------------------------------------------ helpers

def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def host_threads() -> int:
    """Host threads this process may use (torchrun sets OMP_NUM_THREADS=1 for
    its ranks; the CPU reference is given the affinity count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """SM clocks and throttle reasons sampled through NVML every millisecond
    while the timed region runs (nvidia-smi's own loop samples every 20 ms at
    best, too coarse for a timed region of a few milliseconds)."""
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, torch_device: int):
        self.dev = torch_device
        self.samples = []
        self.stop = threading.Event()
        self.t = None
        self.h = None
        self.smax = None
        self.err = None

    def __enter__(self):
        try:
            import pynvml
            import torch
            self.nv = pynvml
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
                uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
                self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[self.dev]) if vis else self.dev
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.bits = (pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap)
            self._sample()
            self.samples.clear()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:   # no NVML: the line says so
            self.err = repr(e)
            self.h = None
        return self

    def _sample(self):
        sm = float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
        rs = int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
        self.samples.append((sm, rs))

    def _run(self):
        while not self.stop.is_set():
            self._sample()
            time.sleep(0.001)

    def __exit__(self, *exc):
        if self.t:
            self.stop.set()
            self.t.join(timeout=2)
            if not self.samples:
                self._sample()

    def summary(self):
        if self.h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.err}
        sm = [a for a, _ in self.samples]
        reasons = sorted({nm for _, r in self.samples for nm, b in zip(self.NAMES, self.bits) if r & b})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax, "reasons": reasons,
                "samples": len(sm), "interval_ms": 1}


def c2_data(nq_total: int):
    from beam_search_collab_b200 import datasets as ds
    s = ds.gen_c2(n=1_000_000, nq=nq_total)
    return s.base, s.queries


def load_graph():
    from beam_search_collab_b200 import datasets as ds
    if not os.path.exists(GRAPH_C2):
        raise SystemExit(f"missing {GRAPH_C2}: build it with the reference settings "
                         "(degree 32, beam 128, alpha 2.0, seed 1234) over the C2 base vectors")
    return ds.read_graph(GRAPH_C2)


def gpu_ground_truth(base_t, q_t, k, chunk=None):
    """Exact top-k ids by squared L2, ties by id (float64 on the GPU: exact for
    these integer-valued vectors).  `chunk` queries at a time (default: a
    [chunk, n] float64 block of about 4 GB)."""
    import torch
    b64 = base_t.double()
    bn = (b64 * b64).sum(1)
    out = np.empty((q_t.shape[0], k), dtype=np.int64)
    extra = 32
    chunk = chunk or max(1, min(512, (4 << 30) // (8 * base_t.shape[0])))
    for s in range(0, q_t.shape[0], chunk):
        q = q_t[s:s + chunk].double()
        d = bn[None, :] - 2.0 * (q @ b64.T) + (q * q).sum(1, keepdim=True)
        vals, idx = torch.topk(d, k + extra, dim=1, largest=False, sorted=True)
        vals, idx = vals.cpu().numpy(), idx.cpu().numpy()
        for r in range(idx.shape[0]):
            o = np.lexsort((idx[r], vals[r]))
            out[s + r] = idx[r][o][:k]
    return out


def recall_at_k(pred, gt, k=K):
    hits = 0
    for p, g in zip(pred[:, :k], gt[:, :k]):
        hits += len(set(p.tolist()) & set(g.tolist()))
    return hits / (gt.shape[0] * k)


CLI_SEARCH = {"filter_capacity": 1024, "max_iterations": 1024, "reset_interval": 16}


def run_cli(cli, data, mode, topk, k=None):
    """One run of a gpu_cli-style binary (ours: bin/gpu_cli; the reference's:
    oracle/_ref/gpu_cli) with the reference JSON on stdin.  Both load the
    files, upload the index, run 5 back-to-back searches of all queries with
    the queries already on the device and print "time: X ms  qps: Y" (wall
    clock, mean of the 5 launches; reference src/gpu_cli.cu:153-165) and
    "recall@K: R" against the ground-truth file."""
    import re
    cfg = {"data": data, "search": {"mode": mode, "K": k or K, "topk_size": topk, **CLI_SEARCH}}
    t = time.time()
    p = subprocess.run([cli], input=json.dumps(cfg), capture_output=True, text=True, timeout=600)
    m = re.search(r"time: ([0-9.eE+-]+) ms\s+qps: ([0-9.eE+-]+)", p.stdout)
    r = re.search(r"recall@\d+: ([0-9.eE+-]+)", p.stdout)
    out = {"mode": mode, "topk_size": topk, "rc": p.returncode,
           "ms": float(m.group(1)) if m else None, "qps": round(float(m.group(2)), 1) if m else None,
           "recall@10": float(r.group(1)) if r else None, "wall_s": round(time.time() - t, 2)}
    if p.returncode and p.stderr.strip():
        out["stderr"] = p.stderr.strip().splitlines()[-1]
    return out


def write_cli_files(tmp, base, queries, gt, graph):
    """graph.bin path plus base/query fvecs and a 10-column ground-truth ivecs
    in `tmp`: the file set both CLIs read."""
    from beam_search_collab_b200 import datasets as ds
    data = {"graph": graph, "base": os.path.join(tmp, "base.fvecs"), "query": os.path.join(tmp, "query.fvecs"),
            "gt": os.path.join(tmp, "gt.ivecs")}
    ds.write_fvecs(data["base"], base)
    ds.write_fvecs(data["query"], queries)
    ds.write_ivecs(data["gt"], np.ascontiguousarray(gt[:, :K]).astype(np.int32))
    return data


# --------------------------------------------------------------- our arm

def query_share(rank, world, strong):
    """This rank's query range: weak scaling gives every rank its own
    NQ_PER_GPU queries; strong scaling splits the workload's NQ_PER_GPU
    queries over the ranks (contiguous ranges)."""
    if not strong:
        return rank * NQ_PER_GPU, (rank + 1) * NQ_PER_GPU
    return rank * NQ_PER_GPU // world, (rank + 1) * NQ_PER_GPU // world


def useful_distance_count(B, base, edges, queries, params, local_rank):
    """Distances the reference search itself computes for these queries (one
    per distinct pushed node): the gather-layout kernel with a visited table
    that never resets counts exactly those (pinned against the CPU oracle by
    the GPU tests).  Untimed; the block layout scores every row of a block."""
    old = os.environ.get("BSEARCH_LAYOUT")
    os.environ["BSEARCH_LAYOUT"] = "gather"
    try:
        gx = B.Index.from_arrays(base, edges, device=local_rank)
    finally:
        if old is None:
            os.environ.pop("BSEARCH_LAYOUT")
        else:
            os.environ["BSEARCH_LAYOUT"] = old
    try:
        # one warp per block: room for a 16k-slot table (reset only past 12k
        # inserts, i.e. hundreds of expansions); the results do not depend on
        # the warps per block
        mode = "warp1" if params.mode in ("base", "warp1", "warp2", "warp4", "warp8") else params.mode
        p = B.SearchParams(mode=mode, K=params.K, topk_size=params.topk_size, filter_capacity=1 << 14)
        _, _, st = gx.search(queries, p, with_dists=False)
        return st.distances, st.expansions
    finally:
        gx.close()


def run_ours(args, rank, world, local_rank):
    import torch
    import beam_search_collab_b200 as B

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = CONFIGS[CFG_NAME]
    strong = args.scaling == "strong"
    t0 = time.time()
    base, queries_all, edges, codebook = config_data(CFG_NAME, NQ_PER_GPU * (1 if strong else world))
    q0, q1 = query_share(rank, world, strong)
    queries = np.ascontiguousarray(queries_all[q0:q1])
    nq = len(queries)
    nq_job = NQ_PER_GPU if strong else NQ_PER_GPU * world
    log(f"[rank {rank}] data ready in {time.time() - t0:.1f}s: base {base.shape}, graph {edges.shape}, "
        f"{nq} queries")
    ix = B.Index.from_arrays(base, edges, device=local_rank)
    if codebook:
        ix.load_codebook(codebook)
    entry = ix.rabitq_entry() if args.mode == "rabitq" else B.NO_NODE
    if entry == B.NO_NODE:
        entry = ix.entry_point()

    # exact top-10 (the library's brute-force ground truth, bs_ground_truth)
    q_std = torch.from_numpy(queries_all[:NQ_PER_GPU]).to(dev)
    torch.cuda.synchronize()
    t_gt = time.time()
    gt_ids, _ = ix.ground_truth(q_std, 10, with_dists=False)
    torch.cuda.synchronize()
    t_gt = time.time() - t_gt
    gt = gt_ids.cpu().numpy().view(np.uint32).astype(np.int64)

    # operating point: smallest beam reaching the recall target (same on every rank)
    chosen, sweep = None, []
    for T in ([args.topk] if args.topk else cfg["sweep"]):
        ids, _, st = ix.search(q_std, mode=args.mode, K=K, topk_size=T)
        torch.cuda.synchronize()
        if st.error_flags:
            raise SystemExit(f"search kernel reported error flags {st.error_flags:#x}")
        r = recall_at_k(ids.cpu().numpy().astype(np.int64), gt)
        sweep.append({"topk_size": T, "recall@10": round(r, 5)})
        if r >= TARGET_RECALL:
            chosen = T
            break
    if chosen is None:
        chosen = sweep[-1]["topk_size"]
    params = B.SearchParams(mode=args.mode, K=K, topk_size=chosen)

    # per-query counters at the operating point (untimed) for the roofline
    q_dev = torch.from_numpy(queries).to(dev)
    ids_d = torch.empty((nq, K), dtype=torch.int32, device=dev)
    dists_d = torch.empty((nq, K), dtype=torch.float32, device=dev)
    _, _, st = ix.search(q_dev, params)
    torch.cuda.synchronize()
    if st.error_flags:
        raise SystemExit(f"search kernel reported error flags {st.error_flags:#x}")
    dim, deg = base.shape[1], edges.shape[1]
    # query read + per expansion either one neighbourhood block (adjacency row
    # and all neighbour rows, copied whole) or the adjacency row and the rows of
    # the scored candidates as stored (u8 copy: 1 B/dim) + ids and distances
    useful_d = None
    if args.mode == "rabitq":
        # per expansion: adjacency row, the neighbours' 1-bit codes (pdim/8 B
        # each) and 3 f32 factors each, and the parent's exact row; then the
        # exact rerank rows of the final beam.  The node blocks carry exactly
        # these (padded to 16 B), one bulk copy per expansion.
        pdim = 1 << (dim - 1).bit_length()
        useful = (st.expansions * (4 * deg + deg * pdim // 8 + 12 * deg + st.row_bytes)
                  + st.rerank * st.row_bytes)
        per_expansion = (st.expansions * st.block_bytes + st.rerank * st.row_bytes) if st.block_bytes else useful
    elif st.block_bytes:
        per_expansion = st.expansions * st.block_bytes
        # the bytes the search needs in the stored row format: adjacency rows
        # and the rows of the distinct candidates the reference scores
        useful_d, _ = useful_distance_count(B, base, edges, queries, params, local_rank)
        useful = st.expansions * 4 * deg + useful_d * st.row_bytes
    else:
        per_expansion = st.expansions * 4 * deg + st.distances * st.row_bytes
        useful = per_expansion
    io_bytes = nq * 4 * dim + nq * 8 * K
    alg_bytes = io_bytes + per_expansion
    useful_bytes = io_bytes + useful

    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step():
        ix.search_raw(q_dev.data_ptr(), nq, ids_d.data_ptr(), dists_d.data_ptr(), params,
                      stream=stream.cuda_stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            flush.zero_()
            step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.zero_()                       # L2 flush, outside the timed window
                ev[i][0].record(stream)
                step()
                ev[i][1].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    t_ms = sum(step_ms)
    # the timed launches are asynchronous: their kernels' error bits are in the
    # index's error word
    kernel_errors = ix.take_errors(stream.cuda_stream)

    # e2e through the same public call with pinned host buffers
    hq = torch.from_numpy(queries).pin_memory()
    hid = torch.empty((nq, K), dtype=torch.int32).pin_memory()
    hdist = torch.empty((nq, K), dtype=torch.float32).pin_memory()
    # (steps enqueued back to back as for `value`: each step's kernel reads its
    # queries from the page-locked buffer over the bus and writes its result
    # rows back into page-locked memory, inside the step's events)
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        ix.search_raw(hq.data_ptr(), nq, hid.data_ptr(), hdist.data_ptr(), params, stream=stream.cuda_stream)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(e2e_steps)]
    with torch.cuda.stream(stream):
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            ix.search_raw(hq.data_ptr(), nq, hid.data_ptr(), hdist.data_ptr(), params, stream=stream.cuda_stream)
            b.record(stream)
    stream.synchronize()
    e2e_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    assert np.array_equal(hid.numpy(), ids_d.cpu().numpy()), "e2e results differ from device-resident results"
    kernel_errors |= ix.take_errors(stream.cuda_stream)

    # max over ranks (and any rank's kernel error bits)
    if world > 1:
        t = torch.tensor([t_ms, e2e_ms, float(kernel_errors)], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_ms, e2e_ms, kernel_errors = float(t[0]), float(t[1]), int(t[2])
    if kernel_errors:
        raise SystemExit(f"search kernels reported error flags {kernel_errors:#x} during the timed run")
    ms_per_step = t_ms / args.steps
    value = nq_job / (ms_per_step / 1e3)
    e2e_value = nq_job / (e2e_ms / 1e3)

    if rank != 0:
        return None
    peak, peak_kind = peaks()
    achieved = alg_bytes / (statistics.mean(step_ms) / 1e3) / 1e9
    achieved_useful = useful_bytes / (statistics.mean(step_ms) / 1e3) / 1e9
    traffic = None
    # DRAM bytes of one launch of this kernel on this workload
    # (dram__bytes_read.sum + dram__bytes_write.sum of an ncu capture of the
    # same launch, kept beside the ncu summaries)
    tp = os.path.join(ROOT, "profiles", f"traffic_{CFG_NAME}.json")
    if os.path.exists(tp) and not strong and world == 1:
        with open(tp) as f:
            tj = json.load(f)
        if tj.get("topk_size") == chosen and tj.get("mode") == args.mode and tj.get("layout") == (
                "blocks" if st.block_bytes else "gather"):
            traffic = tj.get("dram_bytes_per_launch")
    line = {
        "metric": "QPS at recall@10>=0.95",
        "value": round(value, 1),
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        # rows stored as bytes (128 B for the 128-d C2 rows): u8 products
        # summed exactly in int32 with __dp4a
        "dtype": "u8" if st.integer_exact and st.row_bytes == base.shape[1] else "f32",
        "data": cfg["data"],
        "config": {
            "workload": cfg["workload"] if not strong else cfg["workload"].replace(
                "per GPU", f"split over {world} GPU(s)"),
            "mode": args.mode, "K": K, "topk_size": chosen,
            "recall@10": sweep[-1]["recall@10"] if chosen == sweep[-1]["topk_size"] else None,
            "recall_sweep": sweep,
            "entry_point": entry,
            "queries_per_gpu": nq,
            "distance_path": ("integer-exact" if st.integer_exact else "sequential per lane")
                             + f", stored row {st.row_bytes} B",
            "layout": ((f"RaBitQ node blocks (adjacency, codes, factors, own row), {st.block_bytes} B bulk copy "
                        "per expansion" if args.mode == "rabitq" else
                        f"neighbourhood blocks, {st.block_bytes} B bulk copy per expansion")
                       if st.block_bytes else "gather"),
            "expansions_per_query": round(st.expansions / nq, 2),
            "distances_per_query": round(st.distances / nq, 2),
            "reference_distances_per_query": round(useful_d / nq, 2) if useful_d is not None else None,
            "l2": "256 MiB write before every timed step (outside the timed window); index "
                  f"{(base.nbytes * (st.row_bytes / (4 * base.shape[1])) + edges.nbytes) / 1e6:.0f} MB > L2",
            "parallelism": f"query-sharded dp{world}, replicated index",
            "kernel_errors": kernel_errors,
            "ground_truth": f"bs_ground_truth (exact brute force on the GPU), {round(t_gt, 3)} s for "
                            f"{NQ_PER_GPU} queries",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": int(alg_bytes),
            # the same time over the bytes the search itself needs (adjacency
            # rows + the rows of the distinct candidates the reference scores,
            # as stored): the layout moves more than that to save a round trip
            "useful_bytes_per_launch": int(useful_bytes),
            "achieved_useful": round(achieved_useful, 1),
            "frac_useful": round(achieved_useful / peak, 4),
        },
        "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                # all ranks' queries and results (the job's step, like `value`)
                "h2d_bytes_per_step": int(nq_job * base.shape[1] * 4),
                "d2h_bytes_per_step": int(nq_job * K * 8)},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"], ref_ids = cpu_baseline(base, queries, chosen, entry, codebook, sample=args.cpu_sample)
        if ref_ids is not None:
            line["parity"] = parity_vs_reference(ref_ids, ids_d.cpu().numpy().view(np.uint32),
                                                 dists_d.cpu().numpy(), base, queries, gt)
    if not args.no_cli and world == 1 and not codebook and CFG_NAME == "c2":
        # the drop-in CLI on the same files with the reference CLI's own
        # timing (the reference arm runs the reference gpu_cli the same way)
        import beam_search_collab_b200 as Bm
        with tempfile.TemporaryDirectory() as tmp:
            data = write_cli_files(tmp, base, queries, gt, os.path.join(DATA_DIR, cfg.get("data_dir", CFG_NAME),
                                                                         "graph.bin"))
            runs = [run_cli(Bm.CLI_PATH, data, args.mode, chosen), run_cli(Bm.CLI_PATH, data, args.mode, 64)]
        line["cli"] = {"binary": "bin/gpu_cli (this build's drop-in CLI)", "runs": runs,
                       "timing": "the CLI's own: wall clock, mean of 5 searches of all queries, queries on the "
                                 "device (reference src/gpu_cli.cu:153-165)"}
    return line


def parity_vs_reference(ref_ids, ids, dists, base, queries, gt):
    """Our result rows against the reference CPU search's rows for the same
    queries (the first len(ref_ids) of this rank's): identical rows, ids in
    agreement, our distances against the exact distances of the reference's
    ids (float64), and recall@10 of both against the exact top-10."""
    n = ref_ids.shape[0]
    ours = ids[:n]
    same_rows = (ours == ref_ids).all(axis=1)
    agree = (ours == ref_ids)
    sel = ref_ids != 0xFFFFFFFF
    q = queries[:n].astype(np.float64)
    rel = 0.0
    for i in range(n):
        m = agree[i] & sel[i]
        if not m.any():
            continue
        x = base[ref_ids[i][m]].astype(np.float64)
        exact = ((x - q[i]) ** 2).sum(axis=1)
        rel = max(rel, float(np.max(np.abs(dists[i][m] - exact) / np.maximum(exact, 1e-30))))
    r_ours = recall_at_k(ours.astype(np.int64), gt[:n])
    r_ref = recall_at_k(ref_ids.astype(np.int64), gt[:n])
    return {"queries": int(n), "identical_rows": round(float(same_rows.mean()), 6),
            "ids_match_frac": round(float(agree.mean()), 6), "max_rel_dist_err": rel,
            "recall@10_ours": round(r_ours, 5), "recall@10_reference": round(r_ref, 5),
            "recall_delta": round(r_ours - r_ref, 5),
            "against": "the reference's own CPU search (oracle/_ref/ref_search_omp) on the same graph, "
                       "queries, entry point, K and topk_size"}


# ------------------------------------------------------ reference CPU arm

def _write_inputs(tmp, base, queries):
    from beam_search_collab_b200 import datasets as ds
    bp, qp = os.path.join(tmp, "base.fvecs"), os.path.join(tmp, "query.fvecs")
    ds.write_fvecs(bp, base)
    ds.write_fvecs(qp, queries)
    return os.path.join(DATA_DIR, CONFIGS[CFG_NAME].get("data_dir", CFG_NAME), "graph.bin"), bp, qp


def _ref_search(paths, topk, entry, nq, codebook=None, out=None):
    """The reference CPU search on all host threads (explicitly: torchrun's
    OMP_NUM_THREADS=1 must not reach it).  Returns (info, ids or None)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    g, b, q = paths
    mode = "rabitq" if codebook else "base"
    return O.run_ref_search(g, b, q, K=K, topk=topk, mode=mode, codebook=codebook, threads=host_threads(), nq=nq,
                            entry=entry, out=out)


def _ref_class(codebook):
    return ("CPURabitqSearch (reference include/cpu_search_rabitq.hpp)" if codebook
            else "CPUBaseSearch (reference include/cpu_search_base.hpp)")


def cpu_baseline(base, queries, topk, entry, codebook=None, sample=2000):
    """The reference CPU search timed on a bounded sample of this workload's
    queries; also returns its result ids for the parity check (None when the
    reference tools were not built)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if O.ref_tool("ref_search_omp") is None:
        return {"value": None, "unit": "queries/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref/ref_search_omp not built"}, None
    with tempfile.TemporaryDirectory() as tmp:
        paths = _write_inputs(tmp, base, queries)
        info, ids = _ref_search(paths, topk, entry, min(sample, len(queries)), codebook,
                                out=os.path.join(tmp, "ref_ids.u32"))
    return {"value": round(info["qps"], 1), "unit": "queries/s", "cores": info["threads"], "kind": "reference",
            "sample": f"first {info['nq']} of the {len(queries)} queries, {_ref_class(codebook)} "
                      f"under OpenMP on {info['threads']} host threads, topk_size {topk}, K {K}"}, ids


def run_reference(args, rank, world):
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if O.ref_tool("ref_search_omp") is None:
        return {"impl": "reference", "unavailable": "oracle/_ref/ref_search_omp was not built from the reference tree"}
    cfg = CONFIGS[CFG_NAME]
    base, queries_all, _, codebook = config_data(CFG_NAME, NQ_PER_GPU)
    topk = args.topk or cfg.get("operating_topk") or cfg["sweep"][0]
    entry = None
    if codebook:   # the codebook's stored entry, as cpu_cli's rabitq path uses
        entry = int(np.fromfile(codebook, dtype=np.uint32, count=1)[0])
    if entry is None or entry == 0xFFFFFFFF:
        entry = O.entry_point(base)
    sample = min(args.ref_sample, NQ_PER_GPU)
    with tempfile.TemporaryDirectory() as tmp:
        paths = _write_inputs(tmp, base, queries_all)
        for _ in range(args.warmup):
            _ref_search(paths, topk, entry, sample, codebook)
        infos = [_ref_search(paths, topk, entry, sample, codebook)[0] for _ in range(args.steps)]
    secs = sum(i["seconds"] for i in infos)
    nq = sum(i["nq"] for i in infos)
    value = nq / secs
    cores = infos[0]["threads"]
    ref_gpu = None if (args.no_cli or world > 1) else reference_gpu(base, queries_all, cfg)
    line = {
        "impl": "reference",
        "metric": "QPS at recall@10>=0.95",
        "value": round(value, 1),
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * secs / args.steps, 3),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": cfg["data"],
        "config": {"workload": cfg["workload"], "mode": f"cpu {_ref_class(codebook)}", "K": K,
                   "topk_size": topk, "sample_per_step": sample},
        "cpu_baseline": {"value": round(value, 1), "unit": "queries/s", "cores": cores, "kind": "reference",
                         "sample": f"first {sample} queries per step"},
        "e2e": {"value": round(value, 1), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    return line


# modes and beams of the reference gpu_cli timed beside its CPU search: topk 64
# is its smallest power-of-two beam at recall@10 >= 0.95 on C2 (its
# non-power-of-two beams return recall 0), warp2 its fastest mode there
REF_GPU_RUNS = (("warp2", 64), ("warp4", 64), ("warp1", 64), ("base", 64))


def reference_gpu(base, queries, cfg):
    """The reference's own GPU search (its gpu_cli compiled for sm_100a into
    oracle/_ref/gpu_cli from the reference sources) on the workload's files,
    with its own timing; None when it does not apply.  Only K <= degree is
    run: above it the reference's final flush writes K distances into a
    degree-sized shared-memory buffer (include/gpu_search_warp.cuh:237,
    include/gpu_search_base.cuh:246), the illegal address it raised at K=100
    on the 960-d workload."""
    cli = os.path.join(ROOT, "oracle", "_ref", "gpu_cli")
    if CFG_NAME != "c2" or cfg["codebook"]:
        return None
    if not os.access(cli, os.X_OK):
        return {"unavailable": "oracle/_ref/gpu_cli was not built (make -C oracle gpu REF=<reference tree>)"}
    import torch
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    graph = os.path.join(DATA_DIR, cfg.get("data_dir", CFG_NAME), "graph.bin")
    # exact top-10 for the CLI's recall line: float64 on the GPU (harness code,
    # exact for these integer-valued rows)
    bt = torch.from_numpy(base).cuda()
    gt = gpu_ground_truth(bt, torch.from_numpy(queries[:NQ_PER_GPU]).cuda(), K)
    del bt
    torch.cuda.empty_cache()
    with tempfile.TemporaryDirectory() as tmp:
        data = write_cli_files(tmp, base, queries[:NQ_PER_GPU], gt, graph)
        runs = [run_cli(cli, data, m, t) for m, t in REF_GPU_RUNS]
    ok = [r for r in runs if r["rc"] == 0 and r["qps"] and (r["recall@10"] or 0) >= TARGET_RECALL]
    best = max(ok, key=lambda r: r["qps"]) if ok else None
    return {"binary": "oracle/_ref/gpu_cli (the reference src/gpu_cli.cu, nvcc -arch sm_100a)", "runs": runs,
            "best_at_recall_0.95": best, "queries": NQ_PER_GPU,
            "timing": "the CLI's own: wall clock, mean of 5 searches of all queries, queries on the device "
                      "(reference src/gpu_cli.cu:153-165)"}


def profile_run(args):
    """Minimal launch sequence for an ncu capture of the search kernel on the
    workload's full size: entry-point kernels, `warmup` searches, one search."""
    import torch
    import beam_search_collab_b200 as B
    if args.measure == "codebook":
        # the builder's kernels: `warmup` builds and one more
        from beam_search_collab_b200 import datasets as ds
        s = getattr(ds, CONFIGS[CFG_NAME]["gen"])(nq=1, **CONFIGS[CFG_NAME].get("gen_kwargs", {}))
        ix = B.Index.from_arrays(s.base, ds.read_graph(os.path.join(DATA_DIR, CONFIGS[CFG_NAME].get("data_dir", CFG_NAME), "graph.bin")))
        for _ in range(args.warmup + 1):
            ix.build_codebook(12345)
        torch.cuda.synchronize()
        log("profile run done")
        return
    if args.measure == "graph":
        # the graph builder's kernels: `warmup` builds and one more (the
        # builder's reference settings)
        from beam_search_collab_b200 import datasets as ds
        s = getattr(ds, CONFIGS[CFG_NAME]["gen"])(nq=1, **CONFIGS[CFG_NAME].get("gen_kwargs", {}))
        for _ in range(args.warmup + 1):
            gx = B.Index.from_vectors(s.base, 32)
            gx.build_graph(beam_width=128, alpha=2.0, seed=1234)
            gx.close()
        torch.cuda.synchronize()
        log("profile run done")
        return
    base, queries, edges, codebook = config_data(CFG_NAME, NQ_PER_GPU)
    ix = B.Index.from_arrays(base, edges)
    if args.measure == "ground_truth":
        # the exact brute force (bs_ground_truth): `warmup` runs and one more
        q = torch.from_numpy(queries).cuda()
        for _ in range(args.warmup + 1):
            ix.ground_truth(q, 10, with_dists=False)
        torch.cuda.synchronize()
        log("profile run done")
        return
    if codebook:
        ix.load_codebook(codebook)
    ix.entry_point()
    q = torch.from_numpy(queries).cuda()
    params = B.SearchParams(mode=args.mode, K=K, topk_size=args.topk or 32)
    for _ in range(args.warmup + 1):
        ix.search(q, params)
    torch.cuda.synchronize()
    log("profile run done")


def measure_codebook(args):
    """--measure codebook: the GPU codebook builder (bs_index_build_codebook)
    over the workload's base and graph.  value = edges quantized per second,
    device time of the whole call (medoid, sign table upload, quantization,
    buffers) with CUDA events, L2 flushed before each step; e2e = the drop-in
    CLI bin/build_rabitq end to end (read files, upload, build, write
    codebook.bin), wall clock; cpu_baseline = the reference build_rabitq on
    the same files with all host threads, wall clock; `identical` = the two
    files compared byte for byte."""
    import filecmp
    import torch
    import beam_search_collab_b200 as B
    from beam_search_collab_b200 import datasets as ds
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    s = getattr(ds, CONFIGS[CFG_NAME]["gen"])(nq=1, **CONFIGS[CFG_NAME].get("gen_kwargs", {}))
    graph = os.path.join(DATA_DIR, CONFIGS[CFG_NAME].get("data_dir", CFG_NAME), "graph.bin")
    ix = B.Index.from_arrays(s.base, ds.read_graph(graph))
    n, dim, deg = ix.info()
    for _ in range(args.warmup):
        ix.build_codebook(12345)
    torch.cuda.synchronize()
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    times = []
    for _ in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ix.build_codebook(12345)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    entry = ix.rabitq_entry()
    ix.close()
    edges = n * deg
    with tempfile.TemporaryDirectory() as tmp:
        bp = os.path.join(tmp, "base.fvecs")
        ds.write_fvecs(bp, s.base)
        ours, ref = os.path.join(tmp, "ours.bin"), os.path.join(tmp, "ref.bin")
        t = time.perf_counter()
        subprocess.run([os.path.join(ROOT, "beam_search_collab_b200", "bin", "build_rabitq"), "-base", bp, "-graph",
                        graph, "-out", ours, "-seed", "12345"], check=True, stdout=subprocess.DEVNULL)
        e2e_s = time.perf_counter() - t
        tool = O.ref_tool("build_rabitq")
        ref_s, identical = None, None
        if tool is not None:
            t = time.perf_counter()
            subprocess.run([tool, "-base", bp, "-graph", graph, "-out", ref, "-seed", "12345"], check=True,
                           stdout=subprocess.DEVNULL)
            ref_s = time.perf_counter() - t
            identical = filecmp.cmp(ours, ref, shallow=False)
        file_bytes = os.path.getsize(ours)
    return {
        "metric": "codebook_build_edges_per_s", "value": round(edges / (ms / 1e3)), "unit": "edges/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "f32",
        "data": CONFIGS[CFG_NAME]["data"],
        "config": {"workload": f"RaBitQ codebook of {CFG_NAME}: {n} nodes x {deg} edges, dim {dim}, seed 12345",
                   "l2": "flushed (256 MiB write) before every timed step", "medoid_entry": entry},
        "e2e": {"value": round(edges / e2e_s), "unit": "edges/s", "seconds": round(e2e_s, 3),
                "file_bytes": file_bytes, "h2d_bytes_per_step": None, "d2h_bytes_per_step": file_bytes},
        "cpu_baseline": {"value": round(edges / ref_s) if ref_s else None, "unit": "edges/s",
                         "seconds": round(ref_s, 3) if ref_s else None, "cores": os.cpu_count(),
                         "kind": "reference",
                         "sample": "the whole build, reference build_rabitq (oracle/_ref) under OpenMP on all "
                                   "host threads, wall clock incl. its file reads and codebook write"},
        "identical": identical,
    }


def run_sharded(args, rank, world, local_rank):
    """--sharded: the C5 shape.  The index is cut into `world` shards of
    --shard-rows rows (C5: 8 x 12,500,000 of a 100M-row base), one per GPU;
    each rank draws its own rows, builds its shard's graph (GPU graph builder,
    the reference build_graph's algorithm and file) and RaBitQ codebook (GPU
    build_rabitq, seed 12345) on its own GPU.  A step searches every query on
    every shard (rabitq, K 10, topk 256), all-gathers the shards' lists over
    NCCL and merges them on the GPU into global ids (bs_merge_shards); value =
    queries / max-over-ranks step time.  Checks: the merged rows against the
    merge of the reference's own CPU search run on every shard's files (a
    sample), and recall@10 against the exact top-10 over all shards."""
    import torch
    import torch.distributed as dist
    import beam_search_collab_b200 as B
    from beam_search_collab_b200 import datasets as ds
    from beam_search_collab_b200.sharded import gather_shard_results
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    rows, nq, K_, topk = args.shard_rows, args.sharded_nq, 10, args.topk or 256
    t0 = time.time()
    s = ds.gen_c5_shard(rank, rows, nq)
    t_data = time.time() - t0
    ix = B.Index.from_vectors(s.base, 32, device=local_rank)
    torch.cuda.synchronize()
    t0 = time.time()
    edges = ix.build_graph(beam_width=128, alpha=2.0, seed=1234)
    t_graph = time.time() - t0
    t0 = time.time()
    entry = ix.build_codebook(12345)
    t_cb = time.time() - t0
    log(f"[rank {rank}] shard of {rows} rows: data {t_data:.1f}s, graph {t_graph:.1f}s, codebook {t_cb:.2f}s")
    offsets = [r * rows for r in range(world)]
    q = torch.from_numpy(s.queries).to(dev)
    params = B.SearchParams(mode="rabitq", K=K_, topk_size=topk)
    ids = torch.empty((nq, K_), dtype=torch.int32, device=dev)
    dists = torch.empty((nq, K_), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step():
        ix.search_raw(q.data_ptr(), nq, ids.data_ptr(), dists.data_ptr(), params, stream=stream.cuda_stream)
        with torch.cuda.stream(stream):
            if world > 1:
                ids_all, d_all = gather_shard_results(ids, dists)
            else:
                ids_all, d_all = ids.unsqueeze(0).contiguous(), dists.unsqueeze(0).contiguous()
            return B.merge_shards(d_all, ids_all, offsets, K_, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            ev[i][0].record(stream)
            out_ids, out_d = step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    errs = ix.take_errors(stream.cuda_stream)
    # the search alone (its share of the step)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    ix.search_raw(q.data_ptr(), nq, ids.data_ptr(), dists.data_ptr(), params, stream=stream.cuda_stream)
    b.record(stream)
    torch.cuda.synchronize()
    search_ms = a.elapsed_time(b)
    t = torch.tensor([ms, search_ms, float(errs)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, search_ms, errs = float(t[0]), float(t[1]), int(t[2])
    if errs:
        raise SystemExit(f"search kernels reported error flags {errs:#x}")
    merged = out_ids.cpu().numpy().view(np.uint32)

    # exact top-10 over all shards for a sample (each rank its shard's top-10, merged)
    ns = min(args.cpu_sample, nq)
    gt_i, gt_d = ix.ground_truth(q[:ns], 10)
    torch.cuda.synchronize()
    gt_local = gt_i.cpu().numpy().view(np.uint32).astype(np.int64)
    qs = s.queries[:ns].astype(np.float64)
    gd = gt_d.cpu().numpy().astype(np.float64)
    gi = torch.from_numpy((gt_local + offsets[rank]).astype(np.int64)).to(dev)
    gdt = torch.from_numpy(gd).to(dev)
    if world > 1:
        gi_all = [torch.empty_like(gi) for _ in range(world)]
        gd_all = [torch.empty_like(gdt) for _ in range(world)]
        dist.all_gather(gi_all, gi)
        dist.all_gather(gd_all, gdt)
        gi_all = torch.cat(gi_all, 1).cpu().numpy()
        gd_all = torch.cat(gd_all, 1).cpu().numpy()
    else:
        gi_all, gd_all = gi.cpu().numpy(), gdt.cpu().numpy()
    gt = np.stack([gi_all[i][np.lexsort((gi_all[i], gd_all[i]))][:10] for i in range(ns)])
    recall = recall_at_k(merged[:ns].astype(np.int64), gt)

    # parity: the reference CPU search on this shard's files, then the same merge
    parity = None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    # (the reference tools need the shard's base, graph and codebook as files:
    # about 5 GB a million rows, so only for shards of up to 2M rows)
    if O.ref_tool("ref_search_omp") is not None and not args.no_cpu_baseline and rows <= 2_000_000:
        with tempfile.TemporaryDirectory() as tmp:
            bp, qp, gp, cp = (os.path.join(tmp, f) for f in ("b.fvecs", "q.fvecs", "g.bin", "cb.bin"))
            ds.write_fvecs(bp, s.base)
            ds.write_fvecs(qp, s.queries[:ns])
            with open(gp, "wb") as f:
                np.array([rows, 32], dtype=np.int32).tofile(f)
                edges.tofile(f)
            ix.build_codebook(12345, cp)
            info, ref_local = O.run_ref_search(gp, bp, qp, K=K_, topk=topk, mode="rabitq", codebook=cp,
                                               threads=host_threads(), nq=ns, out=os.path.join(tmp, "ids.u32"))
        rd = np.full(ref_local.shape, np.inf)
        for i in range(ns):
            ok = ref_local[i] != 0xFFFFFFFF
            rd[i, ok] = ((s.base[ref_local[i][ok]].astype(np.float64) - qs[i]) ** 2).sum(1)
        rg = np.where(ref_local != 0xFFFFFFFF, ref_local.astype(np.int64) + offsets[rank], -1)
        rgt, rdt = torch.from_numpy(rg).to(dev), torch.from_numpy(rd).to(dev)
        if world > 1:
            ra = [torch.empty_like(rgt) for _ in range(world)]
            rda = [torch.empty_like(rdt) for _ in range(world)]
            dist.all_gather(ra, rgt)
            dist.all_gather(rda, rdt)
            ra, rda = torch.cat(ra, 1).cpu().numpy(), torch.cat(rda, 1).cpu().numpy()
        else:
            ra, rda = rgt.cpu().numpy(), rdt.cpu().numpy()
        ref_merged = np.stack([ra[i][np.lexsort((ra[i], rda[i]))][:K_] for i in range(ns)])
        same = (merged[:ns].astype(np.int64) == ref_merged).all(axis=1)
        parity = {"queries": ns, "identical_rows": round(float(same.mean()), 6),
                  "ids_match_frac": round(float((merged[:ns].astype(np.int64) == ref_merged).mean()), 6),
                  "recall@10_reference": round(recall_at_k(ref_merged, gt), 5),
                  "against": "the reference's own CPU RaBitQ search (oracle/_ref/ref_search_omp) on every shard's "
                             "graph and codebook files, merged by (distance, global id)"}
    if rank != 0:
        return None
    return {
        "metric": "QPS (C5 sharded index, every query on every shard)",
        "value": round(nq / (ms / 1e3), 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak (index rows per GPU fixed)", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic: seeded C5 mixture (4,096 Gaussians, ints 0..255), each shard drawn by its rank; graphs "
                "and codebooks built on the GPUs with the reference algorithms",
        "config": {"workload": f"C5 shape: {world} shard(s) x {rows} rows x 128, {nq} queries, rabitq K {K_} "
                               f"topk {topk}, NCCL all-gather + GPU merge",
                   "index_rows": world * rows, "recall@10": round(recall, 5), "recall_sample": ns,
                   "search_ms_max_rank": round(search_ms, 4),
                   "exchange_and_merge_share": round(max(0.0, ms - search_ms) / ms, 4),
                   "graph_build_s_rank0": round(t_graph, 2), "codebook_build_s_rank0": round(t_cb, 3),
                   "parallelism": f"index-sharded over {world} GPU(s)"},
        "parity": parity,
        "gpu_launches": args.steps * 2,
        "clocks": clk.summary(),
    }


def run_replicated(args, rank, world, local_rank):
    """--replicated: the C5 companion run.  A 10M-row index of the C5
    distribution (one draw, the same on every rank) is built on every GPU
    (GPU graph builder and codebook builder, the reference algorithms and
    seeds: the same graph on every rank, checked by a checksum), and the
    100,000 queries are split over the ranks (contiguous ranges; rabitq, K 10,
    topk 256).  value = all queries / max-over-ranks step time (strong
    scaling: the job is fixed); e2e = the same with page-locked host query and
    result buffers.  recall@10 on a sample of rank 0's queries against the
    exact top-10 (bs_ground_truth)."""
    import torch
    import torch.distributed as dist
    import beam_search_collab_b200 as B
    from beam_search_collab_b200 import datasets as ds
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    rows, nq, K_, topk = args.replicated_rows, args.sharded_nq, 10, args.topk or 256
    t0 = time.time()
    s = ds.gen_c5_shard(0, rows, nq)
    t_data = time.time() - t0
    ix = B.Index.from_vectors(s.base, 32, device=local_rank)
    t0 = time.time()
    edges = ix.build_graph(beam_width=128, alpha=2.0, seed=1234)
    t_graph = time.time() - t0
    ix.build_codebook(12345)
    torch.cuda.synchronize()
    csum = int(np.bitwise_xor.reduce((edges.astype(np.uint64) * np.uint64(2654435761)).ravel() ^
                                     np.arange(edges.size, dtype=np.uint64)) & np.uint64((1 << 62) - 1))
    same_graph = True
    if world > 1:
        t = torch.tensor([csum], dtype=torch.int64, device=dev)
        ts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(ts, t)
        same_graph = all(int(x) == csum for x in ts)
    log(f"[rank {rank}] replicated index of {rows} rows: data {t_data:.1f}s, graph {t_graph:.1f}s")
    q0, q1 = rank * nq // world, (rank + 1) * nq // world
    mine = np.ascontiguousarray(s.queries[q0:q1])
    n_mine = len(mine)
    q = torch.from_numpy(mine).to(dev)
    params = B.SearchParams(mode="rabitq", K=K_, topk_size=topk)
    ids = torch.empty((n_mine, K_), dtype=torch.int32, device=dev)
    dists = torch.empty((n_mine, K_), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step(qp, ip, dp):
        ix.search_raw(qp, n_mine, ip, dp, params, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step(q.data_ptr(), ids.data_ptr(), dists.data_ptr())
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.zero_()
                ev[i][0].record(stream)
                step(q.data_ptr(), ids.data_ptr(), dists.data_ptr())
                ev[i][1].record(stream)
        torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    errs = ix.take_errors(stream.cuda_stream)
    # e2e: page-locked host buffers through the same call
    hq = torch.from_numpy(mine).pin_memory()
    hid = torch.empty((n_mine, K_), dtype=torch.int32).pin_memory()
    hd = torch.empty((n_mine, K_), dtype=torch.float32).pin_memory()
    step(hq.data_ptr(), hid.data_ptr(), hd.data_ptr())
    torch.cuda.synchronize()
    ee = []
    for _ in range(max(3, min(args.steps, 5))):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step(hq.data_ptr(), hid.data_ptr(), hd.data_ptr())
        b.record(stream)
        b.synchronize()
        ee.append(a.elapsed_time(b))
    e2e_ms = statistics.mean(ee)
    errs |= ix.take_errors(stream.cuda_stream)
    assert np.array_equal(hid.numpy(), ids.cpu().numpy()), "host-buffer results differ"
    t = torch.tensor([ms, e2e_ms, float(errs)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms, e2e_ms, errs = float(t[0]), float(t[1]), int(t[2])
    if errs:
        raise SystemExit(f"search kernels reported error flags {errs:#x}")
    if rank != 0:
        return None
    ns = min(args.cpu_sample, n_mine)
    gt_i, _ = ix.ground_truth(q[:ns], 10, with_dists=False)
    torch.cuda.synchronize()
    recall = recall_at_k(ids[:ns].cpu().numpy().view(np.uint32).astype(np.int64),
                         gt_i.cpu().numpy().view(np.uint32).astype(np.int64))
    return {
        "metric": "QPS (C5-10M replicated index, queries split over the GPUs)",
        "value": round(nq / (ms / 1e3), 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic: seeded C5 mixture (4,096 Gaussians, ints 0..255), one draw of "
                f"{rows} rows; graph and codebook built on every GPU with the reference algorithms",
        "config": {"workload": f"C5-10M: {rows} x 128 replicated on {world} GPU(s), {nq} queries split over them, "
                               f"rabitq K {K_} topk {topk}",
                   "queries_per_gpu": n_mine, "recall@10": round(recall, 5), "recall_sample": ns,
                   "graph_build_s": round(t_graph, 2), "graph_identical_on_all_ranks": same_graph,
                   "l2": "256 MiB write before every timed step (outside the timed window)",
                   "parallelism": f"query-sharded dp{world}, replicated index"},
        "e2e": {"value": round(nq / (e2e_ms / 1e3), 1), "unit": "queries/s",
                "h2d_bytes_per_step": int(nq * 128 * 4), "d2h_bytes_per_step": int(nq * K_ * 8)},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }


def measure_graph(args):
    """--measure graph: the GPU graph builder (bs_index_build_graph) over the
    workload's base, against the graph the reference build_graph wrote for it
    (bench_data/<config>/graph.bin, --degree 32 --beam-width 128 --alpha 2.0
    --seed 1234).  value = inserted nodes per second, device time of the whole
    build (CUDA events; the upload is outside); e2e = the drop-in CLI
    bin/build_graph end to end (read the fvecs, upload, build, write
    graph.bin), wall clock; cpu_baseline = the reference build_graph on the
    same file with all host threads, wall clock (skipped with
    --no-cpu-baseline); `identical` = the files compared byte for byte."""
    import filecmp
    import torch
    import beam_search_collab_b200 as B
    from beam_search_collab_b200 import datasets as ds
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cfg = CONFIGS[CFG_NAME]
    s = getattr(ds, cfg["gen"])(nq=1, **cfg.get("gen_kwargs", {}))
    ref_graph = os.path.join(DATA_DIR, cfg.get("data_dir", CFG_NAME), "graph.bin")
    ref_edges = ds.read_graph(ref_graph)
    degree = ref_edges.shape[1]
    times, same = [], None
    for i in range(max(1, args.steps)):
        ix = B.Index.from_vectors(s.base, degree)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        edges = ix.build_graph(beam_width=128, alpha=2.0, seed=1234)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
        ix.close()
        rows_same = (edges == ref_edges).all(axis=1)
        same = int(rows_same.sum()) if same is None else min(same, int(rows_same.sum()))
    ms = statistics.median(times)
    n = s.base.shape[0]
    with tempfile.TemporaryDirectory() as tmp:
        bp, gp, rp = os.path.join(tmp, "base.fvecs"), os.path.join(tmp, "ours.bin"), os.path.join(tmp, "ref.bin")
        ds.write_fvecs(bp, s.base)
        t = time.perf_counter()
        subprocess.run([os.path.join(ROOT, "beam_search_collab_b200", "bin", "build_graph"), "--base", bp, "--graph", gp,
                        "--degree", str(degree), "--beam-width", "128", "--alpha", "2.0", "--seed", "1234"],
                       check=True, stdout=subprocess.DEVNULL)
        e2e_s = time.perf_counter() - t
        identical = filecmp.cmp(gp, ref_graph, shallow=False)
        ref_s = None
        tool = O.ref_tool("build_graph")
        if tool is not None and not args.no_cpu_baseline:
            t = time.perf_counter()
            subprocess.run([tool, "--base", bp, "--graph", rp, "--degree", str(degree), "--beam-width", "128",
                            "--alpha", "2.0", "--seed", "1234"], check=True, stdout=subprocess.DEVNULL,
                           env=dict(os.environ, OMP_NUM_THREADS=str(host_threads())))
            ref_s = time.perf_counter() - t
    return {
        "metric": "graph_build_nodes_per_s", "value": round(n / (ms / 1e3)), "unit": "nodes/s",
        "n_gpus": 1, "steps": len(times), "warmup": 0, "ms_per_step": round(ms, 2),
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "u8" if s.base.max() <= 255 and
        np.array_equal(s.base, np.rint(s.base)) and s.base.min() >= 0 else "f32",
        "data": cfg["data"],
        "config": {"workload": f"Vamana graph of {CFG_NAME}: {n} x {s.base.shape[1]}, degree {degree}, beam 128, "
                               "alpha 2.0, seed 1234", "rows_identical_to_reference": same, "rows": n},
        "e2e": {"value": round(n / e2e_s), "unit": "nodes/s", "seconds": round(e2e_s, 2),
                "h2d_bytes_per_step": int(s.base.nbytes), "d2h_bytes_per_step": int(ref_edges.nbytes)},
        "cpu_baseline": {"value": round(n / ref_s) if ref_s else None, "unit": "nodes/s",
                         "seconds": round(ref_s, 2) if ref_s else None, "cores": host_threads(), "kind": "reference",
                         "sample": "the whole build, reference build_graph (oracle/_ref) under OpenMP on all host "
                                   "threads, wall clock incl. its file read and write"},
        "identical": identical,
    }


# -------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2",
                    help="workload (the driver's bench line is c2)")
    ap.add_argument("--mode", default=None, help="search mode (default: the workload's)")
    ap.add_argument("--topk", type=int, default=0, help="fixed topk_size (0: sweep to the recall target)")
    ap.add_argument("--cpu-sample", type=int, default=2000)
    ap.add_argument("--ref-sample", type=int, default=1000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cli", action="store_true",
                    help="skip the gpu_cli runs (ours in our arm, the reference's in the reference arm)")
    ap.add_argument("--sharded", action="store_true",
                    help="C5 shape: an index sharded over the GPUs (see run_sharded)")
    ap.add_argument("--shard-rows", type=int, default=12_500_000)
    ap.add_argument("--replicated", action="store_true",
                    help="C5-10M: one index replicated on every GPU, the queries split over them")
    ap.add_argument("--replicated-rows", type=int, default=10_000_000)
    ap.add_argument("--sharded-nq", type=int, default=100_000)
    ap.add_argument("--scaling", choices=("weak", "strong"), default="weak",
                    help="weak: every GPU searches its own 10,000 queries; strong: the workload's 10,000 "
                         "queries split over the GPUs")
    ap.add_argument("--measure", choices=("search", "codebook", "graph", "ground_truth"), default="search",
                    help="codebook / graph: time the GPU codebook or graph builder instead of the search")
    ap.add_argument("--profile-run", action="store_true",
                    help="for ncu: build the index, run `--warmup` searches and one more, print nothing else")
    args = ap.parse_args()
    global CFG_NAME, K, NQ_PER_GPU
    CFG_NAME = args.config
    K = CONFIGS[CFG_NAME]["K"]
    NQ_PER_GPU = CONFIGS[CFG_NAME]["nq"]
    args.mode = args.mode or CONFIGS[CFG_NAME]["mode"]
    if args.profile_run:
        profile_run(args)
        return None, 0
    args.warmup = max(args.warmup, 3)
    if args.measure == "codebook":
        return measure_codebook(args), 0
    if args.measure == "graph":
        return measure_graph(args), 0

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=torch.device("cuda", local_rank))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    elif args.sharded:
        line = run_sharded(args, rank, world, local_rank)
    elif args.replicated:
        line = run_replicated(args, rank, world, local_rank)
    else:
        line = run_ours(args, rank, world, local_rank)
    if world > 1 and args.impl == "ours":
        import torch
        torch.distributed.destroy_process_group()
    return line, rank


if __name__ == "__main__":
    # stdout carries exactly one JSON line: while the run goes, file
    # descriptor 1 points at stderr (libraries such as NCCL print to stdout)
    sys.stdout.flush()
    _stdout_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        _line, _rank = main()
    finally:
        sys.stdout.flush()
        os.dup2(_stdout_fd, 1)
        os.close(_stdout_fd)
    if _rank == 0 and _line is not None:
        print(json.dumps(_line), flush=True)
