"""ctypes front end of the CPU oracle (oracle/liboracle.so) and runners for the
reference's own CPU tools compiled into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and the
benchmark's CPU-baseline leg, never by the product package.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_u32p = ctypes.POINTER(ctypes.c_uint32)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class OrcStats(ctypes.Structure):
    _fields_ = [("expansions", ctypes.c_uint64), ("distances", ctypes.c_uint64),
                ("estimates", ctypes.c_uint64), ("rerank", ctypes.c_uint64)]


class OrcBatchCfg(ctypes.Structure):
    _fields_ = [("base", _f32p), ("n", ctypes.c_uint64), ("dim", ctypes.c_int),
                ("edges", _u32p), ("degree", ctypes.c_int),
                ("codes", _u32p), ("factors", _f32p), ("signs", _f32p), ("pdim", ctypes.c_int),
                ("topk_size", ctypes.c_int), ("entry", ctypes.c_uint32),
                ("max_iterations", ctypes.c_int), ("K", ctypes.c_int),
                ("filter_bits", ctypes.c_uint32), ("reset_interval", ctypes.c_int),
                ("mode", ctypes.c_int)]


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_entry_point.restype = ctypes.c_uint32
        L.orc_entry_point.argtypes = [_f32p, ctypes.c_uint64, ctypes.c_int]
        L.orc_l2.restype = ctypes.c_float
        L.orc_l2.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.orc_rabitq_quantize.restype = None
        L.orc_rabitq_quantize.argtypes = [_f32p, ctypes.c_int, _f32p, ctypes.c_int, _u8p,
                                          _f32p, _f32p, _i32p]
        L.orc_rabitq_raw.restype = ctypes.c_uint32
        L.orc_rabitq_raw.argtypes = [_u8p, _u32p, ctypes.c_int]
        L.orc_search_batch.restype = ctypes.c_int
        L.orc_search_batch.argtypes = [ctypes.POINTER(OrcBatchCfg), _f32p, ctypes.c_uint64,
                                       _u32p, _f32p, ctypes.POINTER(OrcStats), ctypes.c_int]
        L.orc_recall_cpu.restype = ctypes.c_double
        L.orc_recall_cpu.argtypes = [_u32p, _i32p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        L.orc_recall_gpu.restype = ctypes.c_double
        L.orc_recall_gpu.argtypes = [_u32p, _i32p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_uint64)]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def entry_point(base: np.ndarray) -> int:
    base = np.ascontiguousarray(base, dtype=np.float32)
    return int(lib().orc_entry_point(_p(base, _f32p), base.shape[0], base.shape[1]))


@dataclass
class OracleResult:
    ids: np.ndarray
    dists: np.ndarray
    stats: OrcStats


def search(base, edges, queries, *, K, topk_size, entry, max_iterations=1024, mode="base",
           filter_bits=1024, reset_interval=16, codebook=None, threads=None) -> OracleResult:
    """mode: 'base' (cpu_cli base == warpN/base GPU semantics), 'bloom'
    (bwarpN semantics) or 'rabitq' (cpu_cli rabitq; needs codebook)."""
    base = np.ascontiguousarray(base, dtype=np.float32)
    edges = np.ascontiguousarray(edges, dtype=np.uint32)
    queries = np.ascontiguousarray(queries, dtype=np.float32)
    nq = queries.shape[0]
    cfg = OrcBatchCfg()
    cfg.base = _p(base, _f32p)
    cfg.n = base.shape[0]
    cfg.dim = base.shape[1]
    cfg.edges = _p(edges, _u32p)
    cfg.degree = edges.shape[1]
    keep = []
    if mode == "rabitq":
        codes = np.ascontiguousarray(codebook.codes, dtype=np.uint32)
        factors = np.ascontiguousarray(codebook.factors, dtype=np.float32)
        signs = np.ascontiguousarray(codebook.signs, dtype=np.float32)
        keep += [codes, factors, signs]
        cfg.codes = _p(codes, _u32p)
        cfg.factors = _p(factors, _f32p)
        cfg.signs = _p(signs, _f32p)
        cfg.pdim = codebook.pdim
    cfg.topk_size = topk_size
    cfg.entry = entry
    cfg.max_iterations = max_iterations
    cfg.K = K
    cfg.filter_bits = filter_bits
    cfg.reset_interval = reset_interval
    cfg.mode = {"base": 0, "bloom": 1, "rabitq": 2}[mode]
    ids = np.empty((nq, K), dtype=np.uint32)
    dists = np.empty((nq, K), dtype=np.float32)
    st = OrcStats()
    if threads is None:
        threads = os.cpu_count() or 1
    rc = lib().orc_search_batch(ctypes.byref(cfg), _p(queries, _f32p), nq, _p(ids, _u32p),
                                _p(dists, _f32p), ctypes.byref(st), threads)
    if rc != 0:
        raise RuntimeError(f"oracle search failed ({rc})")
    return OracleResult(ids, dists, st)


def quantize(query, signs, pdim):
    query = np.ascontiguousarray(query, dtype=np.float32)
    signs = np.ascontiguousarray(signs, dtype=np.float32)
    q = np.empty(pdim, dtype=np.uint8)
    low, w, s = ctypes.c_float(), ctypes.c_float(), ctypes.c_int32()
    lib().orc_rabitq_quantize(_p(query, _f32p), query.shape[0], _p(signs, _f32p), pdim,
                              _p(q, _u8p), ctypes.byref(low), ctypes.byref(w), ctypes.byref(s))
    return q, low.value, w.value, s.value


def recall_cpu(pred, gt, K):
    pred = np.ascontiguousarray(pred, dtype=np.uint32)
    gt = np.ascontiguousarray(gt, dtype=np.int32)
    return lib().orc_recall_cpu(_p(pred, _u32p), _p(gt, _i32p), pred.shape[0], K, gt.shape[1])


def recall_gpu(pred, gt, K):
    pred = np.ascontiguousarray(pred, dtype=np.uint32)
    gt = np.ascontiguousarray(gt, dtype=np.int32)
    d = ctypes.c_uint64()
    r = lib().orc_recall_gpu(_p(pred, _u32p), _p(gt, _i32p), pred.shape[0], K, gt.shape[1],
                             ctypes.byref(d))
    return r, d.value


# ------------------------------------------------ reference tools (oracle/_ref)

def ref_tool(name: str) -> str | None:
    p = os.path.join(REF_DIR, name)
    return p if os.access(p, os.X_OK) else None


def run_ref_search(graph, base, query, *, K, topk, mode="base", codebook=None, max_iter=1024,
                   threads=None, nq=None, entry=None, out=None):
    """Runs oracle/_ref/ref_search_omp (the reference's own CPUBaseSearch /
    CPURabitqSearch classes under OpenMP).  Returns (json_info, ids or None)."""
    exe = ref_tool("ref_search_omp")
    if exe is None:
        raise FileNotFoundError("oracle/_ref/ref_search_omp not built")
    cmd = [exe, "--graph", graph, "--base", base, "--query", query, "--mode", mode,
           "--K", str(K), "--topk", str(topk), "--max-iter", str(max_iter)]
    if codebook:
        cmd += ["--codebook", codebook]
    if threads:
        cmd += ["--threads", str(threads)]
    if nq is not None:
        cmd += ["--nq", str(nq)]
    if entry is not None:
        cmd += ["--entry", str(entry)]
    if out:
        cmd += ["--out", out]
    r = subprocess.run(cmd, check=True, capture_output=True, text=True)
    info = json.loads(r.stdout.strip().splitlines()[-1])
    ids = None
    if out:
        ids = np.fromfile(out, dtype=np.uint32).reshape(info["nq"], K)
    return info, ids


def run_cpu_cli(config: dict) -> str:
    """Runs the reference cpu_cli as shipped with a JSON config on stdin and
    returns its stdout."""
    exe = ref_tool("cpu_cli")
    if exe is None:
        raise FileNotFoundError("oracle/_ref/cpu_cli not built")
    r = subprocess.run([exe], input=json.dumps(config), check=True, capture_output=True, text=True)
    return r.stdout
