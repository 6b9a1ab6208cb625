"""B200-native graph ANN beam search with the drop-in surface of
SophiaSun18/beam_search_collab.

The product is native: ``lib/libbsearch_b200.so`` (hand-written sm_100a CUDA
behind the C ABI of ``include/bsearch.h``) and ``bin/gpu_cli`` (the reference
``gpu_cli`` JSON-on-stdin CLI).  This module is a thin ctypes binding of that
ABI for Python callers (tests, benchmark).  It never falls back to a CPU
path: if the library is missing, importing :func:`lib` raises.

    from beam_search_collab_b200 import Index
    ix = Index.load("graph.bin", "base.fvecs")
    ids, dists, stats = ix.search(queries, mode="warp4", K=10, topk_size=64)
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
from dataclasses import dataclass

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libbsearch_b200.so")
CLI_PATH = os.path.join(PKG, "bin", "gpu_cli")
NO_NODE = 0xFFFFFFFF

MODES = ("base", "warp1", "warp2", "warp4", "warp8",
         "bwarp1", "bwarp2", "bwarp4", "bwarp8", "rabitq")

_u32p = ctypes.POINTER(ctypes.c_uint32)
_f32p = ctypes.POINTER(ctypes.c_float)


class BSearchError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"bsearch status {status}: {msg}")
        self.status = status


class _GraphDesc(ctypes.Structure):
    _fields_ = [("num_nodes", ctypes.c_uint64), ("dim", ctypes.c_int32), ("degree", ctypes.c_int32),
                ("vectors", ctypes.c_void_p), ("edges", ctypes.c_void_p)]


class _RabitqDesc(ctypes.Structure):
    _fields_ = [("entry_point", ctypes.c_uint32), ("padded_dim", ctypes.c_int32),
                ("codes", ctypes.c_void_p), ("factors", ctypes.c_void_p), ("signs", ctypes.c_void_p)]


class _BuildParams(ctypes.Structure):
    _fields_ = [("beam_width", ctypes.c_int32), ("alpha", ctypes.c_float), ("seed", ctypes.c_uint32)]


class _Params(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_char_p), ("K", ctypes.c_int32), ("topk_size", ctypes.c_uint32),
                ("filter_capacity", ctypes.c_uint32), ("max_iterations", ctypes.c_int32),
                ("reset_interval", ctypes.c_int32), ("entry_point", ctypes.c_uint32)]


class Stats(ctypes.Structure):
    _fields_ = [("expansions", ctypes.c_uint64), ("distances", ctypes.c_uint64),
                ("estimates", ctypes.c_uint64), ("rerank", ctypes.c_uint64),
                ("error_flags", ctypes.c_uint32), ("entry_point", ctypes.c_uint32),
                ("integer_exact", ctypes.c_uint32), ("row_bytes", ctypes.c_uint32),
                ("block_bytes", ctypes.c_uint32), ("warps_per_query", ctypes.c_uint32)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


# Every symbol include/bsearch.h declares (checked by the CPU test suite).
EXPORTS = ("bs_search_params_default", "bs_index_create", "bs_index_load", "bs_index_attach_rabitq",
           "bs_index_load_codebook", "bs_index_build_codebook", "bs_index_info", "bs_index_entry_point", "bs_index_rabitq_entry",
           "bs_index_build_graph", "bs_ground_truth", "bs_index_prepare", "bs_index_take_errors", "bs_index_destroy", "bs_search", "bs_search_no_alloc", "bs_merge_shards", "bs_device_alloc",
           "bs_device_free",
           "bs_copy_to_device",
           "bs_copy_to_host", "bs_device_fill", "bs_synchronize", "bs_last_error", "bs_version")

_lib = None


def lib() -> ctypes.CDLL:
    """Loads lib/libbsearch_b200.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is missing: run `python -m beam_search_collab_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    vp, st = ctypes.c_void_p, ctypes.c_int
    L.bs_search_params_default.argtypes = [ctypes.POINTER(_Params)]
    L.bs_search_params_default.restype = None
    L.bs_index_create.argtypes = [ctypes.POINTER(_GraphDesc), ctypes.c_int, ctypes.POINTER(vp)]
    L.bs_index_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(vp)]
    L.bs_index_attach_rabitq.argtypes = [vp, ctypes.POINTER(_RabitqDesc)]
    L.bs_index_load_codebook.argtypes = [vp, ctypes.c_char_p]
    L.bs_index_build_codebook.argtypes = [vp, ctypes.c_uint32, ctypes.c_char_p, _u32p]
    L.bs_index_info.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int32),
                                ctypes.POINTER(ctypes.c_int32)]
    L.bs_index_entry_point.argtypes = [vp, _u32p]
    L.bs_index_rabitq_entry.argtypes = [vp, _u32p]
    L.bs_index_take_errors.argtypes = [vp, vp, _u32p]
    L.bs_index_prepare.argtypes = [vp, ctypes.c_char_p]
    L.bs_index_build_graph.argtypes = [vp, ctypes.POINTER(_BuildParams), _u32p]
    L.bs_ground_truth.argtypes = [vp, vp, ctypes.c_uint32, ctypes.c_uint32, vp, vp, vp]
    L.bs_index_destroy.argtypes = [vp]
    L.bs_index_destroy.restype = None
    L.bs_search.argtypes = [vp, ctypes.POINTER(_Params), vp, ctypes.c_uint32, vp, vp,
                            ctypes.POINTER(Stats), vp]
    L.bs_search_no_alloc.argtypes = [vp, ctypes.POINTER(_Params), vp, ctypes.c_uint32, vp, vp, vp]
    L.bs_search_no_alloc.restype = st
    L.bs_merge_shards.argtypes = [vp, vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _u32p,
                                  ctypes.c_uint32, vp, vp, vp]
    L.bs_merge_shards.restype = st
    L.bs_device_alloc.argtypes = [vp, ctypes.c_size_t, ctypes.POINTER(vp)]
    L.bs_device_free.argtypes = [vp, vp]
    L.bs_copy_to_device.argtypes = [vp, vp, vp, ctypes.c_size_t]
    L.bs_copy_to_host.argtypes = [vp, vp, vp, ctypes.c_size_t]
    L.bs_device_fill.argtypes = [vp, vp, ctypes.c_int, ctypes.c_size_t]
    L.bs_synchronize.argtypes = [vp, vp]
    for f in ("bs_index_create", "bs_index_load", "bs_index_attach_rabitq", "bs_index_load_codebook",
              "bs_index_build_codebook",
              "bs_index_info", "bs_index_entry_point", "bs_index_rabitq_entry", "bs_index_take_errors", "bs_index_prepare", "bs_index_build_graph", "bs_ground_truth", "bs_search",
              "bs_device_alloc", "bs_device_free", "bs_copy_to_device", "bs_copy_to_host",
              "bs_device_fill", "bs_synchronize"):
        getattr(L, f).restype = st
    L.bs_last_error.restype = ctypes.c_char_p
    L.bs_last_error.argtypes = []
    L.bs_version.restype = ctypes.c_char_p
    L.bs_version.argtypes = []
    _lib = L
    return L


def _check(status: int) -> None:
    if status != 0:
        raise BSearchError(status, lib().bs_last_error().decode())


def _ptr(a) -> int:
    """Address of a numpy array or a torch tensor (host or device)."""
    if a is None:
        return 0
    if hasattr(a, "data_ptr"):
        return int(a.data_ptr())
    return int(a.ctypes.data)


@dataclass
class SearchParams:
    """The "search" object of the reference JSON config (src/gpu_cli.cu:414-452)."""
    mode: str = "base"
    K: int = 100
    topk_size: int = 256
    filter_capacity: int = 1024
    max_iterations: int = 1024
    reset_interval: int = 16
    entry_point: int = NO_NODE

    def _c(self) -> _Params:
        p = _Params()
        p.mode = self.mode.encode()
        p.K = self.K
        p.topk_size = self.topk_size
        p.filter_capacity = self.filter_capacity
        p.max_iterations = self.max_iterations
        p.reset_interval = self.reset_interval
        p.entry_point = self.entry_point
        return p


class Index:
    """A graph (and optional RaBitQ codebook) resident on one GPU."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)

    # -- construction -----------------------------------------------------
    @classmethod
    def from_arrays(cls, vectors: np.ndarray, edges: np.ndarray, device: int = 0) -> "Index":
        vectors = np.ascontiguousarray(vectors, dtype=np.float32)
        edges = np.ascontiguousarray(edges, dtype=np.uint32)
        if vectors.ndim != 2 or edges.ndim != 2 or vectors.shape[0] != edges.shape[0]:
            raise ValueError("vectors (n, dim) and edges (n, degree) must share n")
        d = _GraphDesc(vectors.shape[0], vectors.shape[1], edges.shape[1], _ptr(vectors), _ptr(edges))
        h = ctypes.c_void_p()
        _check(lib().bs_index_create(ctypes.byref(d), device, ctypes.byref(h)))
        return cls(h.value)

    @classmethod
    def from_vectors(cls, vectors: np.ndarray, degree: int, device: int = 0) -> "Index":
        """An index over `vectors` with no graph yet (for build_graph)."""
        vectors = np.ascontiguousarray(vectors, dtype=np.float32)
        d = _GraphDesc(vectors.shape[0], vectors.shape[1], degree, _ptr(vectors), None)
        h = ctypes.c_void_p()
        _check(lib().bs_index_create(ctypes.byref(d), device, ctypes.byref(h)))
        return cls(h.value)

    def build_graph(self, beam_width: int = 128, alpha: float = 2.0, seed: int = 1234) -> np.ndarray:
        """Builds this index's graph on the GPU with the reference build_graph's
        algorithm (src/build_graph.cpp:255-397); returns the edges [n, degree]."""
        n, _, deg = self.info()
        out = np.empty((n, deg), dtype=np.uint32)
        p = _BuildParams(beam_width, alpha, seed)
        _check(lib().bs_index_build_graph(self._h, ctypes.byref(p), out.ctypes.data_as(_u32p)))
        return out

    @classmethod
    def load(cls, graph_bin: str, base_fvecs: str, device: int = 0) -> "Index":
        h = ctypes.c_void_p()
        _check(lib().bs_index_load(graph_bin.encode(), base_fvecs.encode(), device, ctypes.byref(h)))
        return cls(h.value)

    def attach_rabitq(self, entry: int, padded_dim: int, codes, factors, signs) -> None:
        codes = np.ascontiguousarray(codes, dtype=np.uint32)
        factors = np.ascontiguousarray(factors, dtype=np.float32)
        signs = np.ascontiguousarray(signs, dtype=np.float32)
        d = _RabitqDesc(entry, padded_dim, _ptr(codes), _ptr(factors), _ptr(signs))
        _check(lib().bs_index_attach_rabitq(self._h, ctypes.byref(d)))

    def load_codebook(self, path: str) -> None:
        _check(lib().bs_index_load_codebook(self._h, path.encode()))

    def build_codebook(self, seed: int = 12345, out_path: str | None = None) -> int:
        """Builds the RaBitQ codebook of this index on the GPU (the reference
        build_rabitq rule and arithmetic, src/build_rabitq.cpp:120-285),
        attaches it, optionally writes it as codebook.bin; returns the medoid
        entry point."""
        e = ctypes.c_uint32()
        _check(lib().bs_index_build_codebook(self._h, seed, out_path.encode() if out_path else None,
                                             ctypes.byref(e)))
        return e.value

    def close(self) -> None:
        if self._h and self._h.value:
            lib().bs_index_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- queries -------------------------------------------------------------
    def info(self):
        n, d, g = ctypes.c_uint64(), ctypes.c_int32(), ctypes.c_int32()
        _check(lib().bs_index_info(self._h, ctypes.byref(n), ctypes.byref(d), ctypes.byref(g)))
        return n.value, d.value, g.value

    def entry_point(self) -> int:
        e = ctypes.c_uint32()
        _check(lib().bs_index_entry_point(self._h, ctypes.byref(e)))
        return e.value

    def ground_truth(self, queries, k: int, with_dists: bool = True, stream: int = 0):
        """Exact k nearest rows of each query by brute force (bs_ground_truth):
        (ids, dists) ordered by (distance, id); outputs live where the queries
        live (numpy or a CUDA tensor)."""
        if hasattr(queries, "data_ptr"):
            import torch
            nq = queries.shape[0]
            ids = torch.empty((nq, k), dtype=torch.int32, device=queries.device)
            dists = torch.empty((nq, k), dtype=torch.float32, device=queries.device) if with_dists else None
        else:
            queries = np.ascontiguousarray(queries, dtype=np.float32)
            nq = queries.shape[0]
            ids = np.empty((nq, k), dtype=np.uint32)
            dists = np.empty((nq, k), dtype=np.float32) if with_dists else None
        _check(lib().bs_ground_truth(self._h, ctypes.c_void_p(_ptr(queries)), nq, k, ctypes.c_void_p(_ptr(ids)),
                                     ctypes.c_void_p(_ptr(dists) or None), ctypes.c_void_p(stream or None)))
        return ids, dists

    def prepare(self, mode: str = "warp4") -> None:
        """Builds the device layout `mode` searches on (bs_index_prepare)."""
        _check(lib().bs_index_prepare(self._h, mode.encode()))

    def take_errors(self, stream: int = 0) -> int:
        """Kernel error bits reported by searches on this index since the last
        call (asynchronous ones included), then cleared; 0 = none."""
        f = ctypes.c_uint32()
        _check(lib().bs_index_take_errors(self._h, ctypes.c_void_p(stream or None), ctypes.byref(f)))
        return f.value

    def rabitq_entry(self) -> int:
        e = ctypes.c_uint32()
        _check(lib().bs_index_rabitq_entry(self._h, ctypes.byref(e)))
        return e.value

    def search(self, queries, params: SearchParams | None = None, *, with_dists: bool = True,
               stream: int = 0, **kw):
        """Searches host (numpy) or device (torch CUDA) queries.

        Returns (ids, dists, stats).  Outputs live where the queries live."""
        p = params or SearchParams(**kw)
        if hasattr(queries, "data_ptr"):
            import torch
            nq = queries.shape[0]
            ids = torch.empty((nq, p.K), dtype=torch.int32, device=queries.device)
            dists = torch.empty((nq, p.K), dtype=torch.float32, device=queries.device) if with_dists else None
        else:
            queries = np.ascontiguousarray(queries, dtype=np.float32)
            nq = queries.shape[0]
            ids = np.empty((nq, p.K), dtype=np.uint32)
            dists = np.empty((nq, p.K), dtype=np.float32) if with_dists else None
        st = Stats()
        self.search_raw(_ptr(queries), nq, _ptr(ids), _ptr(dists), p, stats=st, stream=stream)
        return ids, dists, st

    def search_raw(self, queries_ptr: int, nq: int, ids_ptr: int, dists_ptr: int, params: SearchParams,
                   stats: Stats | None = None, stream: int = 0) -> None:
        """bs_search on raw addresses (host or device), on `stream`."""
        c = params._c()
        _check(lib().bs_search(self._h, ctypes.byref(c), ctypes.c_void_p(queries_ptr), nq,
                               ctypes.c_void_p(ids_ptr), ctypes.c_void_p(dists_ptr or None),
                               ctypes.byref(stats) if stats is not None else None,
                               ctypes.c_void_p(stream or None)))


def merge_shards(dists, ids, id_offsets, K_out: int, stream: int = 0):
    """bs_merge_shards on CUDA tensors: dists float32 [S, nq, K], ids int32
    [S, nq, K] (shard-local ids, -1 = none), one id offset per shard.
    Returns (ids [nq, K_out] int32 with global ids, dists [nq, K_out])."""
    import torch
    if not (dists.is_contiguous() and ids.is_contiguous()):
        raise ValueError("merge_shards needs contiguous tensors")
    S, nq, K = ids.shape
    out_ids = torch.empty((nq, K_out), dtype=torch.int32, device=ids.device)
    out_d = torch.empty((nq, K_out), dtype=torch.float32, device=ids.device)
    offs = (ctypes.c_uint32 * S)(*[int(o) for o in id_offsets])
    import contextlib
    with torch.cuda.device(ids.device) if ids.is_cuda else contextlib.nullcontext():
        _check(lib().bs_merge_shards(ctypes.c_void_p(_ptr(dists)), ctypes.c_void_p(_ptr(ids)), S, nq, K, offs,
                                     K_out, ctypes.c_void_p(_ptr(out_ids)), ctypes.c_void_p(_ptr(out_d)),
                                     ctypes.c_void_p(stream or None)))
    return out_ids, out_d


def run_cli(config: dict, timeout: float = 600) -> subprocess.CompletedProcess:
    """Runs bin/gpu_cli with `config` as the JSON on stdin."""
    if not os.path.exists(CLI_PATH):
        raise FileNotFoundError(f"{CLI_PATH} is missing: run `python -m beam_search_collab_b200.build`")
    return subprocess.run([CLI_PATH], input=json.dumps(config), capture_output=True, text=True,
                          timeout=timeout)


def version() -> str:
    return lib().bs_version().decode()
