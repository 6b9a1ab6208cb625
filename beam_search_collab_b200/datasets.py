"""Synthetic stand-ins for the reference's benchmark data, and the reference's
file formats.

The reference benchmarks on SIFT-1M / GIST-1M style sets that are not available
here.  Seeded generators with the shapes and value distributions of each named
configuration stand in for them:

* ``c1``  10,000 x 128 base, 1,000 queries: mixture of 100 isotropic Gaussians,
          centres ~ N(0,1)*4, sigma 1 (CPU plumbing / parity case).
* ``c2``  1,000,000 x 128 base, 10,000 queries: integer values in [0,255] from
          a mixture of 1,024 Gaussians, rounded and clipped (~30% zeros).
* ``c3``  1,000,000 x 96 base, 10,000 queries on the unit sphere: 256 clusters,
          x = normalize(20*mu + N(0, I)).
* ``c4``  1,000,000 x 960 base, 1,000 queries: |N(0,1)| * 0.1 * s_j with a
          per-dimension scale s_j log-uniform in [0.1, 10].
* ``c5``  8 shards of 12,500,000 x 128 (100M rows), 100,000 queries: integer
          values in [0,255] from a mixture of 4,096 Gaussians; each shard is
          drawn on its own (gen_c5_shard) by the rank that holds it.

Every generator takes ``n``/``nq`` overrides so that tests can draw small
samples with the same distributions.  Data seed = 1000 + config index, query
seed = data seed + 1 (numpy PCG64), so every machine with this numpy produces
bit-identical arrays.

File formats follow the reference loaders byte for byte:
``graph.bin``  int32 n, int32 degree, uint32[n*degree]      (include/cpu_graph.hpp:125-144)
``*.fvecs``    per row: int32 d, d x float32                   (include/data_loader.hpp:9-26)
``*.ivecs``    per row: int32 d, d x int32                     (include/data_loader.hpp:28-45)
``codebook``   uint32 entry, n rows of (dim + wpp*deg + 3*deg + deg) 4-byte
               slots, float32 signs[pdim]                      (include/rabitq.hpp:49-97)
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

CONFIG_INDEX = {"c1": 1, "c2": 2, "c3": 3, "c4": 4}


@dataclass
class SyntheticSet:
    name: str
    base: np.ndarray        # (n, dim) float32, C-contiguous
    queries: np.ndarray     # (nq, dim) float32


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _mixture(rng, n, centres, sigma):
    k, dim = centres.shape
    assign = rng.integers(0, k, size=n)
    x = rng.standard_normal(size=(n, dim), dtype=np.float32)
    x *= np.float32(sigma)
    x += centres[assign]
    return x


def gen_c1(n: int = 10_000, nq: int = 1_000, dim: int = 128) -> SyntheticSet:
    seed = 1000 + CONFIG_INDEX["c1"]
    rc = _rng(seed)
    centres = (rc.standard_normal(size=(100, dim)) * 4.0).astype(np.float32)
    base = _mixture(_rng(seed + 10), n, centres, 1.0)
    queries = _mixture(_rng(seed + 1), nq, centres, 1.0)
    return SyntheticSet("c1", np.ascontiguousarray(base), np.ascontiguousarray(queries))


def gen_c2(n: int = 1_000_000, nq: int = 10_000, dim: int = 128) -> SyntheticSet:
    """Integer-valued [0,255] mixture of 1,024 Gaussians (SIFT-like).

    Centres uniform in [-90, 200] with sigma 25, rounded and clipped, gives
    roughly 30% zeros."""
    seed = 1000 + CONFIG_INDEX["c2"]
    rc = _rng(seed)
    centres = rc.uniform(-90.0, 200.0, size=(1024, dim)).astype(np.float32)

    def draw(rng, m):
        out = np.empty((m, dim), dtype=np.float32)
        step = 1 << 17
        for s in range(0, m, step):
            e = min(m, s + step)
            x = _mixture(rng, e - s, centres, 25.0)
            np.rint(x, out=x)
            np.clip(x, 0.0, 255.0, out=x)
            out[s:e] = x
        return out

    base = draw(_rng(seed + 10), n)
    queries = draw(_rng(seed + 1), nq)
    return SyntheticSet("c2", base, queries)


def gen_c3(n: int = 1_000_000, nq: int = 10_000, dim: int = 96) -> SyntheticSet:
    seed = 1000 + CONFIG_INDEX["c3"]
    rc = _rng(seed)
    mu = rc.standard_normal(size=(256, dim)).astype(np.float32)
    mu /= np.linalg.norm(mu, axis=1, keepdims=True)
    mu *= np.float32(20.0)

    def draw(rng, m):
        x = _mixture(rng, m, mu, 1.0)
        x /= np.linalg.norm(x, axis=1, keepdims=True).astype(np.float32)
        return np.ascontiguousarray(x.astype(np.float32))

    return SyntheticSet("c3", draw(_rng(seed + 10), n), draw(_rng(seed + 1), nq))


def gen_c4(n: int = 1_000_000, nq: int = 1_000, dim: int = 960) -> SyntheticSet:
    seed = 1000 + CONFIG_INDEX["c4"]
    rc = _rng(seed)
    scale = np.exp(rc.uniform(np.log(0.1), np.log(10.0), size=dim)).astype(np.float32)

    def draw(rng, m):
        out = np.empty((m, dim), dtype=np.float32)
        step = 1 << 15
        for s in range(0, m, step):
            e = min(m, s + step)
            x = np.abs(rng.standard_normal(size=(e - s, dim), dtype=np.float32))
            x *= np.float32(0.1)
            x *= scale
            out[s:e] = x
        return out

    return SyntheticSet("c4", draw(_rng(seed + 10), n), draw(_rng(seed + 1), nq))


def gen_c5_shard(shard: int, shard_rows: int = 12_500_000, nq: int = 100_000, dim: int = 128) -> SyntheticSet:
    """Shard `shard` of the C5 base: integer values in [0,255] from a mixture of
    4,096 Gaussians (as C2, more centres), rows shard*shard_rows ... of the
    global base, drawn from the shard's own stream so that every rank makes only
    its own rows; the queries are the same for every shard."""
    seed = 1000 + 5
    rc = _rng(seed)
    centres = rc.uniform(-90.0, 200.0, size=(4096, dim)).astype(np.float32)

    def draw(rng, m):
        out = np.empty((m, dim), dtype=np.float32)
        step = 1 << 17
        for s in range(0, m, step):
            e = min(m, s + step)
            x = _mixture(rng, e - s, centres, 25.0)
            np.rint(x, out=x)
            np.clip(x, 0.0, 255.0, out=x)
            out[s:e] = x
        return out

    return SyntheticSet(f"c5s{shard}", draw(_rng(seed + 100 + shard), shard_rows), draw(_rng(seed + 1), nq))


GENERATORS = {"c1": gen_c1, "c2": gen_c2, "c3": gen_c3, "c4": gen_c4}


# --------------------------------------------------------------------- files

def write_fvecs(path: str, x: np.ndarray) -> None:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    rows = np.empty((n, d + 1), dtype=np.float32)
    rows[:, 0] = np.array([d], dtype=np.int32).view(np.float32)[0]
    rows[:, 1:] = x
    rows.tofile(path)


def write_ivecs(path: str, x: np.ndarray) -> None:
    x = np.ascontiguousarray(x, dtype=np.int32)
    n, d = x.shape
    rows = np.empty((n, d + 1), dtype=np.int32)
    rows[:, 0] = d
    rows[:, 1:] = x
    rows.tofile(path)


def read_fvecs(path: str) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.int32)
    if raw.size == 0:
        return np.zeros((0, 0), dtype=np.float32)
    d = int(raw[0])
    return raw.reshape(-1, d + 1)[:, 1:].copy().view(np.float32)


def read_ivecs(path: str) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.int32)
    if raw.size == 0:
        return np.zeros((0, 0), dtype=np.int32)
    d = int(raw[0])
    return raw.reshape(-1, d + 1)[:, 1:].copy()


def write_graph(path: str, edges: np.ndarray) -> None:
    edges = np.ascontiguousarray(edges, dtype=np.uint32)
    n, deg = edges.shape
    with open(path, "wb") as f:
        np.array([n, deg], dtype=np.int32).tofile(f)
        edges.tofile(f)


def read_graph(path: str) -> np.ndarray:
    with open(path, "rb") as f:
        n, deg = np.fromfile(f, dtype=np.int32, count=2)
        edges = np.fromfile(f, dtype=np.uint32, count=int(n) * int(deg))
    return edges.reshape(int(n), int(deg))


def padded_dim(dim: int) -> int:
    """include/rabitq.hpp:53-56: next power of two >= dim."""
    p = 1
    while p < dim:
        p <<= 1
    return p


@dataclass
class Codebook:
    entry: int
    codes: np.ndarray      # (n, deg, wpp) uint32
    factors: np.ndarray    # (n, 3, deg) float32  [triple_x | factor_dq | factor_vq]
    signs: np.ndarray      # (pdim,) float32
    pdim: int


def read_codebook(path: str, n: int, dim: int, deg: int) -> Codebook:
    """Reads the rows the way include/rabitq.hpp:49-97 does (codes, factors,
    signs; the raw vector and neighbour-id slots are skipped)."""
    pdim = padded_dim(dim)
    wpp = pdim // 32
    row = dim + wpp * deg + 4 * deg
    with open(path, "rb") as f:
        entry = int(np.fromfile(f, dtype=np.uint32, count=1)[0])
        rows = np.fromfile(f, dtype=np.uint32, count=n * row).reshape(n, row)
        signs = np.fromfile(f, dtype=np.float32, count=pdim)
    codes = np.ascontiguousarray(rows[:, dim:dim + wpp * deg]).reshape(n, deg, wpp)
    factors = np.ascontiguousarray(rows[:, dim + wpp * deg:dim + wpp * deg + 3 * deg]).view(np.float32)
    return Codebook(entry, codes, factors.reshape(n, 3, deg), signs, pdim)


# ----------------------------------------------------------- ground truth

def ground_truth(base: np.ndarray, queries: np.ndarray, k: int = 100, block: int = 256) -> np.ndarray:
    """Exact top-k ids by squared L2 in float64, ties by id (CPU, numpy).

    Suitable for the small CPU cases; the benchmark computes the large ones on
    the GPU with the same float64 rule."""
    base64 = base.astype(np.float64)
    bn = (base64 * base64).sum(1)
    out = np.empty((queries.shape[0], k), dtype=np.int32)
    ids = np.arange(base.shape[0])
    for s in range(0, queries.shape[0], block):
        q = queries[s:s + block].astype(np.float64)
        d = bn[None, :] - 2.0 * (q @ base64.T) + (q * q).sum(1)[:, None]
        part = np.argpartition(d, kth=min(k, d.shape[1] - 1), axis=1)[:, :k + 1]
        for r in range(q.shape[0]):
            cand = part[r]
            order = np.lexsort((ids[cand], d[r, cand]))
            out[s + r] = cand[order][:k]
    return out


def cache_dir() -> str:
    d = os.environ.get("BS_DATA_DIR") or os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_data")
    os.makedirs(d, exist_ok=True)
    return d
