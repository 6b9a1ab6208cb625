"""Builds the native parts in-tree (no JIT cache): the sm_100a shared library
``lib/libbsearch_b200.so`` (C ABI of include/bsearch.h) and the drop-in CLIs
``bin/gpu_cli``, ``bin/build_rabitq`` and ``bin/build_graph``.

    python -m beam_search_collab_b200.build [--force]

Every translation unit is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3``; units are
rebuilt when they or a header are newer than their object file.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_obj")
LIB_DIR = os.path.join(PKG, "lib")
BIN_DIR = os.path.join(PKG, "bin")
LIB = os.path.join(LIB_DIR, "libbsearch_b200.so")
CLI = os.path.join(BIN_DIR, "gpu_cli")
RQ_CLI = os.path.join(BIN_DIR, "build_rabitq")
BG_CLI = os.path.join(BIN_DIR, "build_graph")

CU_SOURCES = ["bs_search.cu", "bs_search_nb.cu", "bs_search_bq.cu", "bs_rabitq.cu", "bs_rabitq_nb.cu", "bs_graph_build.cu", "bs_ground_truth.cu", "bs_load.cu", "bs_entry.cu", "bs_merge.cu", "bs_codebook.cu",
              "bs_capi.cu"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--ptxas-options=--warn-on-local-memory-usage"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise FileNotFoundError("nvcc not found")


def _cxx() -> str:
    for c in ("/usr/bin/g++", os.environ.get("CXX"), shutil.which("g++")):
        if c and os.path.exists(c):
            return c
    raise FileNotFoundError("g++ not found")


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".hpp", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "bsearch.h"))
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd))
    for line in (r.stdout + r.stderr).splitlines():
        if "warning" in line.lower() and "lmem" not in line:
            sys.stderr.write(line + "\n")


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(BIN_DIR, exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc] + NVCC_FLAGS + ["-I", INCLUDE, "-c", s, "-o", o]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(_run, jobs))
    if force or _stale(LIB, objs):
        _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs)
    cli_src = os.path.join(CSRC, "gpu_cli.cpp")
    if force or _stale(CLI, [cli_src, LIB] + headers):
        _run([_cxx(), "-std=c++20", "-O2", "-Wall", "-I", INCLUDE, cli_src, "-o", CLI,
              "-L", LIB_DIR, "-lbsearch_b200", "-Wl,-rpath,$ORIGIN/../lib"])
    bg_src = os.path.join(CSRC, "build_graph_cli.cpp")
    if force or _stale(BG_CLI, [bg_src, LIB] + headers):
        _run([_cxx(), "-std=c++20", "-O2", "-Wall", "-I", INCLUDE, bg_src, "-o", BG_CLI,
              "-L", LIB_DIR, "-lbsearch_b200", "-Wl,-rpath,$ORIGIN/../lib"])
    rq_src = os.path.join(CSRC, "build_rabitq_cli.cpp")
    if force or _stale(RQ_CLI, [rq_src, LIB, os.path.join(INCLUDE, "bsearch.h")]):
        _run([_cxx(), "-std=c++20", "-O2", "-Wall", "-I", INCLUDE, rq_src, "-o", RQ_CLI,
              "-L", LIB_DIR, "-lbsearch_b200", "-Wl,-rpath,$ORIGIN/../lib"])
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="pass -Xptxas -v (registers, spills)")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
