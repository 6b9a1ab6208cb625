"""CPU: the C-ABI library loads and exports every symbol include/bsearch.h
declares; host-side behaviour that needs no GPU (defaults, error reporting,
the CLI's config handling)."""
import ctypes
import json
import os
import re
import subprocess

import pytest

import beam_search_collab_b200 as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bsearch.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"BS_API\s+[\w\s\*]+?\b(bs_\w+)\s*\(", text)))


def test_header_declares_the_python_export_list():
    assert _declared() == sorted(B.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = B.lib()
    missing = [s for s in _declared() if not hasattr(L, s)]
    assert not missing, missing
    # and nothing else leaks out with default visibility
    out = subprocess.run(["nm", "-D", "--defined-only", B.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (bs_\w+)$", out, re.M)))
    assert exported == _declared()


def test_defaults_are_the_reference_defaults():
    p = B._Params()
    B.lib().bs_search_params_default(ctypes.byref(p))
    assert p.mode == b"base"
    assert (p.K, p.topk_size, p.filter_capacity, p.max_iterations, p.reset_interval) == (100, 256, 1024, 1024, 16)
    assert p.entry_point == 0xFFFFFFFF


def test_version_string():
    assert "sm_100a" in B.version()


def test_null_arguments_are_rejected():
    L = B.lib()
    h = ctypes.c_void_p()
    assert L.bs_index_create(None, 0, ctypes.byref(h)) == 1
    assert "NULL" in L.bs_last_error().decode()
    assert L.bs_index_load(None, None, 0, ctypes.byref(h)) == 1
    assert L.bs_search(None, None, None, 0, None, None, None, None) == 1


def test_missing_files_report_io_error():
    h = ctypes.c_void_p()
    rc = B.lib().bs_index_load(b"/nonexistent/graph.bin", b"/nonexistent/base.fvecs", 0, ctypes.byref(h))
    assert rc == 3
    assert "Cannot open graph file" in B.lib().bs_last_error().decode()


def _cli(cfg_text):
    return subprocess.run([B.CLI_PATH], input=cfg_text, capture_output=True, text=True, timeout=60)


def test_cli_reports_json_errors():
    r = _cli("{ not json")
    assert r.returncode == 1 and "JSON parse error" in r.stderr


def test_cli_requires_data_key():
    r = _cli('{"search": {"mode": "warp1"}}')
    assert r.returncode == 1 and 'Missing "data" key' in r.stderr


def test_cli_accepts_comments_and_reports_missing_files():
    cfg = """
    // reference configs may carry comments (parsed with ignore_comments)
    {"data": {"graph": "/nonexistent/g.bin", /* inline */ "base": "b", "query": "q", "gt": "g"},
     "search": {"mode": "warp1"}}
    """
    r = _cli(cfg)
    assert r.returncode == 1 and "Cannot open graph file: /nonexistent/g.bin" in r.stderr


def test_cli_rejects_legacy_sophia_modes():
    r = _cli(json.dumps({"data": {}, "search": {"mode": "sophia_base"}}))
    assert r.returncode == 1 and "sophia_base" in r.stderr


def _have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_have_gpu(), reason="a GPU is present")
def test_index_create_without_gpu_fails_cleanly():
    import numpy as np
    with pytest.raises(B.BSearchError) as e:
        B.Index.from_arrays(np.zeros((4, 8), np.float32), np.zeros((4, 2), np.uint32))
    assert e.value.status in (4, 5)
