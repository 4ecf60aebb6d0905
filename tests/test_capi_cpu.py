"""The C-ABI library loads and exports every entry point include/ks_b200.h
declares (no compute calls: this runs without a GPU)."""
import ctypes
import os
import re

from conftest import ROOT


def header_functions():
    src = open(os.path.join(ROOT, "include", "ks_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ks_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_operators():
    names = header_functions()
    for n in ("ks_sinkhorn", "ks_sparse_attn", "ks_indexer", "ks_indexer_scores", "ks_topk_rows",
              "ks_indexer_workspace_size", "ks_dsa", "ks_last_error", "ks_device_status"):
        assert n in names


def test_library_exports_every_declared_symbol(built_lib):
    handle = ctypes.CDLL(built_lib)
    missing = [n for n in header_functions() if not hasattr(handle, n)]
    assert not missing, missing


def test_python_signatures_cover_header(built_lib):
    from kernelswift_b200 import _lib

    assert sorted(_lib.SIGNATURES) == header_functions()
    lib = _lib.lib()
    assert lib.ks_version() == 101
    assert lib.ks_last_error() == b""


def test_workspace_size_is_host_only(built_lib):
    from kernelswift_b200 import _lib

    lib = _lib.lib()
    assert lib.ks_indexer_workspace_size(2, 32768, 32768) == 2 * 32768 * 32768 * 2
    assert lib.ks_indexer_workspace_size(1, 3, 5) % 256 == 0


def test_tiny_attention_column_token_floor():
    """The short-row attention kernel (csrc/sparse_attn_tiny.cuh) finds a key
    column's token as floor((c + 1/2) * fp32(1 / kp)) instead of c / kp.  Exact for
    every column c < 256 (SAT_MAX_N) and every slot count it takes (kp = K rounded
    up to 16, K <= 64), with fp32 round-to-nearest as on the GPU."""
    import numpy as np

    for kp in (16, 32, 48, 64):
        inv = np.float32(1.0) / np.float32(kp)
        c = np.arange(256, dtype=np.float32)
        j = np.floor((c + np.float32(0.5)) * inv).astype(np.int64)
        assert np.array_equal(j, np.arange(256) // kp)
