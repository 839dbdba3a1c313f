"""The C-ABI library loads and exports every symbol include/lumina_cuda.h
declares (no compute calls: runs on CPU)."""
import os
import re

import pytest

from conftest import REPO


def declared():
    src = open(os.path.join(REPO, "include", "lumina_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lumina_[a-z0-9_]+)\s*\(", src)))


def test_header_parses():
    names = declared()
    assert "lumina_gemv" in names and "lumina_decode_step" in names and len(names) >= 25


def test_library_exports_every_declared_symbol():
    from lumina_b200 import cuda
    path = cuda.lib_path()
    if not os.path.exists(path):
        pytest.skip("library not built (run __graft_entry__.build())")
    lib = cuda.bound_lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared()) <= set(cuda.SIGNATURES), set(declared()) - set(cuda.SIGNATURES)
    assert lib.lumina_cuda_version() == cuda.VERSION


def test_disable_env(monkeypatch):
    from lumina_b200 import cuda
    monkeypatch.setenv("LUMINA_CUDA_DISABLE", "1")
    assert cuda._init()["ok"] is False
    r = cuda.gemv_int8.__wrapped__ if hasattr(cuda.gemv_int8, "__wrapped__") else None
    assert r is None or callable(r)


def test_loader_reads_reference_file():
    from conftest import GOLDEN
    from lumina_b200.loader import LuminaFile
    with LuminaFile(os.path.join(GOLDEN, "small_g64.lumina")) as f:
        recs = {n: f.record(n) for n in f.names()}
    a = recs["model.layers.0.a.weight"]
    assert a.kind == "int4" and a.shape == (37, 96) and a.pack == "nibble" and a.group == 64
    assert a.codes.size == 37 * 48 and a.scales.shape == (37, 2)
    c = recs["model.layers.0.c.weight"]
    assert c.shape == (17, 33) and c.codes.size == 17 * 17
    d = recs["model.layers.0.d.weight"]
    assert d.kind == "int3" and d.pack == "none" and d.codes.size == 20 * 130
    with LuminaFile(os.path.join(GOLDEN, "small_g128.lumina")) as f:
        h = f.record("model.layers.1.h.weight")
    assert h.kind == "binary" and h.shape == (21, 384) and h.codes.size == 21 * 48
