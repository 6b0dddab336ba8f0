"""The C-ABI library loads without a GPU and exports exactly what
include/mantis_b200.h declares, with the argument layout the binding uses."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from golden_io import REPO, mb

HEADER = REPO / "include" / "mantis_b200.h"
_lib = mb._lib


def _declarations():
    src = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return re.findall(r"(?:int|const char\*)\s+(mb_\w+)\s*\(([^)]*)\)\s*;", src)


def _code(param: str) -> str:
    p = param.strip()
    if "*" in p:
        return "p"
    return {"int": "i", "int64_t": "l", "float": "f"}[p.rsplit(" ", 1)[0]]


def test_header_matches_binding():
    decls = _declarations()
    assert len(decls) >= 25
    for name, params in decls:
        sig = "" if params.strip() == "void" else "".join(_code(x) for x in params.split(","))
        assert _lib.SIGNATURES.get(name) == sig, name
    assert set(_lib.SIGNATURES) == {d[0] for d in decls}


def test_library_loads_and_exports_every_symbol():
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built (run hexo-shrimp-bot_b200/build.py)")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name, _ in _declarations():
        assert hasattr(lib, name), name
    loaded = _lib.load()
    assert loaded.mb_version() >= 1


def test_host_side_validation_without_gpu():
    """Argument checks run before any launch, so they work on a CPU host."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    _lib.load()
    with pytest.raises(ValueError, match="bad dtype"):
        _lib.call("mb_run_reduce", None, 7, 0, 0, None, None, 1, 32, None, 0, None, 0, None, 0, 0, None)
    with pytest.raises(ValueError, match="head_dim"):
        _lib.call("mb_stone_attention", None, None, None, 0, 1, 1, 24, 0, 0, 0, None, 0, None, 0, -1, None, 0, 0, 0,
                  0, None, None)
    with pytest.raises(ValueError, match="must be bf16"):
        _lib.call("mb_segment_attention_grouped", None, 256, None, None, 512, 0, 1, 1, 8, 32, None, 192, None, 0,
                  None, None, None, None, None, None, 1, 300, None, 1, 256, None)
    with pytest.raises(ValueError, match="unsupported heads"):
        _lib.call("mb_segment_attention_grouped", None, 256, None, None, 512, 1, 1, 1, 2, 128, None, 192, None, 0,
                  None, None, None, None, None, None, 1, 300, None, 1, 256, None)
    with pytest.raises(ValueError, match="key_bits"):
        _lib.call("mb_argsort_workspace", 1000, 0, ctypes.byref(ctypes.c_int64(0)))


def test_cell_pass_refuses_misaligned_and_missing_arrays():
    """mb_cell_pass checks its pointers' alignment and the edge arrays before
    any launch (a misaligned vector access would fault the GPU)."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    _lib.load()
    good, odd = 1 << 20, (1 << 20) + 4  # fake device addresses: 16-byte aligned and not
    with pytest.raises(ValueError, match="aligned"):
        _lib.call("mb_cell_pass", odd, 0, 10, good, 5, good, 3, good, good, good, good, 256, good, good, 0, None)
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("mb_cell_pass", good, 0, 10, good, 5, good, 3, None, good, good, good, 256, good, good, 0, None)
