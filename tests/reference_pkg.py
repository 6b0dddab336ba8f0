"""Import helper for the reference package installed in baseline/_ref
(baseline/install_reference.py); tests that need it skip without it."""

from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def available() -> bool:
    return (REF / "mantisnet" / "__init__.py").exists()


def load():
    """The reference's mantisnet package (with the hexo_py stub)."""
    if "hexo_py" not in sys.modules:
        stub = types.ModuleType("hexo_py")
        stub.MODEL_REPR_VERSION = 9  # the one attribute read at import time
        sys.modules["hexo_py"] = stub
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    return importlib.import_module("mantisnet")
