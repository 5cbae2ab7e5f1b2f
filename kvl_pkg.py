"""Loads the `in-c-test_b200/` package (a directory name Python cannot import
directly) under the alias `kvl_b200`."""
from __future__ import annotations

import importlib.util
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parent
PKG_DIR = ROOT / "in-c-test_b200"


def load():
    if "kvl_b200" in sys.modules:
        return sys.modules["kvl_b200"]
    spec = importlib.util.spec_from_file_location("kvl_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["kvl_b200"] = mod
    spec.loader.exec_module(mod)
    return mod
