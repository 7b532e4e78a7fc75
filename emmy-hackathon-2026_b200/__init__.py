"""b200k: a B200-native (sm_100a) kernel backend for Emmy Kernel IR.

The package directory is named ``emmy-hackathon-2026_b200``; import it with
``importlib.import_module("emmy-hackathon-2026_b200")`` (or through
:func:`load` below from a path).  Submodules:

* ``ir``        -- safe loader for the ``*.ir.json`` graph format
* ``runtime``   -- ctypes binding of ``libb200k.so`` (the C ABI in include/b200k.h)
* ``build``     -- nvcc build of ``libb200k.so`` for sm_100a
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

PACKAGE_NAME = "emmy-hackathon-2026_b200"


def load():
    """Return this package (importable by its hyphenated directory name)."""
    root = str(Path(__file__).resolve().parent.parent)
    if root not in sys.path:
        sys.path.insert(0, root)
    return importlib.import_module(PACKAGE_NAME)


def submodule(name: str):
    return importlib.import_module(f"{PACKAGE_NAME}.{name}")
