"""Locate the ``tila`` package this backend plugs into.

The backend does not re-implement Tila: ``@ti.jit``, the checker, the bounds
proofs and the NumPy interpreter are imported from an installed Tila
(``tila-lang``).  Search order: an importable ``tila``; the directory named
by ``TILA_REFERENCE_PATH``; the ``baseline/_ref`` install beside this
repository (``pip install --target baseline/_ref``).
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

REPO_ROOT = Path(__file__).resolve().parents[1]


def _candidates():
    env = os.environ.get("TILA_REFERENCE_PATH")
    if env:
        yield Path(env)
    yield REPO_ROOT / "baseline" / "_ref"


def import_tila():
    try:
        return importlib.import_module("tila")
    except ImportError:
        pass
    for path in _candidates():
        if (path / "tila" / "__init__.py").exists():
            sys.path.insert(0, str(path))
            try:
                return importlib.import_module("tila")
            except ImportError:
                sys.path.remove(str(path))
    raise ImportError(
        "the Tila package (tila-lang) is not importable; install it, or set "
        "TILA_REFERENCE_PATH to a directory containing the `tila` package")


tila = import_tila()
