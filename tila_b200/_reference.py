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


def reference_tree() -> Path:
    """The directory holding Tila's ``examples/`` and ``tests/`` (copied beside
    the package by ``tila_b200.build.ensure_reference_install``, or named by
    ``TILA_REFERENCE_TREE``)."""
    env = os.environ.get("TILA_REFERENCE_TREE")
    for path in ([Path(env)] if env else []) + [REPO_ROOT / "baseline" / "_ref" / "tila_reference_tree"]:
        if (path / "examples").is_dir():
            return path
    raise ImportError(
        "Tila's examples/ are not installed: run __graft_entry__.build() (or "
        "tila_b200.build.ensure_reference_install with a Tila checkout), or set "
        "TILA_REFERENCE_TREE to a directory containing examples/ and tests/")


def example(module: str):
    """Import one of Tila's own example modules (``examples/<module>.py``)
    unchanged; the kernels they define run on the backend as they are."""
    path = str(reference_tree() / "examples")
    if path not in sys.path:
        sys.path.insert(0, path)
    return importlib.import_module(module)
