"""Run Tila programs on the reference NumPy interpreter (the oracle).

The interpreter is Tila's own CPU executor: ``kernel[grid](numpy arrays)``
goes through the full launch contract (runtime.py:726-1039) and then
``interp.run_kernel`` (interp.py:407), which executes the typed TIR program by
program with NumPy block operations.  TEST INFRASTRUCTURE ONLY.
"""

from __future__ import annotations

import numpy as np


def run(kernel, grid, arrays, *scalars, **consts):
    """Launch ``kernel`` on NumPy arrays (outputs are written in place)."""
    arrays = [np.ascontiguousarray(a) if a.flags.c_contiguous else a for a in arrays]
    kernel[grid](*arrays, *scalars, **consts)
    return arrays
