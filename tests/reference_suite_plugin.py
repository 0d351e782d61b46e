"""pytest plugin that runs Tila's own GPU suites (``tests/gpu_*.py`` of the
Tila tree) against the B200 backend.

Loaded with ``-p reference_suite_plugin`` in the child pytest that
``tests/test_gpu_reference_suites.py`` starts.  Importing ``tila_b200``
installs the backend into ``tila.runtime._Launcher``, so the suites' CUDA
launches go to the generated sm_100a kernels instead of Triton; nothing in the
suites is edited.  The plugin counts the launches that reached the backend
and every Triton kernel run (there must be none) and writes the counts to the
JSON file named by ``TILA_SUITE_REPORT`` when the session ends.
"""

import json
import os

import tila_b200
from tila_b200 import backend

_counts = {"b200_launches": 0, "triton_runs": 0, "tila_b200": tila_b200.__file__}

_execute = backend.execute


def _counting_execute(*args, **kwargs):
    _counts["b200_launches"] += 1
    return _execute(*args, **kwargs)


backend.execute = _counting_execute

try:
    import triton

    _triton_run = triton.runtime.jit.JITFunction.run

    def _counting_run(self, *args, **kwargs):
        if not kwargs.get("warmup"):
            _counts["triton_runs"] += 1
        return _triton_run(self, *args, **kwargs)

    triton.runtime.jit.JITFunction.run = _counting_run
except Exception:          # Triton is optional: the backend never imports it
    pass


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("TILA_SUITE_REPORT")
    if path:
        with open(path, "w") as f:
            json.dump(dict(_counts, exitstatus=int(exitstatus)), f)
