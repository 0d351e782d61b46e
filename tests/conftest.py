"""Test configuration: the repository root on sys.path and the ``gpu`` marker.

Tests marked ``gpu`` need a B200 (sm_100) and fail without one; the rest run
on any machine (the CUDA code is still generated and compiled by NVRTC).
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
