"""Tila's own GPU test suites, run unchanged against the B200 backend.

Tila gates its CUDA path with the suites that ``tools/gpu_audit.py`` runs
(``tests/gpu_semantics.py``, ``gpu_examples.py``, ``gpu_launch.py``,
``gpu_backend.py``, ``gpu_capabilities.py``, ``gpu_alignment.py``,
``gpu_matrix_gaps.py``, ``gpu_atomic.py``, ``gpu_race.py``,
``gpu_soundness.py``, ``gpu_c2.py``; tools/gpu_audit.py:95-108).  Each one
runs here in a child pytest, in the installed Tila tree, with the audit's
environment switches and with ``reference_suite_plugin`` loaded: importing
``tila_b200`` routes every CUDA launch to the generated sm_100a kernels.  The
suites' own assertions are the bar (bit-exact integers, the exp/exp2
tolerance classes, dot accumulator rounding, the example kernels' bounds,
launch-contract negatives).  A suite passes when its child pytest exits 0,
the backend ran at least one launch, and no Triton kernel ran.

``EXCLUDED`` lists the cases that test the Triton lowering itself (its
generated source or its compiler) rather than kernel behaviour, each with
the reason.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
TESTS = Path(__file__).resolve().parent

SUITES = ["gpu_examples.py", "gpu_semantics.py", "gpu_capabilities.py", "gpu_matrix_gaps.py",
          "gpu_launch.py", "gpu_alignment.py", "gpu_atomic.py", "gpu_race.py",
          "gpu_soundness.py", "gpu_backend.py", "gpu_c2.py"]

# node id -> why it does not apply to a backend that does not generate Triton
EXCLUDED = {
    "gpu_backend.py::test_real_compiler_failure_mapping_and_replay":
        "plants a fault in the Triton source (Lowering.kernel_source) and expects Triton's "
        "compiler to reject it; the B200 path generates no Triton source (its NVRTC failure "
        "mapping to TILA-TARGET-010 with the replayable artifact is tests/test_native.py)",
    "gpu_backend.py::test_real_shared_memory_overflow_never_launches":
        "expects the 256x256x128 matmul tile to overflow SM86 shared memory (TILA-TARGET-011); "
        "on B200 its two 128 KB operand tiles fit, and the B200 backend rejects the tile earlier "
        "with TILA-TARGET-009 because it does not lower dots of more than 128 rows per program",
    "gpu_semantics.py::test_existing_suite[integer]":
        "the interpreter half of gpu_integer_smoke.py (unsigned_scalar with value 2**64-1, "
        "divmod64) raises OverflowError inside Tila's NumPy interpreter under NumPy 2.x "
        "(the reference pins numpy 1.24.3), before the B200 launch; the same kernels run on "
        "the B200 against exact expectations in tests/test_gpu_semantics.py",
    "gpu_alignment.py::test_aligned_hint_on_off":
        "counts a second Triton kernel after patching Lowering.alignment_prefix out of the "
        "Triton source; the B200 path does not use Lowering (its own alignment facts are "
        "covered by the suite's other cases and tests/test_codegen.py)",
}


def _tree():
    from tila_b200._reference import reference_tree
    return reference_tree()


@pytest.mark.parametrize("suite", SUITES)
def test_reference_gpu_suite(suite, tmp_path):
    tests_dir = _tree() / "tests"
    assert (tests_dir / suite).exists(), f"{suite} is not in the installed Tila tree"
    report = tmp_path / "report.json"
    env = dict(os.environ)
    env.update(
        PYTHONPATH=os.pathsep.join([str(ROOT), str(TESTS), str(ROOT / "baseline" / "_ref")]),
        PYTHONHASHSEED="0", PYTEST_ADDOPTS="", PYTEST_DISABLE_PLUGIN_AUTOLOAD="1",
        TILA_INTERP="0", TRITON_INTERPRET="0", TILA_SAFETY="strict", TILA_DEBUG="0",
        TILA_EFFECTS="warn", TILA_RACE="warn", TILA_RACE_MAX_PAIRS="4096",
        TILA_GPU_KERNELS=str(tmp_path / "kernels"), TMPDIR=str(tmp_path),
        TILA_C2_FAILURE_DIR=str(tmp_path / "c2-failures"),
        TILA_BACKEND_ARTIFACTS=str(tmp_path / "backend"), TILA_SUITE_REPORT=str(report))
    (tmp_path / "kernels").mkdir()
    deselect = []
    for node in EXCLUDED:
        if node.startswith(suite + "::"):
            deselect += ["--deselect", node]
    cmd = [sys.executable, "-m", "pytest", suite, "-q", "-p", "reference_suite_plugin",
           "-p", "no:cacheprovider", "-c", os.devnull, "--rootdir", str(tests_dir), *deselect]
    proc = subprocess.run(cmd, cwd=tests_dir, env=env, capture_output=True, text=True, timeout=1500)
    out = proc.stdout + proc.stderr
    log_dir = os.environ.get("TILA_SUITE_LOG_DIR")
    if log_dir:
        Path(log_dir).mkdir(parents=True, exist_ok=True)
        (Path(log_dir) / (suite + ".log")).write_text(out)
    summary = [ln for ln in out.splitlines() if ln.startswith(("FAILED", "ERROR"))]
    assert proc.returncode == 0, f"{suite} failed on the B200 backend:\n" + "\n".join(summary[:40]) \
        + "\n" + out[-3000:]
    counts = json.loads(report.read_text())
    assert counts["triton_runs"] == 0, counts
    assert counts["b200_launches"] > 0, counts
    assert Path(counts["tila_b200"]).resolve().is_relative_to(ROOT), counts
