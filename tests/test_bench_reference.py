"""The benchmark's reference arm: Tila's NumPy interpreter spread over worker
processes by contiguous shards of the program axis.  A shard is a slice of
the inputs launched with the grid that slice calls for; the shards together
must compute exactly what one launch over the whole sample computes (the
timing then measures the reference's own work, split, not something else)."""

import numpy as np

import bench
from tila_b200 import workloads as W


def test_sharded_add_matches_one_launch():
    x, y = W.add_inputs(6 * 1024, seed=3)
    whole = np.zeros_like(x)
    W.add_kernel[(6,)](x, y, whole, BLOCK=1024)
    out = np.zeros_like(x)
    bench._REF_DATA["add"] = (x, y, out)
    try:
        for lo, hi in bench._ref_shards(6, 4):
            bench._ref_run("add", lo, hi)
    finally:
        bench._REF_DATA.pop("add")
    np.testing.assert_array_equal(out, whole)


def test_sharded_softmax_matches_one_launch():
    x = W.softmax_inputs(40, 1000, seed=4)
    whole = np.zeros_like(x)
    W.softmax_kernel[(40,)](x, whole, BN=1024)
    out = np.zeros_like(x)
    bench._REF_DATA["softmax"] = (x, out)
    try:
        for lo, hi in bench._ref_shards(40, 3):
            bench._ref_run("softmax", lo, hi)
    finally:
        bench._REF_DATA.pop("softmax")
    np.testing.assert_array_equal(out, whole)


def test_reference_samples_cover_their_program_axis():
    for key, (length, desc) in bench._REF_SAMPLE.items():
        for parts in (1, 7, 16, 64):
            shards = bench._ref_shards(length, parts)
            assert shards[0][0] == 0 and shards[-1][1] == length
            assert all(a[1] == b[0] for a, b in zip(shards, shards[1:]))
        units, unit, scale = bench._ref_units(key)
        assert units > 0 and unit in ("GB/s", "TFLOP/s") and desc


def test_reference_arm_prints_the_contract_line():
    """``bench.py --impl reference`` (what the driver runs beside the GPU arm)
    prints one JSON line with the reference keys: no GPU is needed for it."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(bench.__file__).resolve().parent
    out = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", "--workload", "add",
                          "--only", "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["higher_is_better"] is True and line["config"]["workload"] == "add"
    base = line["cpu_baseline"]
    assert base["kind"] == "reference" and base["cores"] >= 1 and base["value"] == line["value"]
    assert "worker processes" in base["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
