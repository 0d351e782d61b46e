"""Golden fixtures from the reference's own example kernels.

Runs the reference examples (``examples/add_kernel.py``, ``softmax.py``,
``matmul.py``, ``self_attention.py``, ``fused_attention.py``) on Tila's NumPy
interpreter - the reference implementation - with the seeds, shapes, grids
and Consts of the reference's example suite (tests/gpu_examples.py:28-97),
plus small instances of the benchmarked configurations, and stores inputs and
outputs as ``tests/golden/<case>.npz``.  The tests read only those files.

Usage (in a container that has the reference source tree):

    python tests/golden/make_golden.py --reference <Tila checkout>
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def cdiv(a, b):
    return -(-a // b)


def load_example(ref: Path, name: str):
    spec = importlib.util.spec_from_file_location(f"ref_example_{name}", ref / "examples" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cases():
    """(case, example module, kernel name, inputs, out shape, grid, scalars, consts)."""
    out = []
    for n in (127, 128, 129):
        rng = np.random.default_rng(301)
        x, y = [rng.normal(size=n).astype(np.float32) for _ in range(2)]
        out.append((f"add_n{n}", "add_kernel", "add_kernel", [x, y], (n,), (cdiv(n, 128),), [],
                    {"BLOCK": 128}))
    for n in (31, 32, 33):
        x = np.random.default_rng(302).normal(size=(3, n)).astype(np.float32)
        out.append((f"softmax_n{n}", "softmax", "softmax_kernel", [x], x.shape, (3,), [], {"BN": 64}))
    for m, n, k in ((16, 16, 16), (19, 23, 35)):
        rng = np.random.default_rng(303)
        a = rng.normal(size=(m, k)).astype(np.float16)
        b = rng.normal(size=(k, n)).astype(np.float16)
        out.append((f"matmul_{m}x{n}x{k}", "matmul", "matmul_kernel", [a, b], (m, n),
                    (cdiv(m, 16), cdiv(n, 16)), [], {"BM": 16, "BN": 16, "BK": 32}))
    for n in (32, 65):
        rng = np.random.default_rng(304)
        ins = [rng.normal(size=(n, 32)).astype(np.float16) for _ in range(3)]
        out.append((f"self_attention_n{n}", "self_attention", "self_attention_kernel", ins, (n, 32),
                    (cdiv(n, 32),), [1 / np.sqrt(32)], {"BM": 32, "BN": 32, "BD": 32}))
    for n in (32, 65):
        for causal in (0, 1):
            rng = np.random.default_rng(305)
            ins = [rng.normal(size=(2, n, 32)).astype(np.float16) for _ in range(3)]
            out.append((f"fused_attention_n{n}_causal{causal}", "fused_attention", "fused_attention_kernel",
                        ins, (2, n, 32), (cdiv(n, 32), 2), [1 / np.sqrt(32)],
                        {"BM": 32, "BN": 32, "BD": 32, "CAUSAL": causal}))
    # small instances of the benchmarked configurations (the benchmark's input
    # distributions: U[-1,1) for add, N(0,2) for softmax, N(0,1/sqrt(K)) f16
    # for matmul, N(0,1) f16 for attention; seed 0)
    rng = np.random.default_rng(0)
    x = rng.uniform(-1.0, 1.0, 4096).astype(np.float32)
    y = rng.uniform(-1.0, 1.0, 4096).astype(np.float32)
    out.append(("bench_add_4096", "add_kernel", "add_kernel", [x, y], (4096,), (4,), [], {"BLOCK": 1024}))
    x = np.random.default_rng(0).normal(0.0, 2.0, (16, 1000)).astype(np.float32)
    out.append(("bench_softmax_16x1000", "softmax", "softmax_kernel", [x], x.shape, (16,), [], {"BN": 1024}))
    rng = np.random.default_rng(0)
    sd = 1.0 / np.sqrt(256)
    a = rng.normal(0.0, sd, (256, 256)).astype(np.float16)
    b = rng.normal(0.0, sd, (256, 256)).astype(np.float16)
    out.append(("bench_matmul_256", "matmul", "matmul_kernel", [a, b], (256, 256), (2, 2), [],
                {"BM": 128, "BN": 128, "BK": 64}))
    rng = np.random.default_rng(0)
    ins = [rng.normal(0.0, 1.0, (2, 256, 128)).astype(np.float16) for _ in range(3)]
    out.append(("bench_fused_attention_2x256x128", "fused_attention", "fused_attention_kernel", ins,
                (2, 256, 128), (2, 2), [128 ** -0.5], {"BM": 128, "BN": 128, "BD": 128, "CAUSAL": 0}))
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a Tila source checkout (with src/ and examples/)")
    args = ap.parse_args(argv)
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "src"))
    import tila  # noqa: F401  (the reference package)
    mods = {}
    for case, modname, kname, inputs, oshape, grid, scalars, consts in cases():
        mod = mods.setdefault(modname, load_example(ref, modname))
        kern = getattr(mod, kname)
        o = np.zeros(oshape, np.float32)
        with np.errstate(all="ignore"):
            kern[grid](*inputs, o, *scalars, **consts)
        meta = {"example": f"examples/{modname}.py", "kernel": kname, "grid": list(grid),
                "scalars": [float(s) for s in scalars], "consts": consts}
        arrays = {f"in{i}": a for i, a in enumerate(inputs)}
        np.savez_compressed(HERE / f"{case}.npz", out=o, meta=np.array(json.dumps(meta)), **arrays)
        print(case, o.shape, float(np.abs(o).max()))


if __name__ == "__main__":
    main()
