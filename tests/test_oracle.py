"""The oracle, pinned: the golden fixtures (the reference's example kernels
run on its NumPy interpreter, tests/golden/make_golden.py) reproduced by

* the installed example kernels (tila_b200.workloads loads them from the
  installed Tila tree) on the interpreter of this environment, bit for bit -
  the kernels the backend is measured on are the ones the fixtures came from,
  and this NumPy computes what the generating one did;
* the NumPy restatement (oracle.restate) - bit for bit for add and softmax,
  within the reference suite's bounds for matmul and attention
  (tests/gpu_examples.py:28-97);

plus the reference's known answer for f16 dot rounding
(tests/test_m3_capabilities.py:15-30).  CPU only.
"""

import json
from pathlib import Path

import numpy as np
import pytest

import tila_b200
from tila_b200 import workloads as W
from oracle import restate
import semantics_support as S

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(case):
    z = np.load(GOLDEN / f"{case}.npz")
    meta = json.loads(str(z["meta"]))
    inputs = [z[f"in{i}"] for i in range(sum(1 for k in z.files if k.startswith("in")))]
    return inputs, z["out"], meta


def example_kernel(meta):
    ex, consts = meta["example"], dict(meta["consts"])
    if ex.endswith("add_kernel.py"):
        return W.add_kernel, consts
    if ex.endswith("softmax.py"):
        return W.softmax_kernel, consts
    if ex.endswith("matmul.py"):
        return W.matmul_kernel, consts
    if ex.endswith("self_attention.py"):
        return W.self_attention_kernel, consts
    return W.fused_attention_kernel, consts


def test_fixtures_present():
    assert len(CASES) >= 18


@pytest.mark.parametrize("case", CASES)
def test_installed_examples_reproduce_fixtures_bit_exact(case):
    inputs, want, meta = load(case)
    prog, consts = example_kernel(meta)
    out = np.zeros_like(want)
    with np.errstate(all="ignore"):
        prog[tuple(meta["grid"])](*inputs, out, *meta["scalars"], **consts)
    np.testing.assert_array_equal(out, want)


@pytest.mark.parametrize("case", CASES)
def test_restatement_matches_fixture(case):
    inputs, want, meta = load(case)
    ex = meta["example"]
    if ex.endswith("add_kernel.py"):
        np.testing.assert_array_equal(restate.vector_add(*inputs), want)
    elif ex.endswith("softmax.py"):
        np.testing.assert_array_equal(restate.row_softmax_f32(inputs[0], meta["consts"]["BN"]), want)
        np.testing.assert_allclose(want, restate.row_softmax_f64(inputs[0]), rtol=2e-6, atol=2e-7)
    elif ex.endswith("matmul.py"):
        a, b = inputs
        assert np.all(np.abs(want - restate.matmul_f64(a, b)) <= restate.matmul_bound(a, b))
    else:
        causal = ex.endswith("self_attention.py") or meta["consts"].get("CAUSAL", 0) == 1
        ref = restate.attention_f64(*inputs, scale=meta["scalars"][0], causal=causal)
        np.testing.assert_allclose(want, ref, rtol=2e-3, atol=2e-3)
        assert restate.rel_frobenius(want, ref) <= 2e-3


def test_half_dot_rounds_before_widening(tmp_path):
    """Known answer: an f16 dot output is rounded to f16 once, after the f32
    accumulation (tests/test_m3_capabilities.py:15-30)."""
    kernel = S.dot_program(tmp_path, acc="f16")
    a = np.zeros((16, 32), np.float16)
    b = np.zeros((32, 16), np.float16)
    a[:, 0] = 1
    b[0, :] = np.resize(np.array([2**-11, 3 * 2**-11, -2**-12, 2**-10], np.float16), 16)
    c = np.ones((16, 16), np.float16)
    out = np.zeros((16, 16), np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64) + c
    expected = exact.astype(np.float16).astype(np.float32)
    assert np.any(expected != exact)
    kernel[(1,)](a, b, c, out)
    np.testing.assert_array_equal(out, expected)
