"""The B200 backend on the golden fixtures (the reference's example kernels'
inputs and interpreter outputs, tests/golden/): the same programs launched on
CUDA tensors, held to the reference suite's bars - add bit-exact, softmax
rtol 1e-6, matmul K*eps_f32 elementwise, attention (causal and not) 2e-3."""

import numpy as np
import pytest
import torch

import tila_b200
from tila_b200 import workloads as W
from oracle import restate
from test_oracle import CASES, load, example_kernel

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("case", CASES)
def test_golden_on_b200(case):
    inputs, want, meta = load(case)
    prog, consts = example_kernel(meta)
    out = torch.zeros(want.shape, dtype=torch.float32, device="cuda")
    prog[tuple(meta["grid"])](*(_cuda(a) for a in inputs), out, *meta["scalars"], **consts)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    got = out.cpu().numpy()
    ex = meta["example"]
    if ex.endswith("add_kernel.py"):
        np.testing.assert_array_equal(got, want)
    elif ex.endswith("softmax.py"):
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=0)
    elif ex.endswith("matmul.py"):
        a, b = inputs
        assert np.all(np.abs(got - restate.matmul_f64(a, b)) <= restate.matmul_bound(a, b))
        assert restate.rel_frobenius(got, want) <= 2e-3
    else:
        causal = ex.endswith("self_attention.py") or meta["consts"].get("CAUSAL", 0) == 1
        ref = restate.attention_f64(*inputs, scale=meta["scalars"][0], causal=causal)
        np.testing.assert_allclose(got, ref, rtol=2e-3, atol=2e-3)
        assert restate.rel_frobenius(got, want) <= 2e-3


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("l,d", [(128, 64), (300, 64), (384, 128)])
def test_causal_flash_attention_128_tiles(l, d, warps):
    """The two-stage causal kernel (stage loops whose trip count depends on
    program_id(0): two programs per CTA with different trip counts) at
    128x128 tiles."""
    q, k, v = W.attention_inputs(2, l, d, seed=17)
    o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    W.fused_attention_kernel[(-(-l // 128), 2)].with_options(num_warps=warps)(
        _cuda(q), _cuda(k), _cuda(v), o, d ** -0.5, CAUSAL=1, BM=128, BN=128, BD=d)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    ref = restate.attention_f64(q, k, v, causal=True)
    assert restate.rel_frobenius(o.cpu().numpy(), ref) <= 2e-3


def test_causal_flash_attention_heavy_first_order():
    """11 heads at L=1000: the heavy-first CTA numbering of the causal kernel
    covers one full group of 8 heads and a partial group of 3; every query
    block of every head is computed once (eight blocks, the last partial)."""
    q, k, v = W.attention_inputs(11, 1000, 128, seed=23)
    o = torch.full(q.shape, float("nan"), dtype=torch.float32, device="cuda")
    W.fused_attention_kernel[(-(-1000 // 128), 11)](
        _cuda(q), _cuda(k), _cuda(v), o, 128 ** -0.5, CAUSAL=1, BM=128, BN=128, BD=128)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    got = o.cpu().numpy()
    assert np.isfinite(got).all()
    for h in (0, 7, 8, 10):
        ref = restate.attention_f64(q[h:h + 1], k[h:h + 1], v[h:h + 1], causal=True)
        assert restate.rel_frobenius(got[h:h + 1], ref) <= 2e-3
