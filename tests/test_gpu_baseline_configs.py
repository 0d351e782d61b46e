"""Parity at the benchmarked configurations, through ``kernel[grid]`` on the
reference's own example kernels (and the three unfused-attention programs).

The same launches the benchmark times - full grids, full K and sequence
lengths, the tail waves of the CTA schedule - checked where a full CPU
reference is affordable on sampled rows and heads:

* matmul 4096^3 (128/128/64): every element of 256 sampled rows (spread over
  all 32 tile rows, first and last included) within the reference's K*eps_f32
  bound of the f64 product (tests/gpu_examples.py:52-64), and the sample's
  relative Frobenius error <= 2e-3;
* fused attention B4 H32 L4096 D128 (CAUSAL=0, BM=BN=128): two sampled heads
  within 2e-3 relative Frobenius error of the f64 attention, and one head
  against the interpreter running the same kernel on that head;
* causal fused attention at the same size (CAUSAL=1): two sampled heads;
* unfused attention B8 H16 L1024 D64 (three launches, S materialised): three
  sampled heads within 2e-3 of the f64 attention;
* softmax 8192x1000 and add 2^20 run at full size in tests/test_gpu_parity.py.
"""

import numpy as np
import pytest

import tila_b200
from tila_b200 import workloads as W
from oracle import interp, restate

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _no_device_errors():
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0


def test_matmul_4096_cubed():
    a, b = W.matmul_inputs(4096, 4096, 4096, seed=0)
    c = torch.zeros((4096, 4096), dtype=torch.float32, device="cuda")
    W.matmul_kernel[(32, 32)](_cuda(a), _cuda(b), c, BM=128, BN=128, BK=64)
    _no_device_errors()
    rng = np.random.default_rng(1)
    rows = np.unique(np.concatenate([np.arange(0, 8), np.arange(4088, 4096),
                                     rng.choice(4096, 240, replace=False)]))[:256]
    got = c[torch.from_numpy(rows).cuda()].cpu().numpy()
    ref = restate.matmul_f64(a[rows], b)
    bound = restate.matmul_bound(a[rows], b)
    assert np.all(np.abs(got - ref) <= bound)
    assert restate.rel_frobenius(got, ref) <= 2e-3


def _fused(causal, warps):
    bh, l, d = 128, 4096, 128
    q, k, v = W.attention_inputs(bh, l, d, seed=0)
    o = torch.zeros((bh, l, d), dtype=torch.float32, device="cuda")
    W.fused_attention_kernel[(l // 128, bh)].with_options(num_warps=warps)(
        _cuda(q), _cuda(k), _cuda(v), o, d ** -0.5, CAUSAL=causal, BM=128, BN=128, BD=128)
    _no_device_errors()
    return (q, k, v), o


def test_fused_attention_full_size():
    (q, k, v), o = _fused(0, 4)
    for h in (0, 77):
        ref = restate.attention_f64(q[h], k[h], v[h])
        assert restate.rel_frobenius(o[h].cpu().numpy(), ref) <= 2e-3
    # one head against the interpreter running the same kernel on that head
    h = 127
    cpu = np.zeros((1, 4096, 128), np.float32)
    interp.run(W.fused_attention_kernel, (32, 1), [q[h:h + 1], k[h:h + 1], v[h:h + 1], cpu],
               128 ** -0.5, CAUSAL=0, BM=128, BN=128, BD=128)
    assert restate.rel_frobenius(o[h].cpu().numpy(), cpu[0]) <= 2e-3


def test_causal_fused_attention_full_size():
    (q, k, v), o = _fused(1, 8)
    for h in (3, 126):
        ref = restate.attention_f64(q[h], k[h], v[h], causal=True)
        assert restate.rel_frobenius(o[h].cpu().numpy(), ref) <= 2e-3


def test_unfused_attention_full_size():
    bh, l, d = 128, 1024, 64
    q, k, v = W.attention_inputs(bh, l, d, seed=0)
    qg, kg, vg = _cuda(q), _cuda(k), _cuda(v)
    s = torch.empty((bh, l, l), device="cuda")
    p = torch.empty_like(s)
    o = torch.zeros((bh, l, d), device="cuda")
    W.attention_scores[(l // 128, l // 128, bh)](qg, kg, s, 0.125, BM=128, BN=128, BD=64)
    W.softmax_kernel[(bh * l,)](s.view(bh * l, l), p.view(bh * l, l), BN=1024)
    W.attention_pv[(l // 128, bh)](p, vg, o, BM=128, BN=128, BD=64)
    _no_device_errors()
    for h in (0, 64, 127):
        ref = restate.attention_f64(q[h], k[h], v[h], scale=0.125)
        assert restate.rel_frobenius(o[h].cpu().numpy(), ref) <= 2e-3
