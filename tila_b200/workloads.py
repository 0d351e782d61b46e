"""The five benchmarked workloads: the kernels, their seeded inputs and their work.

Four of the five are Tila's own example kernels, imported unchanged from the
installed Tila tree (``examples/add_kernel.py:12-27``, ``examples/softmax.py:14-29``,
``examples/matmul.py:10-40``, ``examples/fused_attention.py:34-128``; the latter
with ``CAUSAL=0`` is the benchmarked fused attention and with ``CAUSAL=1`` its
causal variant), plus ``examples/self_attention.py:18-73``.  The unfused
attention has no example in Tila; it is written here as three ordinary Tila
programs (scores, the row softmax of ``examples/softmax.py``, P@V).  Nothing in
any of them is specific to the B200 backend: the same kernel runs on the
NumPy interpreter (CPU arrays) and on the B200 backend (CUDA tensors).  Each
workload also provides its seeded synthetic inputs and its algorithmic work
(bytes or flops) for the roofline.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ._reference import example, tila as ti

BH = ti.Dim("BH")
L = ti.Dim("L")
BD = ti.Dim("BD")


# ---------------------------------------------------------------------------
# Tila's example kernels, unchanged
# ---------------------------------------------------------------------------

add_kernel = example("add_kernel").add_kernel                     # K1
softmax_kernel = example("softmax").softmax_kernel                # K2 (also the middle launch of K4)
matmul_kernel = example("matmul").matmul_kernel                   # K3
fused_attention_kernel = example("fused_attention").fused_attention_kernel   # K5 (CAUSAL=0)
self_attention_kernel = example("self_attention").self_attention_kernel


# ---------------------------------------------------------------------------
# K4: unfused attention = scores (QK^T * scale) -> row softmax -> P @ V
# ---------------------------------------------------------------------------

@ti.jit
def attention_scores(
    q: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    k: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    s: ti.Buffer[ti.f32, (BH, L, L), ti.WriteOnly],
    scale: ti.f32,
    BM: ti.Const[int, ti.PowerOfTwo] = 128,
    BN: ti.Const[int, ti.PowerOfTwo] = 128,
    BD: ti.Const[int, ti.PowerOfTwo] = 64,
):
    qb = ti.program_id(0)
    kb = ti.program_id(1)
    h = ti.program_id(2)
    qi = qb * BM + ti.arange(0, BM)
    ki = kb * BN + ti.arange(0, BN)
    di = ti.arange(0, BD)
    q_ok = qi < L
    k_ok = ki < L
    qt = ti.load(q, (h, qi[:, None], di[None, :]), mask=q_ok[:, None])
    kt = ti.load(k, (h, ki[None, :], di[:, None]), mask=k_ok[None, :])      # (BD, BN) = K^T
    ti.store(s, (h, qi[:, None], ki[None, :]), ti.dot(qt, kt) * scale,
             mask=q_ok[:, None] & k_ok[None, :])


@ti.jit
def attention_pv(
    p: ti.Buffer[ti.f32, (BH, L, L), ti.ReadOnly],
    v: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    o: ti.Buffer[ti.f32, (BH, L, BD), ti.WriteOnly],
    BM: ti.Const[int, ti.PowerOfTwo] = 128,
    BN: ti.Const[int, ti.PowerOfTwo] = 128,
    BD: ti.Const[int, ti.PowerOfTwo] = 64,
):
    qb = ti.program_id(0)
    h = ti.program_id(1)
    qi = qb * BM + ti.arange(0, BM)
    kn = ti.arange(0, BN)
    di = ti.arange(0, BD)
    q_ok = qi < L
    out = ti.zeros((BM, BD), ti.f32)
    for n0 in ti.range(0, L, BN):
        ki = n0 + kn
        k_ok = ki < L
        pt = ti.load(p, (h, qi[:, None], ki[None, :]), mask=q_ok[:, None] & k_ok[None, :])
        vt = ti.load(v, (h, ki[:, None], di[None, :]), mask=k_ok[:, None])
        out = ti.dot(ti.cast[ti.f16](pt), vt, acc=out)
    ti.store(o, (h, qi[:, None], di[None, :]), out, mask=q_ok[:, None])


# ---------------------------------------------------------------------------
# configurations (the benchmarked sizes) and their synthetic inputs
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Workload:
    key: str
    description: str
    roofline: str          # "hbm" or "tensor"
    unit: str              # GB/s or TFLOP/s


WORKLOADS = {
    "add": Workload("add", "vector add, x,y f32 (N=1048576), BLOCK=1024", "hbm", "GB/s"),
    "softmax": Workload("softmax", "row softmax, f32 [8192, 1000], BN=1024", "hbm", "GB/s"),
    "matmul": Workload("matmul", "matmul f16 [4096,4096] x [4096,4096] -> f32, 128/128/64",
                       "tensor", "TFLOP/s"),
    "unfused_attention": Workload("unfused_attention",
                                  "unfused attention B=8 H=16 L=1024 D=64, S materialised",
                                  "hbm", "TFLOP/s"),
    "fused_attention": Workload("fused_attention",
                                "flash attention B=4 H=32 L=4096 D=128, non-causal, BM=BN=128",
                                "tensor", "TFLOP/s"),
}


def add_inputs(n=1 << 20, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, n).astype(np.float32)
    y = rng.uniform(-1.0, 1.0, n).astype(np.float32)
    return x, y


def softmax_inputs(m=8192, n=1000, seed=0):
    rng = np.random.default_rng(seed)
    return rng.normal(0.0, 2.0, (m, n)).astype(np.float32)


def matmul_inputs(m=4096, n=4096, k=4096, seed=0):
    rng = np.random.default_rng(seed)
    sd = 1.0 / np.sqrt(k)
    a = rng.normal(0.0, sd, (m, k)).astype(np.float16)
    b = rng.normal(0.0, sd, (k, n)).astype(np.float16)
    return a, b


def attention_inputs(bh, l, d, seed=0):
    rng = np.random.default_rng(seed)
    return tuple(rng.normal(0.0, 1.0, (bh, l, d)).astype(np.float16) for _ in range(3))


# algorithmic work per run (bytes for HBM-bound, flops for tensor-bound)
def add_bytes(n=1 << 20):
    return 3 * 4 * n


def softmax_bytes(m=8192, n=1000):
    return 2 * 4 * m * n


def matmul_flops(m=4096, n=4096, k=4096):
    return 2 * m * n * k


def unfused_bytes(bh=128, l=1024, d=64):
    qk = 2 * bh * l * d * 2
    s = bh * l * l * 4
    return qk + 4 * s + bh * l * d * 2 + bh * l * d * 4


def unfused_flops(bh=128, l=1024, d=64):
    return 2 * 2 * bh * l * l * d


def fused_flops(bh=128, l=4096, d=128):
    return 4 * bh * l * l * d


def causal_flops(bh=128, l=4096, d=128):
    """Causal attention counted as half of the full score and P@V work (the
    usual convention; the kernel also computes the masked half of the
    diagonal blocks)."""
    return 2 * bh * l * l * d


def cdiv(a, b):
    return -(-a // b)
