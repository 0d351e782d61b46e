"""The five judged workloads, written as ordinary Tila programs.

These are the programs the backend is measured on: vector add, row softmax,
tiled matmul, unfused self-attention (three launches with the score matrix S
materialised in HBM) and fused flash attention.  They are plain ``@ti.jit``
kernels - nothing in them is specific to the B200 backend - so the same
program runs on the NumPy interpreter (CPU arrays) and on the B200 backend
(CUDA tensors).  Each workload also provides its seeded synthetic inputs and
its algorithmic work (bytes or flops) for the roofline.

The programs express the algorithms of the reference examples
(examples/add_kernel.py:12-27, examples/softmax.py:14-29,
examples/matmul.py:10-40, examples/fused_attention.py:104-126 for the
non-causal loop; the causal variants follow examples/fused_attention.py:62-103
and examples/self_attention.py); ``tests/test_oracle.py`` checks, on the
interpreter, that they produce bit-identical results to those examples on the
fixtures in ``tests/golden/``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ._reference import tila as ti

N = ti.Dim("N")
M = ti.Dim("M")
K = ti.Dim("K")
BH = ti.Dim("BH")
L = ti.Dim("L")
BD = ti.Dim("BD")

LOG2E = 1.4426950408889634


# ---------------------------------------------------------------------------
# K1: vector add
# ---------------------------------------------------------------------------

@ti.jit
def vector_add(
    x: ti.Buffer[ti.f32, (N,), ti.ReadOnly],
    y: ti.Buffer[ti.f32, (N,), ti.ReadOnly],
    out: ti.Buffer[ti.f32, (N,), ti.WriteOnly],
    BLOCK: ti.Const[int, ti.PowerOfTwo] = 1024,
):
    block = ti.program_id(0)
    idx = block * BLOCK + ti.arange(0, BLOCK)
    live = idx < N
    ti.store(out, idx, ti.load(x, idx, mask=live) + ti.load(y, idx, mask=live), mask=live)


# ---------------------------------------------------------------------------
# K2: row softmax (one program per row; masked tail lanes read -1e30)
# ---------------------------------------------------------------------------

@ti.jit
def row_softmax(
    x: ti.Buffer[ti.f32, (M, N), ti.ReadOnly],
    o: ti.Buffer[ti.f32, (M, N), ti.WriteOnly],
    BN: ti.Const[int, ti.PowerOfTwo] = 1024,
):
    r = ti.program_id(0)
    cols = ti.arange(0, BN)
    inside = cols < N
    vals = ti.load(x, (r, cols), mask=inside, other=-1.0e30)
    peak = ti.max(vals, 0)
    num = ti.exp(vals - peak)
    den = ti.sum(num, 0)
    ti.store(o, (r, cols), num / den, mask=inside)


# ---------------------------------------------------------------------------
# K3: tiled matmul, f16 inputs, f32 accumulation and output
# ---------------------------------------------------------------------------

@ti.jit
def tiled_matmul(
    a: ti.Buffer[ti.f16, (M, K), ti.ReadOnly],
    b: ti.Buffer[ti.f16, (K, N), ti.ReadOnly],
    c: ti.Buffer[ti.f32, (M, N), ti.WriteOnly],
    BM: ti.Const[int, ti.PowerOfTwo] = 128,
    BN: ti.Const[int, ti.PowerOfTwo] = 128,
    BK: ti.Const[int] = 64,
):
    tm = ti.program_id(0)
    tn = ti.program_id(1)
    rows = tm * BM + ti.arange(0, BM)
    cols = tn * BN + ti.arange(0, BN)
    ks = ti.arange(0, BK)
    row_ok = rows < M
    col_ok = cols < N
    total = ti.zeros((BM, BN), ti.f32)
    for k0 in ti.range(0, K, BK):
        kk = k0 + ks
        k_ok = kk < K
        lhs = ti.load(a, (rows[:, None], kk[None, :]), mask=row_ok[:, None] & k_ok[None, :])
        rhs = ti.load(b, (kk[:, None], cols[None, :]), mask=k_ok[:, None] & col_ok[None, :])
        total = ti.dot(lhs, rhs, acc=total)
    ti.store(c, (rows[:, None], cols[None, :]), total, mask=row_ok[:, None] & col_ok[None, :])


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
# K5: fused flash attention (non-causal), online softmax in the exp2 domain
# ---------------------------------------------------------------------------

@ti.jit
def flash_attention(
    q: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    k: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    v: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    o: ti.Buffer[ti.f32, (BH, L, BD), ti.WriteOnly],
    sm_scale: ti.f32 | ti.Positive,
    BM: ti.Const[int, ti.PowerOfTwo] = 128,
    BN: ti.Const[int, ti.PowerOfTwo] = 128,
    BD: ti.Const[int, ti.PowerOfTwo] = 128,
):
    qb = ti.program_id(0)
    h = ti.program_id(1)
    qi = qb * BM + ti.arange(0, BM)
    kn = ti.arange(0, BN)
    di = ti.arange(0, BD)
    q_ok = qi < L
    qt = ti.load(q, (h, qi[:, None], di[None, :]), mask=q_ok[:, None])
    scale2 = sm_scale * LOG2E
    m_run = ti.zeros((BM, 1), ti.f32) - 1.0e30
    l_run = ti.zeros((BM, 1), ti.f32)
    acc = ti.zeros((BM, BD), ti.f32)
    for n0 in ti.range(0, L, BN):
        ki = n0 + kn
        k_ok = ki < L
        kt = ti.load(k, (h, ki[None, :], di[:, None]), mask=k_ok[None, :])
        sc = ti.dot(qt, kt) * scale2 + ti.where(k_ok[None, :], 0.0, -1.0e6)
        m_blk = ti.max(sc, 1)[:, None]
        m_new = ti.where(m_blk > m_run, m_blk, m_run)
        corr = ti.exp2(m_run - m_new)
        pr = ti.exp2(sc - m_new)
        vt = ti.load(v, (h, ki[:, None], di[None, :]), mask=k_ok[:, None])
        l_blk = ti.sum(pr, 1)
        acc = acc * corr
        acc = ti.dot(ti.cast[ti.f16](pr), vt, acc=acc)
        l_run = l_run * corr + l_blk[:, None]
        m_run = m_new
    ti.store(o, (h, qi[:, None], di[None, :]), acc / l_run, mask=q_ok[:, None])


# ---------------------------------------------------------------------------
# causal variants (the adjacent kernels of the same examples: the CAUSAL=1
# branch of examples/fused_attention.py:62-103 and examples/self_attention.py)
# ---------------------------------------------------------------------------

@ti.jit
def flash_attention_causal(
    q: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    k: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    v: ti.Buffer[ti.f16, (BH, L, BD), ti.ReadOnly],
    o: ti.Buffer[ti.f32, (BH, L, BD), ti.WriteOnly],
    sm_scale: ti.f32 | ti.Positive,
    BM: ti.Const[int, ti.PowerOfTwo] = 64,
    BN: ti.Const[int, ti.PowerOfTwo] = 64,
    BD: ti.Const[int, ti.PowerOfTwo] = 64,
):
    # two stages: key blocks strictly below the diagonal band need no mask;
    # the band [qb*BM, qb*BM + BM) applies the causal mask as an additive bias
    qb = ti.program_id(0)
    h = ti.program_id(1)
    qi = qb * BM + ti.arange(0, BM)
    kn = ti.arange(0, BN)
    di = ti.arange(0, BD)
    q_ok = qi < L
    qt = ti.load(q, (h, qi[:, None], di[None, :]), mask=q_ok[:, None])
    scale2 = sm_scale * LOG2E
    m_run = ti.zeros((BM, 1), ti.f32) - 1.0e30
    l_run = ti.zeros((BM, 1), ti.f32)
    acc = ti.zeros((BM, BD), ti.f32)
    for n0 in ti.range(0, qb * BM, BN):
        ki = n0 + kn
        k_ok = ki < L
        kt = ti.load(k, (h, ki[None, :], di[:, None]), mask=k_ok[None, :])
        sc = ti.dot(qt, kt) * scale2
        m_blk = ti.max(sc, 1)[:, None]
        m_new = ti.where(m_blk > m_run, m_blk, m_run)
        corr = ti.exp2(m_run - m_new)
        pr = ti.exp2(sc - m_new)
        vt = ti.load(v, (h, ki[:, None], di[None, :]), mask=k_ok[:, None])
        l_blk = ti.sum(pr, 1)
        acc = acc * corr
        acc = ti.dot(ti.cast[ti.f16](pr), vt, acc=acc)
        l_run = l_run * corr + l_blk[:, None]
        m_run = m_new
    for n0 in ti.range(qb * BM, qb * BM + BM, BN):
        ki = n0 + kn
        k_ok = ki < L
        keep = (qi[:, None] >= ki[None, :]) & k_ok[None, :]
        kt = ti.load(k, (h, ki[None, :], di[:, None]), mask=k_ok[None, :])
        sc = ti.dot(qt, kt) * scale2 + ti.where(keep, 0.0, -1.0e6)
        m_blk = ti.max(sc, 1)[:, None]
        m_new = ti.where(m_blk > m_run, m_blk, m_run)
        corr = ti.exp2(m_run - m_new)
        pr = ti.exp2(sc - m_new)
        vt = ti.load(v, (h, ki[:, None], di[None, :]), mask=k_ok[:, None])
        l_blk = ti.sum(pr, 1)
        acc = acc * corr
        acc = ti.dot(ti.cast[ti.f16](pr), vt, acc=acc)
        l_run = l_run * corr + l_blk[:, None]
        m_run = m_new
    ti.store(o, (h, qi[:, None], di[None, :]), acc / l_run, mask=q_ok[:, None])


@ti.jit
def causal_self_attention(
    q: ti.Buffer[ti.f16, (M, BD), ti.ReadOnly],
    k: ti.Buffer[ti.f16, (N, BD), ti.ReadOnly],
    v: ti.Buffer[ti.f16, (N, BD), ti.ReadOnly],
    o: ti.Buffer[ti.f32, (M, BD), ti.WriteOnly],
    scale: ti.f32 | ti.Positive,
    BM: ti.Const[int, ti.PowerOfTwo] = 64,
    BN: ti.Const[int, ti.PowerOfTwo] = 64,
    BD: ti.Const[int, ti.PowerOfTwo] = 64,
):
    # one loop over every key block; masked scores are replaced (not biased)
    # and exp runs in the natural base
    qb = ti.program_id(0)
    qi = qb * BM + ti.arange(0, BM)
    kn = ti.arange(0, BN)
    di = ti.arange(0, BD)
    q_ok = qi < M
    qt = ti.load(q, (qi[:, None], di[None, :]), mask=q_ok[:, None])
    m_run = ti.zeros((BM, 1), ti.f32) - 1.0e30
    l_run = ti.zeros((BM, 1), ti.f32)
    acc = ti.zeros((BM, BD), ti.f32)
    for n0 in ti.range(0, N, BN):
        ki = n0 + kn
        k_ok = ki < N
        keep = (qi[:, None] >= ki[None, :]) & k_ok[None, :]
        kt = ti.load(k, (ki[None, :], di[:, None]), mask=k_ok[None, :] & (di[:, None] >= 0))
        sc = ti.where(keep, ti.dot(qt, kt) * scale, -1.0e30)
        m_blk = ti.max(sc, 1)[:, None]
        m_new = ti.where(m_blk > m_run, m_blk, m_run)
        corr = ti.exp(m_run - m_new)
        pr = ti.where(keep, ti.exp(sc - m_new), 0.0)
        vt = ti.load(v, (ki[:, None], di[None, :]), mask=k_ok[:, None])
        acc = acc * corr
        l_run = l_run * corr + ti.sum(pr, 1)[:, None]
        acc = ti.dot(ti.cast[ti.f16](pr), vt, acc=acc)
        m_run = m_new
    ti.store(o, (qi[:, None], di[None, :]), acc / l_run, mask=q_ok[:, None])


# ---------------------------------------------------------------------------
# configurations (the judged sizes) and their synthetic inputs
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
