"""NumPy restatement of the five workloads - TEST INFRASTRUCTURE ONLY.

Each function restates what the Tila program computes on the interpreter,
citing the reference semantics it follows.  The f32 functions reproduce the
interpreter's arithmetic (same NumPy calls in the same order) so they can
stand in for it where its per-program loop would take minutes; the f64
functions are the exact references that the reference's GPU tests bound
against (tests/gpu_examples.py:28-97).
"""

from __future__ import annotations

import numpy as np


def vector_add(x, y):
    """out = x + y in f32 (examples/add_kernel.py:21-27; interp.py:199-235)."""
    return (np.asarray(x, np.float32) + np.asarray(y, np.float32)).astype(np.float32)


def row_softmax_f32(x, bn):
    """Row softmax as the interpreter runs examples/softmax.py:14-29 with a
    BN-wide tile: masked tail lanes load -1e30 (interp.py:171-176), max,
    f32 exp (interp.py:265-269), pairwise f32 sum over the BN lanes
    (interp.py:324-333), IEEE f32 division."""
    x = np.asarray(x, np.float32)
    m, n = x.shape
    tile = np.full((m, bn), np.float32(-1.0e30), dtype=np.float32)
    tile[:, :n] = x
    out = np.empty_like(x)
    for r in range(m):
        v = tile[r]
        mx = np.max(v, axis=0)
        e = np.asarray(np.exp(np.asarray(v - mx, dtype=np.float32)), dtype=np.float32)
        s = np.asarray(np.sum(e, axis=0, dtype=np.float32)).astype(np.float32)
        out[r] = (e / s)[:n]
    return out


def row_softmax_f64(x):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def matmul_f64(a, b):
    return np.asarray(a, np.float64) @ np.asarray(b, np.float64)


def matmul_bound(a, b):
    """|C - A B| <= K * eps_f32 * |A| |B|: f16 products are exact in f32, so
    only the f32 accumulation rounds (tests/gpu_examples.py:52-64)."""
    k = a.shape[1]
    return (k * np.finfo(np.float32).eps) * (np.abs(np.asarray(a, np.float64)) @
                                            np.abs(np.asarray(b, np.float64)))


def attention_f64(q, k, v, scale=None, causal=False):
    """softmax(Q K^T * scale) V in f64, optionally with the causal mask
    (tests/gpu_examples.py:67-73)."""
    q64, k64, v64 = (np.asarray(t, np.float64) for t in (q, k, v))
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    s = q64 @ k64.swapaxes(-1, -2) * scale
    if causal:
        s = np.where(np.tril(np.ones(s.shape[-2:], bool)), s, -np.inf)
    p = np.exp(s - s.max(axis=-1, keepdims=True))
    p /= p.sum(axis=-1, keepdims=True)
    return p @ v64


def rel_frobenius(actual, expected):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-300))
