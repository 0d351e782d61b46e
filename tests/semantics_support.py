"""Small Tila programs that pin down TIR semantics, generated per dtype.

Tila reads a kernel's source with ``inspect.getsource``, so each program is
written to a module file and imported.  Used by the GPU semantics tests (B200
against the interpreter) and by the CPU code-generation tests.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import tila_b200  # noqa: F401  (installs the backend, makes `tila` importable)

_CACHE = {}


def load_source(directory: Path, name: str, source: str):
    key = (name, source)
    if key in _CACHE:
        return _CACHE[key]
    directory.mkdir(parents=True, exist_ok=True)
    path = directory / f"{name}.py"
    path.write_text(source)
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    _CACHE[key] = module.kernel
    return module.kernel


def dot_program(directory, acc="f16"):
    """out = f32(dot(a, b, acc=c)) on 16x32 @ 32x16 tiles; with an f16
    accumulator the dot result is rounded to f16 before the widening cast."""
    return load_source(directory, f"sem_dot_{acc}", f'''import tila as ti

@ti.jit
def kernel(a: ti.Buffer[ti.f16, (16, 32), ti.ReadOnly],
           b: ti.Buffer[ti.f16, (32, 16), ti.ReadOnly],
           c: ti.Buffer[ti.{acc}, (16, 16), ti.ReadOnly],
           out: ti.Buffer[ti.f32, (16, 16), ti.WriteOnly]):
    r = ti.arange(0, 16)
    kk = ti.arange(0, 32)
    lhs = ti.load(a, (r[:, None], kk[None, :]))
    rhs = ti.load(b, (kk[:, None], r[None, :]))
    init = ti.load(c, (r[:, None], r[None, :]))
    ti.store(out, (r[:, None], r[None, :]), ti.cast[ti.f32](ti.dot(lhs, rhs, acc=init)))
''')


UNARY = {"copy": "v", "exp": "ti.exp(v)", "exp2": "ti.exp2(v)", "neg": "-v",
         "add1": "v + 1", "exp_widen": "ti.cast[ti.f32](ti.exp(v))",
         "exp2_widen": "ti.cast[ti.f32](ti.exp2(v))"}


def unary_program(directory, dtype, op, out_dtype=None, cast_to=None):
    """Element-wise program over a length-N vector in 8-wide programs."""
    out_dtype = out_dtype or dtype
    expr = f"ti.cast[ti.{cast_to}](v)" if cast_to else UNARY[op]
    name = f"sem_un_{dtype}_{op}_{out_dtype}_{cast_to}"
    return load_source(directory, name, f'''import tila as ti
N = ti.Dim("N")

@ti.jit
def kernel(x: ti.Buffer[ti.{dtype}, (N,), ti.ReadOnly],
           out: ti.Buffer[ti.{out_dtype}, (N,), ti.WriteOnly]):
    i = ti.program_id(0) * 8 + ti.arange(0, 8)
    ok = i < N
    v = ti.load(x, i, mask=ok)
    ti.store(out, i, {expr}, mask=ok)
''')


def binary_program(directory, dtype, op):
    name = f"sem_bin_{dtype}_{op.replace('/', 'div').replace('%', 'mod').replace('*', 'mul').replace('+', 'add').replace('-', 'sub').replace('<', 'shl').replace('>', 'shr').replace('&', 'and').replace('|', 'or').replace('^', 'xor')}"
    return load_source(directory, name, f'''import tila as ti
N = ti.Dim("N")

@ti.jit
def kernel(x: ti.Buffer[ti.{dtype}, (N,), ti.ReadOnly],
           y: ti.Buffer[ti.{dtype}, (N,), ti.ReadOnly],
           out: ti.Buffer[ti.{dtype}, (N,), ti.WriteOnly]):
    i = ti.program_id(0) * 32 + ti.arange(0, 32)
    ok = i < N
    a = ti.load(x, i, mask=ok)
    b = ti.load(y, i, mask=ok)
    ti.store(out, i, a {op} b, mask=ok)
''')


def reduce_program(directory, dtype, op, axis):
    """Reduce an (R, 64) tile along ``axis`` (rows of 8 x 64 per program)."""
    name = f"sem_red_{dtype}_{op}_{axis}"
    if axis == 1:
        body = f'''    t = ti.load(x, (r[:, None], c[None, :]), mask=(r[:, None] < M) & (c[None, :] < N))
    red = ti.{op}(t, 1)
    ti.store(out, (r,), red, mask=r < M)'''
        out_shape = "(M,)"
    else:
        body = f'''    t = ti.load(x, (r[:, None], c[None, :]), mask=(r[:, None] < M) & (c[None, :] < N))
    red = ti.{op}(t, 0)
    ti.store(out, (pid, c), red, mask=c < N)'''
        out_shape = "(G, N)"
    return load_source(directory, name, f'''import tila as ti
M = ti.Dim("M")
N = ti.Dim("N")
G = ti.Dim("G")

@ti.jit
def kernel(x: ti.Buffer[ti.{dtype}, (M, N), ti.ReadOnly],
           out: ti.Buffer[ti.{dtype}, {out_shape}, ti.WriteOnly]):
    pid = ti.program_id(0)
    r = pid * 8 + ti.arange(0, 8)
    c = ti.arange(0, 64)
{body}
''')


def scalar_div_program(directory, dtype, op, lo, hi):
    """x // d or x % d with a divisor the launch contract bounds away from 0
    (Tila rejects a data-dependent divisor it cannot prove nonzero)."""
    tag = "div" if op == "//" else "mod"
    sign = "neg" if hi < 0 else "pos"
    return load_source(directory, f"sem_sdiv_{dtype}_{tag}_{sign}", f'''import tila as ti
N = ti.Dim("N")

@ti.jit
def kernel(x: ti.Buffer[ti.{dtype}, (N,), ti.ReadOnly],
           out: ti.Buffer[ti.{dtype}, (N,), ti.WriteOnly],
           d: ti.{dtype} | ti.Range[{lo}, {hi}]):
    i = ti.program_id(0) * 32 + ti.arange(0, 32)
    ok = i < N
    a = ti.load(x, i, mask=ok)
    ti.store(out, i, a {op} d, mask=ok)
''')


def uniform_div_program(directory, kind):
    """x / d where every element of a program divides by the same value: a
    scalar parameter, or the sum of a row of ``y`` (one value per program)."""
    if kind == "scalar":
        params = "d: ti.f32"
        divisor = "d"
    else:
        params = "y: ti.Buffer[ti.f32, (G, 256), ti.ReadOnly]"
        divisor = "ti.sum(ti.load(y, (pid, ti.arange(0, 256))), 0)"
    return load_source(directory, f"sem_udiv_{kind}", f'''import tila as ti
N = ti.Dim("N")
G = ti.Dim("G")

@ti.jit
def kernel(x: ti.Buffer[ti.f32, (N,), ti.ReadOnly],
           out: ti.Buffer[ti.f32, (N,), ti.WriteOnly],
           {params}):
    pid = ti.program_id(0)
    i = pid * 1024 + ti.arange(0, 1024)
    ok = i < N
    ti.store(out, i, ti.load(x, i, mask=ok) / {divisor}, mask=ok)
''')


def atomic_program(directory, dtype="i32", kind="buffer"):
    """Every lane adds ``values[i]`` to x[offset] (offset 0 for all lanes, or
    its own lane) and stores the old value it saw; ``kind`` selects the
    Buffer form (x, offset) or the Ptr form (x + offset)."""
    annotation = (f"ti.Buffer[ti.{dtype}, (64,), ti.ReadWrite]" if kind == "buffer"
                  else f"ti.RWPtr[ti.{dtype}, 64]")
    target = "x, offset" if kind == "buffer" else "x + offset"
    return load_source(directory, f"sem_atomic_{dtype}_{kind}", f'''import tila as ti

@ti.jit
def kernel(x: {annotation}, values: ti.Buffer[ti.{dtype}, (64,), ti.ReadOnly],
           old: ti.Buffer[ti.{dtype}, (64,), ti.WriteOnly],
           COUNT: ti.Const[int] = 64, COLLIDE: ti.Const[bool] = True):
    i = ti.program_id(0) * 32 + ti.arange(0, 32)
    if COLLIDE:
        offset = i * 0
    else:
        offset = i
    value = ti.load(values, i, mask=i < COUNT, other=0)
    before = ti.atomic_add({target}, value, mask=i < COUNT)
    ti.store(old, i, before, mask=i < 64)
''')


def ptr_copy_program(directory, dtype="f32"):
    """out[i] = 2 * x[i] through Ptr parameters (x + i, out + i)."""
    return load_source(directory, f"sem_ptr_copy_{dtype}", f'''import tila as ti
N = ti.Dim("N")

@ti.jit
def kernel(x: ti.ReadPtr[ti.{dtype}, N], out: ti.WritePtr[ti.{dtype}, N]):
    i = ti.program_id(0) * 64 + ti.arange(0, 64)
    ok = i < N
    v = ti.load(x + i, mask=ok, other=0)
    ti.store(out + i, v + v, mask=ok)
''')


def batched_matmul_program(directory):
    """c[h] = a[h] @ b[h] over a 3-D grid (row tile, column tile, batch):
    the batch axis keeps the block from being coarsened, so the kernel uses
    the per-program pipelined contraction ring."""
    return load_source(directory, "sem_bmm", '''import tila as ti
B = ti.Dim("B")
M = ti.Dim("M")
N = ti.Dim("N")
K = ti.Dim("K")

@ti.jit
def kernel(a: ti.Buffer[ti.f16, (B, M, K), ti.ReadOnly],
           b: ti.Buffer[ti.f16, (B, K, N), ti.ReadOnly],
           c: ti.Buffer[ti.f32, (B, M, N), ti.WriteOnly],
           BM: ti.Const[int, ti.PowerOfTwo] = 128,
           BN: ti.Const[int, ti.PowerOfTwo] = 128,
           BK: ti.Const[int] = 64):
    tm = ti.program_id(0)
    tn = ti.program_id(1)
    h = ti.program_id(2)
    rows = tm * BM + ti.arange(0, BM)
    cols = tn * BN + ti.arange(0, BN)
    ks = ti.arange(0, BK)
    row_ok = rows < M
    col_ok = cols < N
    total = ti.zeros((BM, BN), ti.f32)
    for k0 in ti.range(0, K, BK):
        kk = k0 + ks
        k_ok = kk < K
        lhs = ti.load(a, (h, rows[:, None], kk[None, :]), mask=row_ok[:, None] & k_ok[None, :])
        rhs = ti.load(b, (h, kk[:, None], cols[None, :]), mask=k_ok[:, None] & col_ok[None, :])
        total = ti.dot(lhs, rhs, acc=total)
    ti.store(c, (h, rows[:, None], cols[None, :]), total, mask=row_ok[:, None] & col_ok[None, :])
''')


def rank3_program(directory, op="sum", axis=2):
    """512-element blocks reshaped to (4, 8, 16) tiles, reduced along one
    axis (sum or max, after an element-wise exp / scale and a product with a
    (4, 1, 16) broadcast operand), reshaped back to 1-D and stored."""
    keep = [d for i, d in enumerate((4, 8, 16)) if i != axis]
    n_out = keep[0] * keep[1]
    body = "ti.exp(t * 0.25)" if op == "max" else "t * 2.0"
    return load_source(directory, f"sem_r3_{op}_{axis}", f'''import tila as ti
N = ti.Dim("N")
M = ti.Dim("M")

@ti.jit
def kernel(x: ti.Buffer[ti.f32, (N,), ti.ReadOnly],
           w: ti.Buffer[ti.f32, (M,), ti.ReadOnly],
           out: ti.Buffer[ti.f32, (M,), ti.WriteOnly]):
    pid = ti.program_id(0)
    i = pid * 512 + ti.arange(0, 512)
    v = ti.load(x, i, mask=i < N, other=0.0)
    k = pid * 64 + ti.arange(0, 64)
    g = ti.load(w, k, mask=k < M, other=1.0)
    t = ti.reshape(v, (4, 8, 16))
    b = ti.reshape(g, (4, 1, 16))
    s = ti.{op}({body} * b, {axis})
    u = ti.reshape(s, ({n_out},))
    j = pid * {n_out} + ti.arange(0, {n_out})
    ti.store(out, j, u, mask=j < M)
''')


def assume_gather_program(directory):
    """The reference's gather (tests/test_bounds.py:144-163) with a second,
    stricter assumption ``idx < limit`` that the caller can make false while
    every index stays inside the buffer."""
    return load_source(directory, "sem_assume_gather", '''import tila as ti
N = ti.Dim("N")

@ti.jit
def kernel(idx_buf: ti.Buffer[ti.i32, (N,), ti.ReadOnly],
           data: ti.Buffer[ti.f32, (N,), ti.ReadOnly],
           out: ti.Buffer[ti.f32, (N,), ti.WriteOnly],
           limit: ti.i32,
           BLOCK: ti.Const[int, ti.PowerOfTwo] = 64):
    pid = ti.program_id(0)
    offs = pid * BLOCK + ti.arange(0, BLOCK)
    m = offs < N
    idx = ti.load(idx_buf, offs, mask=m, other=0)
    ti.assume((idx >= 0) & (idx < N))
    ti.assume(idx < limit)
    v = ti.load(data, idx)
    ti.store(out, offs, v, mask=m)
''')


def expand3_program(directory):
    """expand of 2-D tiles (x[None, :] and x[:, None] insert a unit axis at 0
    and 1) broadcast against 3-D tiles built by chained expands."""
    return load_source(directory, "sem_expand3", '''import tila as ti


@ti.jit
def kernel(x: ti.Buffer[ti.f32, (4, 8), ti.ReadOnly],
           o0: ti.Buffer[ti.f32, (2, 4, 8), ti.WriteOnly],
           o1: ti.Buffer[ti.f32, (4, 2, 8), ti.WriteOnly]):
    r = ti.arange(0, 4)
    c = ti.arange(0, 8)
    k = ti.arange(0, 2)
    t = ti.load(x, (r[:, None], c[None, :]))
    kf = ti.cast[ti.f32](k)
    ti.store(o0, (k[:, None][:, None], r[:, None][None, :], c[None, :][None, :]),
             t[None, :] + kf[:, None][:, None])
    ti.store(o1, (r[:, None][:, None], k[:, None][None, :], c[None, :][None, :]),
             t[:, None] * 2.0 + kf[:, None][None, :])
''')


def ptr_tile_program(directory):
    """Pointer tiles bound to names: a 1-D tile (p = x + i) and a 2-D tile
    built from an expanded index (x + r[:, None] * 8 + c[None, :])."""
    return load_source(directory, "sem_ptr_tiles", '''import tila as ti
N = ti.Dim("N")


@ti.jit
def kernel(x: ti.ReadPtr[ti.f32, N], out: ti.WritePtr[ti.f32, N], out2: ti.WritePtr[ti.f32, N]):
    i = ti.program_id(0) * 64 + ti.arange(0, 64)
    ok = i < N
    p = x + i
    q = out + i
    v = ti.load(p, mask=ok, other=0)
    ti.store(q, v * 3.0, mask=ok)
    r = ti.program_id(0) * 8 + ti.arange(0, 8)
    c = ti.arange(0, 8)
    j = r[:, None] * 8 + c[None, :]
    ok2 = j < N
    p2 = x + j
    w = ti.load(p2, mask=ok2, other=0)
    ti.store(out2 + j, w + 1.0, mask=ok2)
''')
