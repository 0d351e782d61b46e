"""TIR semantics on B200 against the interpreter: dot accumulator rounding,
transcendental tolerance classes, the float cast matrix, wrapping integer
arithmetic with floor division, and NaN-propagating reductions.

Known answers and bounds follow the reference's GPU suites
(tests/test_m3_capabilities.py:15-30, tests/gpu_matrix_gaps.py:82-111,
tests/gpu_capabilities.py:34-75, tests/gpu_semantics.py).
"""

from pathlib import Path

import ml_dtypes
import numpy as np
import pytest
import torch

import tila_b200
import semantics_support as S

pytestmark = pytest.mark.gpu

NP = dict(f16=np.float16, bf16=ml_dtypes.bfloat16, f32=np.float32, f64=np.float64,
          i8=np.int8, i16=np.int16, i32=np.int32, i64=np.int64,
          u8=np.uint8, u16=np.uint16, u32=np.uint32, u64=np.uint64)
TORCH = dict(f16=torch.float16, bf16=torch.bfloat16, f32=torch.float32, f64=torch.float64,
             i8=torch.int8, i16=torch.int16, i32=torch.int32, i64=torch.int64,
             u8=torch.uint8, u16=torch.uint16, u32=torch.uint32, u64=torch.uint64)
KDIR = Path(__file__).resolve().parent / ".kernels"


def up(x, dt):
    if dt == "bf16":
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16).cuda()
    if x.flags.c_contiguous:
        return torch.from_numpy(x).cuda()
    return torch.from_numpy(np.ascontiguousarray(x.T)).cuda().T


def down(t):
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(ml_dtypes.bfloat16)
    return t.cpu().numpy()


def both(kernel, grid, inputs, dts, out_shape, out_dt, warps=4):
    cpu = np.zeros(out_shape, NP[out_dt])
    gpu = torch.zeros(out_shape, dtype=TORCH[out_dt], device="cuda")
    launch = kernel[grid].with_options(num_warps=warps)
    launch(*inputs, cpu)
    launch(*(up(x, d) for x, d in zip(inputs, dts)), gpu)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    return cpu, down(gpu)


@pytest.mark.parametrize("acc", ["f16", "f32"])
@pytest.mark.parametrize("case", ["rounding", "random"])
@pytest.mark.parametrize("strided", [False, True])
@pytest.mark.parametrize("warps", [4, 8])
def test_dot_accumulator(acc, case, strided, warps):
    kernel = S.dot_program(KDIR, acc)
    rng = np.random.default_rng(306)
    a = rng.normal(size=(16, 32)).astype(np.float16)
    b = rng.normal(size=(32, 16)).astype(np.float16)
    c = rng.normal(size=(16, 16)).astype(NP[acc])
    if case == "rounding":
        a[:] = 0
        b[:] = 0
        a[:, 0] = 1
        b[0, :] = np.resize(np.array([2**-11, 3 * 2**-11, -2**-12, 2**-10], np.float16), 16)
        c[:] = 1
    if strided:
        a, b, c = [np.ascontiguousarray(v.T).T for v in (a, b, c)]
    ref = a.astype(np.float64) @ b.astype(np.float64) + c.astype(np.float64)
    bound = 33 * np.finfo(np.float32).eps * (np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
                                             + np.abs(c.astype(np.float64)))
    if acc == "f16":
        bound += 2**-11 * (np.abs(ref) + bound) + 2**-24
    cpu, gpu = both(kernel, (1,), [a, b, c], ["f16", "f16", acc], (16, 16), "f32", warps)
    for out in (cpu, gpu):
        assert np.all(np.abs(out - ref) <= bound)
        if case == "rounding":
            np.testing.assert_array_equal(out, ref.astype(NP[acc]).astype(np.float32))
        if acc == "f16":
            np.testing.assert_array_equal(out, out.astype(np.float16).astype(np.float32))


SPECIALS = [-4, -1, -0.0, 0.0, 0.125, 0.5, 1, 4, -np.inf, np.inf, np.nan]


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32", "f64"])
@pytest.mark.parametrize("op", ["exp", "exp2"])
def test_exponentials(dtype, op):
    kernel = S.unary_program(KDIR, dtype, op)
    x = np.array(SPECIALS, dtype=NP[dtype])
    cpu, gpu = both(kernel, (2,), [x], [dtype], x.shape, dtype)
    ref = getattr(np, op)(x.astype(np.float64))
    tol = dict(f16=2**-9, bf16=2**-6, f32=2e-6, f64=2e-14)[dtype]
    for out in (cpu, gpu):
        np.testing.assert_allclose(out.astype(np.float64), ref, rtol=tol, atol=0, equal_nan=True)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("op", ["exp_widen", "exp2_widen"])
def test_narrow_exp_rounds_before_widening(dtype, op):
    kernel = S.unary_program(KDIR, dtype, op, out_dtype="f32")
    x = np.array([.125, .25, .5, .75, 1, 1.25, 1.5, 2], dtype=NP[dtype])
    cpu, gpu = both(kernel, (1,), [x], [dtype], (8,), "f32")
    fn = np.exp if op == "exp_widen" else np.exp2
    ref = fn(x.astype(np.float32)).astype(NP[dtype]).astype(np.float32)
    np.testing.assert_array_equal(cpu, ref)
    np.testing.assert_array_equal(gpu, ref)


@pytest.mark.parametrize("src", ["f16", "bf16", "f32", "f64"])
@pytest.mark.parametrize("dst", ["f16", "bf16", "f32", "f64"])
def test_float_cast_matrix(src, dst):
    kernel = S.unary_program(KDIR, src, "cast", dst, cast_to=dst)
    x = np.array([-np.inf, -3.5, -0.0, 0.0, .125, 1, 1.00390625, 1.00048828125, 65504, np.inf, np.nan],
                 dtype=NP[src])
    cpu, gpu = both(kernel, (2,), [x], [src], x.shape, dst)
    ref = x.astype(NP[dst])
    for out in (cpu, gpu):
        np.testing.assert_equal(out.astype(np.float64), ref.astype(np.float64))
        np.testing.assert_array_equal(np.signbit(out[2:4]), [True, False])


INTS = ["i8", "i16", "i32", "i64", "u8", "u16", "u32", "u64"]


@pytest.mark.parametrize("dtype", INTS)
def test_integer_add_wraps(dtype):
    kernel = S.unary_program(KDIR, dtype, "add1")
    info = np.iinfo(NP[dtype])
    x = np.array([info.min, info.min + 1, -1 if info.min < 0 else 1, 0, 1, info.max - 1, info.max,
                  7, 100], dtype=NP[dtype])
    bits = info.bits
    exp = [(int(v) + 1) % (1 << bits) for v in x]
    if info.min < 0:
        exp = [v - (1 << bits) if v >= 1 << (bits - 1) else v for v in exp]
    exp = np.array(exp, dtype=NP[dtype])
    if dtype == "i64":
        # the interpreter's own i64 wrap overflows under NumPy 2.x
        # (numeric.py:56-63); check the GPU against the exact expectation
        gpu = torch.zeros(x.shape, dtype=torch.int64, device="cuda")
        kernel[(2,)](up(x, dtype), gpu)
        np.testing.assert_array_equal(down(gpu), exp)
        return
    cpu, gpu = both(kernel, (2,), [x], [dtype], x.shape, dtype)
    np.testing.assert_array_equal(cpu, exp)
    np.testing.assert_array_equal(gpu, exp)


@pytest.mark.parametrize("dtype", ["i8", "i32", "u16", "u32"])
@pytest.mark.parametrize("op", ["+", "-", "*", "&", "|", "^"])
def test_integer_binary_bit_exact(dtype, op):
    kernel = S.binary_program(KDIR, dtype, op)
    info = np.iinfo(NP[dtype])
    rng = np.random.default_rng(307)
    n = 100
    x = rng.integers(info.min, info.max, size=n, dtype=NP[dtype], endpoint=True)
    y = rng.integers(info.min, info.max, size=n, dtype=NP[dtype], endpoint=True)
    cpu, gpu = both(kernel, (4,), [x, y], [dtype, dtype], (n,), dtype)
    np.testing.assert_array_equal(gpu, cpu)


@pytest.mark.parametrize("dtype", ["i8", "i16", "i32", "u16", "u32"])
@pytest.mark.parametrize("op", ["//", "%"])
@pytest.mark.parametrize("sign", [1, -1])
def test_floor_division_by_scalar(dtype, op, sign):
    info = np.iinfo(NP[dtype])
    if sign < 0 and info.min == 0:
        pytest.skip("unsigned divisors are positive")
    lo, hi = (1, 100) if sign > 0 else (-100, -1)
    kernel = S.scalar_div_program(KDIR, dtype, op, lo, hi)
    rng = np.random.default_rng(309)
    x = rng.integers(info.min, info.max, size=64, dtype=NP[dtype], endpoint=True)
    x[:3] = [info.min, info.max, 0]
    for d in ((7, 1, 64) if sign > 0 else (-7, -1, -64)):
        c = np.zeros_like(x)
        g = torch.zeros(x.shape, dtype=TORCH[dtype], device="cuda")
        kernel[(2,)](x, c, d)
        kernel[(2,)](up(x, dtype), g, d)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(down(g), c)
        # Python floor semantics, MIN // -1 wrapping to MIN
        py = [(int(v) // d if op == "//" else int(v) % d) for v in x]
        bits = info.bits
        py = [((v % (1 << bits)) - (1 << bits)) if info.min < 0 and (v % (1 << bits)) >= 1 << (bits - 1)
              else v % (1 << bits) for v in py]
        np.testing.assert_array_equal(c, np.array(py, dtype=NP[dtype]))


@pytest.mark.parametrize("dtype", ["f32", "i32"])
@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("axis", [0, 1])
def test_reductions(dtype, op, axis):
    kernel = S.reduce_program(KDIR, dtype, op, axis)
    rng = np.random.default_rng(308)
    m, n = 24, 50
    if dtype == "f32":
        x = rng.normal(size=(m, n)).astype(np.float32)
        x[3, 7] = np.nan
        x[10, 2] = np.inf
        x[11, :] = -0.0
    else:
        x = rng.integers(-2**31, 2**31 - 1, size=(m, n), dtype=np.int32)
    out_shape = (m,) if axis == 1 else (m // 8, n)
    cpu, gpu = both(kernel, (m // 8,), [x], [dtype], out_shape, dtype)
    if dtype == "f32":
        if op == "max":
            np.testing.assert_array_equal(gpu, cpu)       # max is exact, NaN propagates
        else:
            np.testing.assert_allclose(gpu, cpu, rtol=1e-5, atol=1e-5, equal_nan=True)
        assert np.isnan(gpu.reshape(-1)).any()
    else:
        np.testing.assert_array_equal(gpu, cpu)           # wrapping integer sum / max


def _division_cases(rng, n):
    """Dividends over every exponent and sign, plus zeros, subnormals,
    infinities, NaN and the ends of the range."""
    bits = rng.integers(0, 2**32, size=n, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32).copy()
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1.1754942e-38,
                        1.1754944e-38, 3.4028235e38, -3.4028235e38, 1.0, -1.0, 2.0**-60,
                        2.0**60, np.nextafter(np.float32(2.0**60), np.float32(0)),
                        np.nextafter(np.float32(2.0**-60), np.float32(0))], dtype=np.float32)
    x[: special.size] = special
    # dense band of ordinary values (the common case, all on the fast path)
    x[special.size: n // 2] = rng.normal(0.0, 1.0, n // 2 - special.size).astype(np.float32)
    return x


DIVISORS = [3.0, -7.25, 1.0 / 3.0, 0.1, 1e-30, 1e30, 2.0**-60, 2.0**60, 2.0**-61, 1.5 * 2.0**59,
            1e-40, 0.0, -0.0, float("inf"), float("nan"), 1.0, 65504.0, 6.1e-05]


def _same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    assert np.array_equal(nan, np.isnan(b))
    np.testing.assert_array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("kind", ["scalar", "reduced"])
def test_division_by_uniform_divisor_is_ieee(kind):
    """A divisor shared by a whole program (a scalar, or a row reduction
    broadcast) takes the reciprocal-and-correct path; every quotient must
    still be the IEEE f32 quotient, bit for bit, as NumPy computes it."""
    kernel = S.uniform_div_program(KDIR, kind)
    rng = np.random.default_rng(311)
    n = 1024 * len(DIVISORS)
    x = _division_cases(rng, n)
    out = torch.zeros(n, device="cuda")
    if kind == "scalar":
        for j, d in enumerate(DIVISORS):
            blk = x[j * 1024:(j + 1) * 1024].copy()
            g = torch.zeros(1024, device="cuda")
            kernel[(1,)](up(blk, "f32"), g, float(d))
            torch.cuda.synchronize()
            with np.errstate(all="ignore"):
                _same_bits(down(g), blk / np.float32(d))
    else:
        y = np.zeros((len(DIVISORS), 256), np.float32)
        y[:, 0] = np.array(DIVISORS, np.float32)
        cpu = np.zeros(n, np.float32)
        with np.errstate(all="ignore"):
            kernel[(len(DIVISORS),)](x, cpu, y)
        kernel[(len(DIVISORS),)](up(x, "f32"), out, up(y, "f32"))
        torch.cuda.synchronize()
        _same_bits(down(out), cpu)
        with np.errstate(all="ignore"):
            _same_bits(cpu, x / np.repeat(y.sum(1, dtype=np.float32), 1024))
    assert tila_b200.read_device_errors() == 0


def test_division_by_uniform_divisor_many_pairs():
    """Ten million random (dividend, divisor) pairs in the fast range against
    NumPy's IEEE quotients."""
    kernel = S.uniform_div_program(KDIR, "reduced")
    rng = np.random.default_rng(312)
    g = 8192
    n = 1024 * g
    e = rng.integers(-59, 59, size=n)
    x = (rng.uniform(1.0, 2.0, n) * np.exp2(e)).astype(np.float32) * rng.choice([-1, 1], n).astype(np.float32)
    d = (rng.uniform(1.0, 2.0, g) * np.exp2(rng.integers(-59, 59, size=g))).astype(np.float32)
    y = np.zeros((g, 256), np.float32)
    y[:, 0] = d
    out = torch.zeros(n, device="cuda")
    kernel[(g,)](up(x, "f32"), out, up(y, "f32"))
    torch.cuda.synchronize()
    _same_bits(down(out), x / np.repeat(d, 1024))


ATOMIC_NP = dict(i32=np.int32, u32=np.uint32, f32=np.float32)


@pytest.mark.parametrize("dtype", ["i32", "u32", "f32"])
@pytest.mark.parametrize("kind", ["buffer", "ptr"])
@pytest.mark.parametrize("count", [0, 5, 61, 64])
def test_atomic_tickets_and_tail(dtype, kind, count):
    """All lanes add 1 to x[0]: the old values are the tickets 0..count-1 in
    some order and the masked tail reads 0 (tests/gpu_atomic.py:23-40)."""
    kernel = S.atomic_program(KDIR, dtype, kind)
    npd = ATOMIC_NP[dtype]
    values = np.ones(64, npd)
    cpu, old_cpu = np.zeros(64, npd), np.zeros(64, npd)
    kernel[(2,)](cpu, values, old_cpu, COUNT=count)
    x = torch.zeros(64, dtype=TORCH[dtype], device="cuda")
    old = torch.zeros(64, dtype=TORCH[dtype], device="cuda")
    for _ in range(3):
        x.zero_()
        kernel[(2,)](x, up(values, dtype), old, COUNT=count)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(down(x), cpu)
        tickets = down(old)
        np.testing.assert_array_equal(np.sort(tickets[:count]), np.arange(count, dtype=npd))
        np.testing.assert_array_equal(tickets[count:], 0)
    assert tila_b200.read_device_errors() == 0


@pytest.mark.parametrize("dtype", ["i32", "u32", "f32"])
@pytest.mark.parametrize("kind", ["buffer", "ptr"])
def test_atomic_noncolliding(dtype, kind):
    """Each lane updates its own element: the result and the old values are
    deterministic and equal the interpreter's, wrapping at the integer ends."""
    kernel = S.atomic_program(KDIR, dtype, kind)
    npd = ATOMIC_NP[dtype]
    initial = np.arange(64).astype(npd)
    if dtype == "i32":
        initial[1] = 2**31 - 1
    if dtype == "u32":
        initial[1] = 2**32 - 1
    values = np.ones(64, npd)
    cpu, old_cpu = initial.copy(), np.zeros(64, npd)
    kernel[(2,)](cpu, values, old_cpu, COUNT=61, COLLIDE=False)
    x = up(initial.copy(), dtype)
    old = torch.zeros(64, dtype=TORCH[dtype], device="cuda")
    kernel[(2,)](x, up(values, dtype), old, COUNT=61, COLLIDE=False)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(down(x), cpu)
    np.testing.assert_array_equal(down(old), old_cpu)


@pytest.mark.parametrize("n", [1, 64, 100, 1000])
def test_ptr_form_load_store(n):
    """Ptr parameters with element offsets (x + i) load and store like the
    Buffer form, masked tail included."""
    kernel = S.ptr_copy_program(KDIR, "f32")
    x = np.random.default_rng(313).normal(size=n).astype(np.float32)
    cpu = np.zeros(n, np.float32)
    kernel[(-(-n // 64),)](x, cpu)
    out = torch.zeros(n, device="cuda")
    kernel[(-(-n // 64),)](up(x, "f32"), out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(down(out), cpu)
    np.testing.assert_array_equal(cpu, x + x)


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("axis", [0, 1, 2])
def test_rank3_tiles_match_interpreter(tmp_path, op, axis):
    """(4, 8, 16) tiles from reshape: element-wise work, a broadcast (4, 1, 16)
    operand and a reduction along each axis, against the interpreter."""
    k = S.rank3_program(tmp_path, op, axis)
    n_out = {0: 128, 1: 64, 2: 32}[axis]
    progs = 5
    rng = np.random.default_rng(40 + axis)
    x = rng.standard_normal(512 * progs - 37).astype(np.float32)
    w = rng.standard_normal(max(64, n_out) * progs).astype(np.float32)
    cpu = np.zeros_like(w)
    k[(progs,)](x, w, cpu)
    gpu = torch.zeros(w.size, device="cuda")
    k[(progs,)](torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), gpu)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    got = gpu.cpu().numpy()
    if op == "max":
        np.testing.assert_allclose(got, cpu, rtol=1e-6, atol=0)
    else:
        np.testing.assert_allclose(got, cpu, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n", [64, 300, 512])
def test_named_pointer_tiles_match_interpreter(tmp_path, n):
    """p = x + i and x + r[:, None] * 8 + c[None, :] bound to names, loaded
    and stored through Ptr parameters, bit-exact against the interpreter."""
    k = S.ptr_tile_program(tmp_path)
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    progs = -(-n // 64)
    c1, c2 = np.zeros(n, np.float32), np.zeros(n, np.float32)
    k[(progs,)](x, c1, c2)
    g1, g2 = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    k[(progs,)](torch.from_numpy(x).cuda(), g1, g2)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    np.testing.assert_array_equal(g1.cpu().numpy(), c1)
    np.testing.assert_array_equal(g2.cpu().numpy(), c2)


def test_expand_of_rank2_tiles_matches_interpreter(tmp_path):
    """Unit axes inserted at 0 and 1 of a (4, 8) tile broadcast against 3-D
    index tiles (src/tila/interp.py:305-307 expand semantics), bit-exact."""
    k = S.expand3_program(tmp_path)
    x = np.random.default_rng(7).standard_normal((4, 8)).astype(np.float32)
    c0, c1 = np.zeros((2, 4, 8), np.float32), np.zeros((4, 2, 8), np.float32)
    k[(1,)](x, c0, c1)
    g0, g1 = torch.zeros(2, 4, 8, device="cuda"), torch.zeros(4, 2, 8, device="cuda")
    k[(1,)](torch.from_numpy(x).cuda(), g0, g1)
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0
    np.testing.assert_array_equal(g0.cpu().numpy(), c0)
    np.testing.assert_array_equal(g1.cpu().numpy(), c1)
    np.testing.assert_array_equal(c0[1], x + 1.0)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f64"])
@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("axis", [0, 1])
def test_reductions_narrow_and_wide_floats(dtype, op, axis):
    """f16/bf16 sums accumulate in f32 and round once to the input type;
    f64 stays f64; max is exact and propagates NaN (interp.py:324-333,
    ADR-008)."""
    kernel = S.reduce_program(KDIR, dtype, op, axis)
    rng = np.random.default_rng(309)
    m, n = 24, 50
    x = rng.normal(size=(m, n)).astype(np.float32).astype(NP[dtype])
    x[3, 7] = np.nan
    x[11, :] = -0.0
    out_shape = (m,) if axis == 1 else (m // 8, n)
    cpu, gpu = both(kernel, (m // 8,), [x], [dtype], out_shape, dtype)
    c, g = np.asarray(cpu, np.float64), np.asarray(gpu, np.float64)
    assert np.array_equal(np.isnan(c), np.isnan(g)) and np.isnan(g).any()
    if op == "max":
        np.testing.assert_array_equal(g, c)
    else:
        # one rounding of the f32 (f64) sum: orders of summation may differ by
        # an ulp of the accumulator, which the final rounding usually hides
        ulp = {"f16": 2.0 ** -10, "bf16": 2.0 ** -7, "f64": 2.0 ** -50}[dtype]
        np.testing.assert_allclose(g, c, rtol=2 * ulp, atol=2 * ulp, equal_nan=True)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f64"])
@pytest.mark.parametrize("op", ["+", "-", "*", "/"])
def test_float_binary_correctly_rounded(dtype, op):
    """Narrow floats compute in f32 and round once; f32 carries more than
    2p+2 bits for p = 11 and p = 8, so the result is the correctly rounded
    narrow operation, bit for bit the interpreter's."""
    kernel = S.binary_program(KDIR, dtype, op)
    rng = np.random.default_rng(311)
    n = 100
    x = (rng.normal(size=n) * 8).astype(np.float32).astype(NP[dtype])
    y = (rng.normal(size=n) * 8).astype(np.float32).astype(NP[dtype])
    x[:6] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1.0]
    y[:6] = [0.0, 0.0, np.inf, 2.0, 1.0, -0.0]
    cpu, gpu = both(kernel, (4,), [x, y], [dtype, dtype], (n,), dtype)
    nan = np.isnan(np.asarray(cpu, np.float64))
    assert np.array_equal(nan, np.isnan(np.asarray(gpu, np.float64)))
    bits = {"f16": np.uint16, "bf16": np.uint16, "f64": np.uint64}[dtype]
    np.testing.assert_array_equal(gpu[~nan].view(bits), cpu[~nan].view(bits))
