"""GPU parity of the five workloads against Tila's interpreter (the oracle).

Mirrors the reference's differential tests (tests/gpu_examples.py:19-97):
fixed seeds, the CPU interpreter and the B200 backend run the same program on
the same inputs.  Bars: bit-exact for add; rtol 1e-6 against the interpreter
for softmax; relative Frobenius error <= 2e-3 for the f16-dot kernels (plus
the K * eps_f32 elementwise bound of the reference for matmul).
"""

import numpy as np
import pytest

import tila_b200
from tila_b200 import workloads as W
from oracle import restate

ti = tila_b200.tila
torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a) if a.flags.c_contiguous else a).cuda() \
        if a.flags.c_contiguous else torch.from_numpy(np.ascontiguousarray(a.T)).cuda().T


def _no_device_errors():
    torch.cuda.synchronize()
    assert tila_b200.read_device_errors() == 0


def execute(kernel, grid, inputs, out_shape, *scalars, warps=4, **consts):
    """Run on the interpreter (NumPy) and on the B200 backend (CUDA)."""
    cpu = np.zeros(out_shape, np.float32)
    gpu = torch.zeros(out_shape, dtype=torch.float32, device="cuda")
    launch = kernel[grid].with_options(num_warps=warps)
    launch(*inputs, cpu, *scalars, **consts)
    launch(*(_cuda(x) for x in inputs), gpu, *scalars, **consts)
    _no_device_errors()
    return cpu, gpu.cpu().numpy()


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("n", [127, 128, 129])
def test_add_bit_exact(n, warps):
    rng = np.random.default_rng(301)
    x, y = [rng.normal(size=n).astype(np.float32) for _ in range(2)]
    cpu, gpu = execute(W.add_kernel, (ti.cdiv(n, 128),), [x, y], (n,), warps=warps, BLOCK=128)
    np.testing.assert_array_equal(cpu, x + y)
    np.testing.assert_array_equal(gpu, cpu)


def test_add_full_size_bit_exact():
    x, y = W.add_inputs()
    out = torch.zeros(x.shape, dtype=torch.float32, device="cuda")
    W.add_kernel[(ti.cdiv(x.size, 1024),)](_cuda(x), _cuda(y), out, BLOCK=1024)
    _no_device_errors()
    np.testing.assert_array_equal(out.cpu().numpy(), restate.vector_add(x, y))


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("n", [31, 32, 33])
def test_softmax(n, warps):
    x = np.random.default_rng(302).normal(size=(3, n)).astype(np.float32)
    cpu, gpu = execute(W.softmax_kernel, (3,), [x], x.shape, warps=warps, BN=64)
    ref = restate.row_softmax_f64(x)
    np.testing.assert_allclose(gpu, ref, rtol=2e-6, atol=2e-7)
    np.testing.assert_allclose(gpu, cpu, rtol=1e-6, atol=0)


def test_softmax_full_size():
    x = W.softmax_inputs()
    out = torch.zeros(x.shape, dtype=torch.float32, device="cuda")
    W.softmax_kernel[(x.shape[0],)](_cuda(x), out, BN=1024)
    _no_device_errors()
    got = out.cpu().numpy()
    # the interpreter's arithmetic restated (bit-for-bit the same NumPy calls)
    ref = restate.row_softmax_f32(x[:512], 1024)
    np.testing.assert_allclose(got[:512], ref, rtol=1e-6, atol=0)
    # every row sums to one (size-independent property over all rows)
    np.testing.assert_allclose(got.astype(np.float64).sum(axis=1), 1.0, rtol=1e-5)


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("shape", [(16, 16, 16), (19, 23, 35)])
@pytest.mark.parametrize("strided", [False, True])
def test_matmul_small(shape, strided, warps):
    m, n, k = shape
    rng = np.random.default_rng(303)
    a = rng.normal(size=(m, k)).astype(np.float16)
    b = rng.normal(size=(k, n)).astype(np.float16)
    if strided:
        a = np.ascontiguousarray(a.T).T
        b = np.ascontiguousarray(b.T).T
    cpu, gpu = execute(W.matmul_kernel, (ti.cdiv(m, 16), ti.cdiv(n, 16)), [a, b], (m, n),
                       warps=warps, BM=16, BN=16, BK=32)
    ref = restate.matmul_f64(a, b)
    bound = restate.matmul_bound(a, b)
    assert np.all(np.abs(gpu - ref) <= bound)
    assert restate.rel_frobenius(gpu, cpu) <= 2e-3


@pytest.mark.parametrize("shape", [(256, 256, 256), (300, 200, 136)])
def test_matmul_128_tiles(shape):
    m, n, k = shape
    a, b = W.matmul_inputs(m, n, k, seed=7)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    W.matmul_kernel[(ti.cdiv(m, 128), ti.cdiv(n, 128))](_cuda(a), _cuda(b), c, BM=128, BN=128, BK=64)
    _no_device_errors()
    got = c.cpu().numpy()
    assert np.all(np.abs(got - restate.matmul_f64(a, b)) <= restate.matmul_bound(a, b))


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("n", [32, 65])
def test_fused_attention_small(n, warps):
    rng = np.random.default_rng(305)
    q, k, v = [rng.normal(size=(2, n, 32)).astype(np.float16) for _ in range(3)]
    cpu, gpu = execute(W.fused_attention_kernel, (ti.cdiv(n, 32), 2), [q, k, v], (2, n, 32),
                       1 / np.sqrt(32), warps=warps, CAUSAL=0, BM=32, BN=32, BD=32)
    ref = restate.attention_f64(q, k, v)
    np.testing.assert_allclose(gpu, ref, rtol=2e-3, atol=2e-3)
    assert restate.rel_frobenius(gpu, cpu) <= 2e-3


def test_fused_attention_128_tiles():
    q, k, v = W.attention_inputs(2, 384, 128, seed=11)
    o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    W.fused_attention_kernel[(ti.cdiv(384, 128), 2)](_cuda(q), _cuda(k), _cuda(v), o, 128 ** -0.5,
                                              CAUSAL=0, BM=128, BN=128, BD=128)
    _no_device_errors()
    assert restate.rel_frobenius(o.cpu().numpy(), restate.attention_f64(q, k, v)) <= 2e-3


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("l,d", [(300, 64), (300, 128), (128, 128), (1000, 128)])
def test_fused_attention_ragged_128_tiles(l, d, warps):
    """128x128 tiles (two programs per CTA, pipelined score MMAs; with 8
    warps each program's rows are split into two column halves) with a
    partial last key block, a partial last query block, and odd numbers of
    query blocks (a CTA whose second program does not exist)."""
    q, k, v = W.attention_inputs(3, l, d, seed=13)
    o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    W.fused_attention_kernel[(ti.cdiv(l, 128), 3)].with_options(num_warps=warps)(
        _cuda(q), _cuda(k), _cuda(v), o, d ** -0.5, CAUSAL=0, BM=128, BN=128, BD=d)
    _no_device_errors()
    assert restate.rel_frobenius(o.cpu().numpy(), restate.attention_f64(q, k, v)) <= 2e-3


@pytest.mark.parametrize("l,d,blk", [(65, 32, 32), (256, 64, 128), (200, 64, 128)])
def test_unfused_attention(l, d, blk):
    bh = 2
    q, k, v = W.attention_inputs(bh, l, d, seed=12)
    scale = d ** -0.5
    qg, kg, vg = (_cuda(t) for t in (q, k, v))
    s = torch.zeros((bh, l, l), dtype=torch.float32, device="cuda")
    p = torch.zeros_like(s)
    o = torch.zeros((bh, l, d), dtype=torch.float32, device="cuda")
    W.attention_scores[(ti.cdiv(l, blk), ti.cdiv(l, blk), bh)](qg, kg, s, scale, BM=blk, BN=blk, BD=d)
    bn = 1 << (l - 1).bit_length()
    W.softmax_kernel[(bh * l,)](s.view(bh * l, l), p.view(bh * l, l), BN=max(bn, 16))
    W.attention_pv[(ti.cdiv(l, blk), bh)](p, vg, o, BM=blk, BN=blk, BD=d)
    _no_device_errors()
    ref = restate.attention_f64(q, k, v, scale)
    assert restate.rel_frobenius(o.cpu().numpy(), ref) <= 2e-3
    # scores against the f64 product (f16 inputs are exact in f32 products)
    s_ref = np.asarray(q, np.float64) @ np.asarray(k, np.float64).swapaxes(-1, -2) * scale
    assert restate.rel_frobenius(s.cpu().numpy(), s_ref) <= 1e-5


@pytest.mark.parametrize("world", [2, 3])
def test_program_range_shards_reproduce_the_full_launch(world):
    """Each rank's share of the grid (run here one after another on one GPU)
    writes exactly the rows the full launch writes."""
    from tila_b200.multigpu import shard
    x = torch.from_numpy(W.softmax_inputs(300, 1000, seed=13)).cuda()
    full = torch.zeros_like(x)
    W.softmax_kernel[(300,)](x, full, BN=1024)
    parts = torch.full_like(x, float("nan"))
    for rank in range(world):
        with shard(0, 300, world, rank):
            W.softmax_kernel[(300,)](x, parts, BN=1024)
    _no_device_errors()
    assert torch.equal(parts, full)
    a, b = W.matmul_inputs(384, 256, 128, seed=14)
    ag, bg = _cuda(a), _cuda(b)
    c_full = torch.zeros((384, 256), device="cuda")
    W.matmul_kernel[(3, 2)](ag, bg, c_full, BM=128, BN=128, BK=64)
    c_part = torch.full_like(c_full, float("nan"))
    for rank in range(world):
        with shard(0, 3, world, rank):
            W.matmul_kernel[(3, 2)](ag, bg, c_part, BM=128, BN=128, BK=64)
    _no_device_errors()
    assert torch.equal(c_part, c_full)


@pytest.mark.parametrize("world", [2, 3])
def test_causal_attention_head_shards_reproduce_the_full_launch(world):
    """The warp-specialised causal kernel launched per shard of the head axis
    (as bench.py --gpus N shards it; CTA renumbering within each shard's
    grid): the shards together write exactly the full launch's output."""
    from tila_b200.multigpu import shard
    q, k, v = W.attention_inputs(11, 640, 128, seed=31)
    qg, kg, vg = _cuda(q), _cuda(k), _cuda(v)
    full = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    W.fused_attention_kernel[(5, 11)](qg, kg, vg, full, 128 ** -0.5, CAUSAL=1, BM=128, BN=128, BD=128)
    parts = torch.full_like(full, float("nan"))
    for rank in range(world):
        with shard(1, 11, world, rank):
            W.fused_attention_kernel[(5, 11)](qg, kg, vg, parts, 128 ** -0.5, CAUSAL=1, BM=128, BN=128, BD=128)
    _no_device_errors()
    assert torch.equal(parts, full)


def test_program_shards_write_the_rows_shard_rows_names():
    """3 matmul tile rows of 128 on 2 ranks (programs [0, 2) and [2, 3)): each
    rank's launch writes exactly the rows multigpu.shard_rows gives it (0-255
    and 256-383, not a split of the 384 rows), which is what gather_leading
    collects."""
    from tila_b200.multigpu import shard, shard_rows
    a, b = W.matmul_inputs(384, 256, 128, seed=15)
    ag, bg = _cuda(a), _cuda(b)
    full = torch.zeros((384, 256), device="cuda")
    W.matmul_kernel[(3, 2)](ag, bg, full, BM=128, BN=128, BK=64)
    rows = shard_rows(3, 128, 384, 2)
    assert rows == [(0, 256), (256, 384)]
    for rank, (lo, hi) in enumerate(rows):
        part = torch.full_like(full, float("nan"))
        with shard(0, 3, 2, rank):
            W.matmul_kernel[(3, 2)](ag, bg, part, BM=128, BN=128, BK=64)
        _no_device_errors()
        written = ~torch.isnan(part).all(dim=1)
        assert written.nonzero().flatten().tolist() == list(range(lo, hi))
        assert torch.equal(part[lo:hi], full[lo:hi])


def test_repeated_signature_launches_skip_checks_and_use_new_buffers():
    """A second launch with the same binding signature takes the cached path
    (no re-checking) and reads and writes the new tensors; a different
    signature (shape, aliasing) takes the full path again."""
    from tila_b200 import plugin
    n = 3000
    xs = [torch.randn(n, device="cuda") for _ in range(3)]
    ys = [torch.randn(n, device="cuda") for _ in range(3)]
    outs = [torch.empty(n, device="cuda") for _ in range(3)]
    grid = (ti.cdiv(n, 1024),)
    W.add_kernel[grid](xs[0], ys[0], outs[0], BLOCK=1024)
    hits = plugin.fast_hits
    for i in (1, 2):
        W.add_kernel[grid](xs[i], ys[i], outs[i], BLOCK=1024)
    torch.cuda.synchronize()
    assert plugin.fast_hits == hits + 2
    for i in range(3):
        assert torch.equal(outs[i], xs[i] + ys[i])
    assert W.add_kernel.last_backend_resources is not None
    # a new shape and an aliased output are checked again
    m = 2000
    o2 = torch.empty(m, device="cuda")
    W.add_kernel[(ti.cdiv(m, 1024),)](xs[0][:m], ys[0][:m], o2, BLOCK=1024)
    assert plugin.fast_hits == hits + 2
    torch.cuda.synchronize()
    assert torch.equal(o2, xs[0][:m] + ys[0][:m])
    x_alias = xs[2].clone()
    try:
        W.add_kernel[grid](x_alias, ys[2], x_alias, BLOCK=1024)
    except ti.errors.TilaError:
        pass                       # the checker may reject the aliasing: also not cached
    else:
        torch.cuda.synchronize()
        assert torch.equal(x_alias, xs[2] + ys[2])
    assert plugin.fast_hits == hits + 2
    _no_device_errors()


@pytest.mark.parametrize("shape", [(3, 256, 384, 320), (2, 200, 136, 72)])
def test_batched_matmul_contraction_ring(tmp_path, shape):
    """3-D grid matmul (the per-program TMA ring with split copy / MMA
    threads): within the K * eps_f32 bound of the f64 product per batch."""
    import semantics_support as S
    k = S.batched_matmul_program(tmp_path)
    bsz, m, n, kd = shape
    rng = np.random.default_rng(11)
    a = (rng.standard_normal((bsz, m, kd)) / 8).astype(np.float16)
    b = (rng.standard_normal((bsz, kd, n)) / 8).astype(np.float16)
    c = torch.zeros((bsz, m, n), dtype=torch.float32, device="cuda")
    k[(ti.cdiv(m, 128), ti.cdiv(n, 128), bsz)](_cuda(a), _cuda(b), c, BM=128, BN=128, BK=64)
    _no_device_errors()
    got = c.cpu().numpy()
    for h in range(bsz):
        assert np.all(np.abs(got[h] - restate.matmul_f64(a[h], b[h])) <= restate.matmul_bound(a[h], b[h]))


@pytest.mark.parametrize("k", [320, 4096])
def test_matmul_persistent_split_matches_f64(monkeypatch, k):
    """The opt-in persistent contraction (TILA_B200_STREAMK=1) at 4096 x 4096
    outputs: 256 tiles of 2 x 2 programs on one CTA per SM, K loops split
    evenly, tiles parked by one CTA and finished by the previous one (with
    K = 320 nearly every CTA does both).  Every element within the K*eps_f32
    bound of the f64 product."""
    monkeypatch.setenv("TILA_B200_STREAMK", "1")     # part of the kernel cache key
    kernel = W.matmul_kernel
    a, b = W.matmul_inputs(4096, 4096, k, seed=29)
    c = torch.zeros((4096, 4096), dtype=torch.float32, device="cuda")
    kernel[(32, 32)](_cuda(a), _cuda(b), c, BM=128, BN=128, BK=64)
    _no_device_errors()
    from tila_b200.backend import last_launch
    assert last_launch(kernel).entry.spec.persistent and last_launch(kernel).grid[0] < 256
    rows = np.random.default_rng(k).choice(4096, 256, replace=False)
    got = c.cpu().numpy()[rows]
    want = restate.matmul_f64(a[rows], b)
    assert np.all(np.abs(got - want) <= restate.matmul_bound(a[rows], b))
