"""Code generation on CPU: every workload lowers to CUDA C++ that NVRTC
compiles for sm_100a, and the lowering picks the intended hardware paths
(128-bit vector accesses, TMA + tcgen05 pipelines) from the binding facts."""

import pytest
import torch

import tila_b200
from tila_b200 import native, workloads as W
from tila_b200.backend import binding_facts
from tila_b200.codegen.emitter import KernelEmitter

f16 = torch.float16


def gen(jf, tensors, warps=4, **consts):
    spec = KernelEmitter(jf.tk, consts, binding_facts(jf.tk, tensors), num_warps=warps).generate()
    native.compile_spec(spec)
    return spec


@pytest.mark.parametrize("warps", [4, 8])
def test_add_vectorised(warps):
    spec = gen(W.add_kernel, dict(x=torch.zeros(4096), y=torch.zeros(4096), out=torch.zeros(4096)),
               warps, BLOCK=1024)
    assert "uint4" in spec.source and "tcgen05" not in spec.source
    # element-wise programs keep 32 * num_warps threads (more loads in flight
    # per SM); only small programs that reduce across threads shrink to 2 warps
    assert spec.threads == 32 * warps


def test_softmax_reductions():
    spec = gen(W.softmax_kernel, dict(x=torch.zeros(8, 1000), o=torch.zeros(8, 1000)), BN=1024)
    src = spec.source
    assert "tila::max_nan" in src and "expf" in src and "shfl_xor" in src
    # the two cross-warp stages alternate between halves of their scratch:
    # one barrier each (after the partials are written)
    assert src.count("__syncthreads();") == 2 and src.count("tila_rsel ^= tila_red_half;") == 2
    # small programs that reduce across threads run with 2 warps
    assert spec.threads == 64


def test_matmul_uses_tma_ring_and_tcgen05():
    t = dict(a=torch.zeros(256, 256, dtype=f16), b=torch.zeros(256, 256, dtype=f16), c=torch.zeros(256, 256))
    spec = gen(W.matmul_kernel, t, BM=128, BN=128, BK=64)
    # a 2 x 2 block of programs per CTA sharing A and B tiles, N = 256 MMAs
    assert "2x2 programs per CTA" in spec.source and spec.fuse == {0: 2, 1: 2}
    assert not spec.persistent
    assert "tma_load_2d" in spec.source and "idesc_f16_f32(128, 256" in spec.source
    assert len(spec.tensor_maps) == 3          # A, B loads and the C store
    assert spec.tmem_cols == 512 and spec.smem_bytes <= 227 * 1024


def test_matmul_persistent_form_is_opt_in(monkeypatch):
    """TILA_B200_STREAMK=1 gives the persistent contraction (K loops split
    evenly over one CTA per SM when there are more tiles than SMs), with its
    workspace and flag arguments; it compiles."""
    monkeypatch.setenv("TILA_B200_STREAMK", "1")
    t = dict(a=torch.zeros(256, 256, dtype=f16), b=torch.zeros(256, 256, dtype=f16), c=torch.zeros(256, 256))
    spec = gen(W.matmul_kernel, t, BM=128, BN=128, BK=64)
    assert "2x2-program tiles" in spec.source and spec.fuse == {0: 2, 1: 2}
    assert spec.persistent and {"skws", "skflags"} <= {k for k, _, _ in spec.params}
    native.compile_spec(spec)


def test_streamk_split_covers_every_unit_once():
    """The persistent contraction's split (CTA b takes units [T b / P,
    T (b + 1) / P)) with P = #SMs and more tiles than SMs: every (tile, K
    step) unit is computed exactly once; a CTA's pieces are an optional
    high-K part first, whole tiles, an optional low-K part last; and every
    parked high-K part is finished by the previous CTA."""
    for tiles, kn, P in [(256, 64, 148), (149, 64, 148), (1000, 7, 148), (300, 1, 148)]:
        total = tiles * kn
        seen = {}
        for b in range(P):
            u0, u1 = total * b // P, total * (b + 1) // P
            assert u1 - u0 >= kn
            pieces, p = [], u0
            while p < u1:
                t, ka = divmod(p, kn)
                end = min((t + 1) * kn, u1)
                pieces.append((t, ka, end - t * kn))
                for u in range(p, end):
                    seen[u] = seen.get(u, 0) + 1
                p = end
            kinds = ["park" if ka > 0 else "fin" if kb < kn else "full" for _, ka, kb in pieces]
            assert "park" not in kinds[1:] and "fin" not in kinds[:-1]
            if kinds[-1] == "fin":
                nxt = total * (b + 1) // P
                assert nxt % kn and nxt // kn == pieces[-1][0]     # CTA b + 1 parks this tile
        assert len(seen) == total and set(seen.values()) == {1}


def test_matmul_strided_falls_back_to_register_staging():
    a = torch.zeros(256, 256, dtype=f16).t()
    t = dict(a=a, b=torch.zeros(256, 256, dtype=f16), c=torch.zeros(256, 256))
    spec = gen(W.matmul_kernel, t, BM=128, BN=128, BK=64)
    assert "kmajor_offset" in spec.source          # operand A staged from registers


def test_small_tiles_compile():
    t = dict(a=torch.zeros(19, 35, dtype=f16), b=torch.zeros(35, 23, dtype=f16), c=torch.zeros(19, 23))
    gen(W.matmul_kernel, t, BM=16, BN=16, BK=32)


def test_attention_kernels_compile():
    q = torch.zeros(2, 256, 64, dtype=f16)
    s = gen(W.attention_scores, dict(q=q, k=q.clone(), s=torch.zeros(2, 256, 256)), BM=128, BN=128, BD=64)
    assert "tma_load_3d" in s.source
    gen(W.attention_pv, dict(p=torch.zeros(2, 256, 256), v=q.clone(), o=torch.zeros(2, 256, 64)),
        BM=128, BN=128, BD=64)
    q = torch.zeros(2, 256, 128, dtype=f16)
    gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 256, 128)),
        CAUSAL=0, BM=128, BN=128, BD=128)


@pytest.mark.parametrize("causal", [0, 1])
def test_reference_fused_attention_takes_two_program_plan(causal):
    """examples/fused_attention.py puts each of its loops inside ``if CAUSAL
    == 1: ... else:``; the static if is resolved per specialisation before
    the loop matchers run, so at 128x128 tiles the loop of the taken branch
    runs two 128-row programs per CTA in the warp-specialised form: two
    softmax warpgroups plus a producer warpgroup that issues every copy and
    MMA.  With CAUSAL=1 the below-diagonal loop and the diagonal loop form
    one chain over the K/V tiles, and the two programs of a CTA run
    different numbers of iterations (the producer counts them per program)."""
    q = torch.zeros(2, 512, 128, dtype=f16)
    spec = gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 512, 128)),
               CAUSAL=causal, BM=128, BN=128, BD=128)
    assert spec.fuse == {0: 2} and spec.tmem_cols == 512
    from tila_b200.codegen.wspec import ws_budget
    threads, launch, producer, consumer = ws_budget(128)
    assert spec.threads == threads == 384 and spec.launch_regs == launch == 168
    assert f"tila::reg_alloc<{consumer}>()" in spec.source
    assert f"tila::reg_dealloc<{producer}>()" in spec.source
    assert "tila_nw[1]" in spec.source and "kErrSchedule" in spec.source


def test_heavy_first_cta_order_is_a_bijection():
    """The causal kernel renumbers its CTAs heaviest-first within groups of
    heads (wspec.cta_order_prelude); the prelude, evaluated here for grids
    whose head count is and is not a multiple of the group, maps the
    dispatch order onto every CTA exactly once."""
    import re
    from tila_b200.codegen.wspec import CTA_GROUP, cta_order_prelude
    q = torch.zeros(2, 512, 128, dtype=f16)
    spec = gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 512, 128)),
               CAUSAL=1, BM=128, BN=128, BD=128)
    assert cta_order_prelude(True) in spec.source
    body = spec.source.split(cta_order_prelude(True), 1)[1]
    assert "blockIdx" not in body
    src = cta_order_prelude(True)
    stmts = re.findall(r"const (?:unsigned|bool) ([^;]*);", src)

    def run(lin, X, Y, Z):
        env = dict(gridDim=None)
        vals = {"gridDim.x": X, "gridDim.y": Y, "gridDim.z": Z, "blockIdx.x": lin % X,
                "blockIdx.y": (lin // X) % Y, "blockIdx.z": lin // (X * Y)}
        for st in stmts:
            for decl in re.split(r",\s*(?=tila_)", st):
                name, expr = decl.split("=", 1)
                e = expr
                for k, v in sorted(vals.items(), key=lambda kv: -len(kv[0])):
                    e = re.sub(r"\b" + re.escape(k) + r"\b", str(v), e)
                e = e.replace("u", "").replace("/", "//").replace("?", " if ").replace(":", " else ")
                e = re.sub(r"(.*) if (.*) else (.*)", r"(\2) if (\1) else (\3)", e)
                vals[name.strip()] = int(eval(e))
        return vals["tila_bx"], vals["tila_by"], vals["tila_bz"]
    for X, Y, Z in [(16, 128, 1), (4, CTA_GROUP + 3, 1), (3, 5, 2), (1, 1, 1)]:
        seen = {run(lin, X, Y, Z) for lin in range(X * Y * Z)}
        assert len(seen) == X * Y * Z and all(0 <= a < X and 0 <= b < Y and 0 <= c < Z for a, b, c in seen)
    # the first CTAs dispatched run the heaviest (last) axis-0 position
    assert run(0, 16, 128, 1)[0] == 15


def test_warp_specialised_budgets_fit_the_launch_pool():
    """The warpgroups' setmaxnreg shares add up to at most the registers the
    CTA is launched with (threads x launch registers).  Programs requested
    with 8 warps get the same 4-warp warp-specialised kernel (384 threads)."""
    from tila_b200.codegen.wspec import ws_budget
    threads, launch, producer, consumer = ws_budget(128)
    assert threads == 2 * 128 + 128 and launch == (65536 // threads) // 8 * 8
    assert 128 * producer + 2 * 128 * consumer <= threads * launch
    q = torch.zeros(2, 512, 128, dtype=f16)
    for causal in (0, 1):
        spec = gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 512, 128)),
                   8, CAUSAL=causal, BM=128, BN=128, BD=128)
        assert spec.threads == 384 and spec.launch_regs == 168 and spec.fuse == {0: 2}


def test_warp_specialised_kernel_register_budget(tmp_path):
    """The warpgroups of the warp-specialised kernel trade registers within
    the pool the CTA is launched with (384 threads x 168): ptxas must give the
    kernel exactly 168 registers per thread at launch."""
    import re
    import shutil
    import subprocess
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    q = torch.zeros(2, 512, 128, dtype=f16)
    spec = gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 512, 128)),
               CAUSAL=0, BM=128, BN=128, BD=128)
    cu = tmp_path / "ws.cu"
    cu.write_text(spec.source)
    from tila_b200 import build
    out = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-Xptxas", "-v",
                          f"-I{build.PKG / 'csrc' / 'tile'}", "-c", str(cu), "-o", str(tmp_path / "ws.o")],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr[-2000:]
    regs = re.findall(r"Used (\d+) registers", out.stderr)
    assert regs and int(regs[-1]) == spec.launch_regs == 168
    assert not re.search(r"[1-9]\d* bytes spill stores", out.stderr), out.stderr[-2000:]
    # the causal chain (per-program trip counts, CTA renumbering) too
    spec1 = gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 512, 128)),
                CAUSAL=1, BM=128, BN=128, BD=128)
    cu.write_text(spec1.source)
    out = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-Xptxas", "-v",
                          f"-I{build.PKG / 'csrc' / 'tile'}", "-c", str(cu), "-o", str(tmp_path / "ws.o")],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr[-2000:]
    assert int(re.findall(r"Used (\d+) registers", out.stderr)[-1]) == spec1.launch_regs == 168
    assert not re.search(r"[1-9]\d* bytes spill stores", out.stderr), out.stderr[-2000:]


def test_static_if_resolution_leaves_kernel_untouched():
    from tila_b200.codegen.emitter import resolve_static_ifs
    tk = W.fused_attention_kernel.tk
    before = [type(s).__name__ for s in tk.body]
    assert "TStaticIf" in before
    for causal, loops in ((0, 1), (1, 2)):
        flat = resolve_static_ifs(tk, dict(CAUSAL=causal, BM=128, BN=128, BD=128))
        kinds = [type(s).__name__ for s in flat.body]
        assert "TStaticIf" not in kinds and kinds.count("TFor") == loops
    assert [type(s).__name__ for s in tk.body] == before


def test_tmem_budget_and_occupancy():
    q = torch.zeros(2, 256, 128, dtype=f16)
    spec = gen(W.fused_attention_kernel, dict(q=q, k=q.clone(), v=q.clone(), o=torch.zeros(2, 256, 128)),
               CAUSAL=0, BM=128, BN=128, BD=128)
    cols = spec.tmem_cols
    assert cols in (32, 64, 128, 256, 512)
    resident = 233472 // (spec.smem_bytes + 1024)
    assert resident * cols <= 512, "co-resident CTAs could exhaust tensor memory"


# -- semantic programs of every dtype lower and compile -----------------------------

def _dev_like(shape, dt):
    import ml_dtypes  # noqa: F401
    tmap = dict(f16=torch.float16, bf16=torch.bfloat16, f32=torch.float32, f64=torch.float64,
                i8=torch.int8, i16=torch.int16, i32=torch.int32, i64=torch.int64, u8=torch.uint8,
                u16=torch.uint16, u32=torch.uint32, u64=torch.uint64)
    return torch.zeros(shape, dtype=tmap[dt])


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32", "f64"])
def test_float_programs_compile(dt, tmp_path):
    import semantics_support as S
    for op in ("exp", "exp2", "neg"):
        k = S.unary_program(tmp_path, dt, op)
        gen(k, dict(x=_dev_like(40, dt), out=_dev_like(40, dt)))
    for dst in ("f16", "bf16", "f32", "f64"):
        k = S.unary_program(tmp_path, dt, "cast", dst, cast_to=dst)
        gen(k, dict(x=_dev_like(40, dt), out=_dev_like(40, dst)))


@pytest.mark.parametrize("dt", ["i8", "i16", "i32", "i64", "u8", "u16", "u32", "u64"])
def test_integer_programs_compile(dt, tmp_path):
    import semantics_support as S
    for op in ("+", "-", "*", "//", "%", "&", "|", "^"):
        k = S.binary_program(tmp_path, dt, op)
        gen(k, dict(x=_dev_like(100, dt), y=_dev_like(100, dt), out=_dev_like(100, dt)))


@pytest.mark.parametrize("dt", ["f32", "i32"])
@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("axis", [0, 1])
def test_reduction_programs_compile(dt, op, axis, tmp_path):
    import semantics_support as S
    k = S.reduce_program(tmp_path, dt, op, axis)
    out = _dev_like((24,), dt) if axis == 1 else _dev_like((3, 50), dt)
    gen(k, dict(x=_dev_like((24, 50), dt), out=out), warps=8)


@pytest.mark.parametrize("dt", ["i8", "i32", "u32"])
def test_scalar_division_programs_compile(dt, tmp_path):
    import semantics_support as S
    for op in ("//", "%"):
        k = S.scalar_div_program(tmp_path, dt, op, 1, 100)
        gen(k, dict(x=_dev_like(64, dt), out=_dev_like(64, dt)))


def test_uniform_divisor_takes_reciprocal_path(tmp_path):
    """Division by a per-program value (softmax's row sum, a scalar
    parameter) goes through the shared-reciprocal path (tila::udiv_*);
    element-wise division by a tile keeps IEEE division."""
    import semantics_support as S
    spec = gen(W.softmax_kernel, dict(x=torch.zeros(8, 1000), o=torch.zeros(8, 1000)), BN=1024)
    assert "tila::udiv_q2(" in spec.source and "tila::udiv_track(" in spec.source
    for kind in ("scalar", "reduced"):
        k = S.uniform_div_program(tmp_path, kind)
        t = dict(x=torch.zeros(2048), out=torch.zeros(2048))
        if kind == "reduced":
            t["y"] = torch.zeros(2, 256)
        assert "tila::udiv_q" in gen(k, t).source
    k = S.binary_program(tmp_path, "f32", "/")
    src = gen(k, dict(x=torch.zeros(100), y=torch.zeros(100), out=torch.zeros(100))).source
    assert "udiv" not in src and " / " in src


def test_f32_tile_epilogues_store_through_tma():
    """128-row f32 results held one row per thread (scores, matmul, flash
    attention) are written with TMA box stores from swizzled shared memory."""
    t = dict(q=torch.zeros(2, 256, 64, dtype=f16), k=torch.zeros(2, 256, 64, dtype=f16),
             s=torch.zeros(2, 256, 256))
    src = gen(W.attention_scores, t, BM=128, BN=128, BD=64).source
    assert "tila::tma_store_3d(" in src and "bulk_wait_read" in src
    t = dict(a=torch.zeros(256, 256, dtype=f16), b=torch.zeros(256, 256, dtype=f16), c=torch.zeros(256, 256))
    assert "tila::tma_store_2d(" in gen(W.matmul_kernel, t, BM=128, BN=128, BK=64).source
    # a column offset that is not a multiple of 4 elements keeps plain stores
    t = dict(x=torch.zeros(8, 1000), o=torch.zeros(8, 1000))
    assert "tma_store" not in gen(W.softmax_kernel, t, BN=1024).source


@pytest.mark.parametrize("dt", ["i32", "u32", "f32"])
@pytest.mark.parametrize("kind", ["buffer", "ptr"])
def test_atomic_programs_compile(dt, kind, tmp_path):
    import semantics_support as S
    k = S.atomic_program(tmp_path, dt, kind)
    t = dict(x=_dev_like(64, dt), values=_dev_like(64, dt), old=_dev_like(64, dt))
    for collide in (True, False):
        src = gen(k, t, COUNT=61, COLLIDE=collide).source
        assert "atomicAdd(" in src


def test_ptr_programs_compile(tmp_path):
    import semantics_support as S
    k = S.ptr_copy_program(tmp_path, "f32")
    gen(k, dict(x=torch.zeros(100), out=torch.zeros(100)))


def test_batched_matmul_uses_split_copy_and_mma_threads(tmp_path):
    """A 3-D grid (batch axis) is not coarsened: the per-program contraction
    ring runs with a copy thread (32) and an MMA thread (0)."""
    import semantics_support as S
    k = S.batched_matmul_program(tmp_path)
    t = dict(a=torch.zeros(2, 256, 320, dtype=f16), b=torch.zeros(2, 320, 384, dtype=f16),
             c=torch.zeros(2, 256, 384))
    spec = gen(k, t, BM=128, BN=128, BK=64)
    assert "pipelined contraction loop" in spec.source and "if (tid == 32)" in spec.source
    assert not spec.fuse
    native.compile_spec(spec)


def test_rank3_tiles_compile(tmp_path):
    """Tiles of rank 3 (from reshape) get a blocked layout over the flattened
    leading dimensions; reductions along every axis compile."""
    import semantics_support as S
    for op in ("sum", "max"):
        for axis in (0, 1, 2):
            k = S.rank3_program(tmp_path, op, axis)
            spec = gen(k, dict(x=torch.zeros(1000), w=torch.zeros(384), out=torch.zeros(384)))
            native.compile_spec(spec)


def test_expand_of_rank2_tiles_compiles(tmp_path):
    """x[None, :] and x[:, None] on 2-D tiles insert a unit axis at 0 and 1;
    chained expands of 1-D aranges give 3-D index tiles."""
    import semantics_support as S
    k = S.expand3_program(tmp_path)
    spec = gen(k, dict(x=torch.zeros(4, 8), o0=torch.zeros(2, 4, 8), o1=torch.zeros(4, 2, 8)))
    native.compile_spec(spec)


def test_named_pointer_tiles_compile(tmp_path):
    """Pointer tiles bound to names (1-D and 2-D) lower to masked loads and
    stores through the Ptr parameters."""
    import semantics_support as S
    k = S.ptr_tile_program(tmp_path)
    spec = gen(k, dict(x=torch.zeros(300), out=torch.zeros(300), out2=torch.zeros(300)))
    native.compile_spec(spec)


def test_assume_checks_only_in_debug_builds(tmp_path):
    """ti.assume is free normally; with debug checks each false lane records
    its line and the program stops before the access it guards."""
    import semantics_support as S
    k = S.assume_gather_program(tmp_path)
    t = dict(idx_buf=torch.zeros(100, dtype=torch.int32), data=torch.zeros(100), out=torch.zeros(100))
    facts = binding_facts(k.tk, t)
    plain = KernelEmitter(k.tk, dict(BLOCK=64), facts, num_warps=4).generate()
    debug = KernelEmitter(k.tk, dict(BLOCK=64), facts, num_warps=4, debug=True).generate()
    assert "kErrAssumption" not in plain.source and not plain.assume_lines
    assert "kErrAssumption" in debug.source and "goto tila_program_end" in debug.source
    assert len(debug.assume_lines) == 2
    native.compile_spec(debug)
