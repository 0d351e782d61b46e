"""TIR -> CUDA C++ code generator for sm_100a (one CTA per Tila program).

Input: a checked ``TKernel`` (tir.py:357) specialised with its Const values,
plus launch facts (buffer dtypes, unit strides, alignment).  Output: the
source of one ``extern "C" __global__`` kernel that includes the tile library
(``csrc/tile/tila_tile.cuh``), and a :class:`KernelSpec` saying how to launch
it.  It replaces ``Lowering.kernel_source`` (lowering.py:136-182) and keeps
its ABI order: buffer pointers, Ptr parameters, scalars (lowering.py:204-213);
Consts become compile-time constants of the generated source.

Values of the program are represented as

* ``scalar``  uniform C++ expressions (pids, scalars, loop variables, full
  reductions, scalar loads) - every thread computes the same value;
* ``func``    index-functional tiles (arange, broadcasts of scalars, masks,
  and element-wise functions of those): no storage, an element is a C++
  expression of its index, re-evaluated where it is used;
* ``reg``     materialised tiles: a per-thread register array in a
  :mod:`layouts` layout;
* ``tmem``    f32 dot accumulators resident in tensor memory.

Element-wise operations read their operands in the consumer's layout.  When a
register operand's layout does not hold the needed element in the same
thread at a compile-time slot, it is redistributed through shared memory.
Reductions fold inside a thread, then across threads with xor shuffles and a
shared-memory stage (NaN-propagating max, ADR-008).  Loads and stores are
masked per element; groups of consecutive, aligned, fully active elements
move with 128-bit accesses.  ``dot`` runs on the 5th-generation tensor core:
operands are staged into shared memory in the UMMA K-major layout,
``tcgen05.mma`` accumulates into TMEM, and ``tcgen05.ld`` reads the result
into the TMEM-row layout.
"""

from __future__ import annotations

import os
import re

import dataclasses
import math
from dataclasses import dataclass, field

import numpy as np

from .._reference import tila
from . import dtypes as DT
from .layouts import (Blocked, Derived, Layout, TmemRows, dedupe_owner, owner_predicate,
                      source_slot_map)
from .fused import FusedContractionMixin
from .mma import AsyncLoopMixin, MmaMixin
from .wspec import WarpSpecMixin, ws_budget

T_ = tila.tir
TY = tila.types
D = tila.dtypes
dims_mod = tila.dims


class CodegenError(Exception):
    """The TIR uses something this backend does not lower (TILA-TARGET-009)."""

    def __init__(self, message, line=0):
        super().__init__(message)
        self.line = line


# ---------------------------------------------------------------------------
# values
# ---------------------------------------------------------------------------

@dataclass
class Val:
    kind: str                 # scalar | func | reg | tmem | ptr
    dt: object
    shape: tuple = ()
    expr: str = None          # scalar
    fn: object = None         # func: callable(idx: tuple[str]) -> str
    name: str = None          # reg: C++ array name
    layout: Layout = None     # reg
    tmem_col: int = 0         # tmem: column offset of the accumulator
    ptr: tuple = None         # ptr: (param name, offset Val)
    zero: bool = False        # func known to be all zeros
    smem: object = None       # smem: the shared-memory operand (TMA-loaded tile)
    const: object = None      # compile-time known python value (scalars)


@dataclass
class BufferInfo:
    """Launch facts about one Buffer / Ptr binding (part of the cache key)."""
    name: str
    dtype: object
    rank: int
    unit_last: bool            # last-dim element stride == 1
    stride_div: tuple          # per dim: largest power of two (<= 16) dividing the stride
    base_align: int            # largest power of two (<= 256) dividing the base address
    writable: bool
    is_ptr: bool = False
    tma_ok: bool = False       # f16/f32, unit last stride, 16-byte aligned base and strides

    def key(self):
        return (self.name, self.dtype.name, self.rank, self.unit_last, self.stride_div,
                self.base_align, self.writable, self.is_ptr, self.tma_ok)


@dataclass
class KernelSpec:
    """Everything the host needs to launch a generated kernel."""
    name: str
    source: str
    threads: int
    smem_bytes: int
    params: list               # [(kind, name, ctype)] in launch order
    tmem_cols: int = 0
    notes: list = field(default_factory=list)
    tensor_maps: list = field(default_factory=list)
    persistent: bool = False
    grid_override: object = None
    fuse: dict = field(default_factory=dict)   # {grid axis: programs per CTA along it}
    # compile with multiply-add contraction (tensor-core kernels, whose results
    # are compared within a tolerance; kernels without a dot keep every f32
    # multiply and add separately rounded, like NumPy)
    fp_contract: bool = False
    # Tila lines of the ti.assume checks compiled in (TILA_DEBUG=1 builds)
    assume_lines: list = field(default_factory=list)
    # registers per thread the kernel must have been given at launch (kernels
    # that move registers between warpgroups with setmaxnreg); 0 = any
    launch_regs: int = 0


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def _eval_dim(d, consts):
    if isinstance(d, int):
        return d
    v = dims_mod.eval_num(d, consts)
    return int(v)


def _stmt_names_assigned(stmts, out=None):
    out = set() if out is None else out
    for s in stmts:
        if isinstance(s, T_.TAssign):
            out.add(s.name)
        elif isinstance(s, (T_.TIf, T_.TStaticIf)):
            _stmt_names_assigned(s.then_body, out)
            _stmt_names_assigned(s.else_body, out)
        elif isinstance(s, T_.TFor):
            out.add(s.var)
            _stmt_names_assigned(s.body, out)
    return out


def resolve_static_ifs(tk, consts):
    """The kernel with every ``static_if`` replaced by the branch its Const
    values select, recursively (the statements of the taken branch take the
    place of the ``static_if`` in the enclosing body).

    A ``static_if`` is resolved per Const specialisation (tir.py:324-335); the
    interpreter runs the selected branch in the enclosing scope
    (interp.py:145-154), so splicing it in changes no binding.  Resolving it
    before code generation lets the loop matchers see a loop of the taken
    branch as a statement of the enclosing body: the non-causal loop of
    examples/fused_attention.py:104-126 sits inside ``if CAUSAL == 1: ...
    else:`` and is a top-level loop of the CAUSAL=0 specialisation.  A
    condition that does not evaluate from the Consts (and from names assigned
    once, from Consts only) keeps its ``static_if``; the emitter then decides
    it while emitting.  The caller's kernel object is not modified."""
    ev = tila.runtime._eval_const_operand
    counts = {}

    def count(stmts):
        for s in stmts:
            if isinstance(s, T_.TAssign):
                counts[s.name] = counts.get(s.name, 0) + 1
            elif isinstance(s, (T_.TIf, T_.TStaticIf)):
                count(s.then_body)
                count(s.else_body)
            elif isinstance(s, T_.TFor):
                counts[s.var] = counts.get(s.var, 0) + 2
                count(s.body)
    count(tk.body)
    known = dict(consts)
    changed = [False]

    def walk(stmts, top=False):
        out = []
        for s in stmts:
            if top and out and isinstance(out[-1], T_.TReturn):
                # a return spliced in at the top level ends the program: what
                # follows it never runs (and may not even have matching shapes,
                # being typed for the branch that does not return)
                changed[0] = True
                break
            if isinstance(s, T_.TStaticIf):
                try:
                    taken = bool(ev(s.cond, known))
                except Exception:
                    taken = None
                if taken is None:
                    out.append(dataclasses.replace(s, then_body=walk(s.then_body),
                                                   else_body=walk(s.else_body)))
                else:
                    changed[0] = True
                    out.extend(walk(s.then_body if taken else s.else_body, top))
                continue
            if isinstance(s, T_.TAssign) and counts.get(s.name) == 1 and s.name not in known:
                try:
                    known[s.name] = ev(s.value, known)
                except Exception:
                    pass
            if isinstance(s, T_.TIf):
                s = dataclasses.replace(s, then_body=walk(s.then_body), else_body=walk(s.else_body))
            elif isinstance(s, T_.TFor):
                s = dataclasses.replace(s, body=walk(s.body))
            out.append(s)
        return out
    body = walk(tk.body, top=True)
    return dataclasses.replace(tk, body=body) if changed[0] else tk


class _Smem:
    """Linear plan of the kernel's dynamic shared memory."""

    def __init__(self):
        self.top = 0
        self.scratch = 0        # size of the shared redistribution scratch
        self.red = 0            # one half of the cross-warp reduction scratch

    def alloc(self, nbytes, align=16):
        self.top = (self.top + align - 1) // align * align
        off = self.top
        self.top += nbytes
        return off

    def need_scratch(self, nbytes):
        self.scratch = max(self.scratch, nbytes)

    def need_red(self, nbytes):
        self.red = max(self.red, (nbytes + 127) // 128 * 128)


# ---------------------------------------------------------------------------
# the emitter
# ---------------------------------------------------------------------------

class KernelEmitter(FusedContractionMixin, WarpSpecMixin, AsyncLoopMixin, MmaMixin):
    MAX_SCRATCH = 96 * 1024

    def __init__(self, tk, consts: dict, buffers: dict, num_warps: int = 4,
                 entry_name=None, debug=False, versioning=True, source_map=False, ws=None):
        tk = resolve_static_ifs(tk, consts)
        self.tk = tk
        self._num_warps = num_warps
        # warp-specialised attention loop (see wspec.py): None, or the plan the
        # first generation found ({"q": name of the loop's one-shot operand})
        self._ws = dict(ws) if ws else None
        self._ws_found = None
        self.persistent = False     # the stream-K contraction (fused.py)
        self.source_map = source_map     # annotate the output with Tila source lines
        self.versioning = versioning     # loop bodies specialised for interior tiles
        self.consts = dict(consts)
        self.buffers = buffers
        self.T = 32 * num_warps
        self.debug = debug
        self.entry = entry_name or f"tila_{tk.name}"
        self.lines = []
        self.indent = 1
        self.env = {}
        self.counter = 0
        self.smem = _Smem()
        self.smem.top = 64
        self.tmem_cols = 0
        self.uses_tmem = False
        self.uses_mma = False
        self.conv_cache = {}
        self.slot_cache = {}
        self.scalar_params = {s.name: s for s in tk.scalars}
        self.const_names = {c.name for c in tk.consts}
        self.buffer_params = {b.name: b for b in tk.buffers}
        self.ptr_params = {p.name: p for p in tk.ptr_params}
        self.dot_rows = set()
        self.actx = None
        self._guard_mode = None
        self._pid_expr = {}          # program-id expressions of the program being emitted
        self.fuse = None             # {axis: programs per CTA} when CTAs run program blocks
        self._wg_candidate = False   # an asynchronous loop allows two programs per CTA
        self._free_smem = []         # (offset, bytes) of buffers no longer in use
        self._store_ring = None      # rotating TMA-store staging slots (see _try_tma_store)
        self._contracted = False     # an FMA was contracted (see _try_contract)
        self._uneven_loops = 0       # hand-off loops with program-dependent trip counts
        self._loop_acc_cols = set()  # (column, N) of asynchronous-loop accumulators
        self._prefetch = []          # L2 prefetches of top-level loads (see _prefetch_load)
        self._assume_lines = []      # debug checks of ti.assume (see s_TAssume)
        self._assume_stop = False    # a failed check leaves the program (label at its end)
        self._scan_dots(tk.body)

    # -- small utilities ---------------------------------------------------

    def fresh(self, base="t"):
        self.counter += 1
        return f"{base}_{self.counter}"

    def emit(self, line=""):
        self.lines.append("  " * self.indent + line if line else "")

    def fail(self, msg, line=0):
        raise CodegenError(msg, line)

    def dims(self, vt):
        return tuple(_eval_dim(d, self.consts) for d in vt.dims)

    def vt_info(self, vt):
        """(dtype, shape, is_pointer) of a TIR value type."""
        if isinstance(vt, TY.ScalarT):
            return vt.dtype, (), False
        if isinstance(vt, TY.MaskT):
            return D.bool_, self.dims(vt), False
        if isinstance(vt, TY.BlockT):
            if isinstance(vt.elem, TY.ScalarT):
                return vt.elem.dtype, self.dims(vt), False
            if isinstance(vt.elem, TY.PtrT):
                return vt.elem.element, self.dims(vt), True
        if isinstance(vt, TY.PtrT):
            return vt.element, (), True
        if isinstance(vt, TY.ConstT):
            return vt.dtype, (), False
        self.fail(f"unsupported value type {vt!r}")

    SMALL_PROGRAM_TILE = 2048

    def _small_program(self):
        """Programs without tensor-core work that reduce across threads and
        whose tiles have at most 2048 elements run with 64 threads: more
        programs resident per SM and shorter CTA-wide reductions (measured
        best for row reductions: row softmax 8192x1000).  Element-wise
        programs keep 32 * num_warps threads: the vector add over 2^20 f32
        takes 2.48 us per launch with 128 threads per 1024-element program
        against 2.57 us with 64 (more loads in flight per SM)."""
        if self.dot_rows or self.T != 128:
            return False
        ok = [True]
        reduces = [False]

        def visit(node):
            if isinstance(node, (T_.TDot, T_.TAtomicAdd)):
                ok[0] = False
            if isinstance(node, T_.TReduce):
                reduces[0] = True
            vt = getattr(node, "vt", None)
            if isinstance(vt, (TY.BlockT, TY.MaskT)):
                try:
                    n = int(np.prod(self.dims(vt)))
                except Exception:
                    ok[0] = False
                    return
                if n > self.SMALL_PROGRAM_TILE:
                    ok[0] = False
            if dataclasses.is_dataclass(node):
                for f in dataclasses.fields(node):
                    if f.name in ("vt", "definition", "effect"):
                        continue
                    v = getattr(node, f.name)
                    for x in (v if isinstance(v, list) else [v]):
                        if dataclasses.is_dataclass(x):
                            visit(x)
        for st in self.tk.body:
            visit(st)
        return ok[0] and reduces[0]

    def _scan_dots(self, stmts):
        """Row counts of dot results: 2-D tiles with that many rows default to
        the TMEM-row layout so that soft-max style code around a dot needs no
        redistribution."""
        def visit(node):
            if isinstance(node, T_.TDot):
                dt, shape, _ = self.vt_info(node.vt)
                self.dot_rows.add(tuple(shape))
            if dataclasses.is_dataclass(node):
                for f in dataclasses.fields(node):
                    if f.name in ("vt", "definition", "effect"):
                        continue
                    v = getattr(node, f.name)
                    if isinstance(v, list):
                        for x in v:
                            visit(x)
                    elif dataclasses.is_dataclass(v):
                        visit(v)
        for s in stmts:
            visit(s)

    # -- layouts -----------------------------------------------------------

    def default_layout(self, shape, dt=None) -> Layout:
        if len(shape) == 2 and shape[0] <= 128 and any(
                shape[0] == m and shape[1] in (n, 1) for m, n in self.dot_rows):
            return TmemRows(tuple(shape), self.T)
        if not shape or any(int(n) & (int(n) - 1) for n in shape):
            self.fail(f"tile shape {tuple(shape)} is not a product of powers of two")
        last = shape[-1]
        V = 4
        if dt is not None and DT.size(dt) == 2:
            V = 8
        if dt is not None and DT.size(dt) == 8:
            V = 2
        return Blocked(tuple(shape), self.T, min(V, last))

    def slot_map(self, src: Layout, dst: Layout, dst_shape):
        key = (src.key(), dst.key(), tuple(dst_shape))
        if key not in self.slot_cache:
            self.slot_cache[key] = source_slot_map(src, dst, dst_shape)
        return self.slot_cache[key]

    # -- element access ------------------------------------------------------

    @staticmethod
    def bcast_idx(idx, shape):
        """Index of an operand of ``shape`` broadcast to a consumer index."""
        rank = len(shape)
        idx = tuple(idx)[len(idx) - rank:] if rank else ()
        return tuple("0" if n == 1 else i for i, n in zip(idx, shape))

    def elem(self, v: Val, layout: Layout, r, smap=None) -> str:
        """C++ expression of operand ``v`` at consumer slot ``r`` of ``layout``."""
        if v.kind == "scalar":
            return v.expr
        if v.kind == "func":
            return v.fn(self.bcast_idx(layout.coord(r), v.shape))
        if v.kind == "reg":
            if isinstance(r, int) and smap is not None:
                return f"{v.name}[{smap[r]}]"
            aff = getattr(v, "_affine", None)
            if aff is not None and aff != (0, 1):
                a, b = aff
                if isinstance(r, int):
                    return f"{v.name}[{a + b * r}]"
                return f"{v.name}[{a}]" if b == 0 else f"{v.name}[{a} + {b} * ({r})]"
            return f"{v.name}[{r}]"
        self.fail(f"value of kind {v.kind} used as an element-wise operand")

    def prepare_operands(self, operands, layout, shape):
        """Make every register operand readable in ``layout``; returns
        (operands, maps, straight) where ``straight`` asks for unrolled code."""
        out, maps, straight = [], [], False
        for v in operands:
            if v.kind == "tmem":
                v = self.tmem_to_reg(v)
            if v.kind == "ptr":
                self.fail("pointer tiles are not supported in element-wise code yet")
            if v.kind == "reg":
                m = self.slot_map(v.layout, layout, shape)
                if m is None:
                    v = self.convert(v, layout, shape)
                    m = self.slot_map(v.layout, layout, shape)
                    assert m is not None
                aff = _affine_map(m)
                if aff is None:
                    straight = True
                elif aff != (0, 1):
                    # read through an affine slot expression in loop form
                    v = dataclasses.replace(v, name=v.name, layout=v.layout)
                    v._affine = aff
                maps.append(m)
            else:
                maps.append(None)
            out.append(v)
        if not straight:
            maps = [None] * len(out)
        return out, maps, straight

    def pick_layout(self, operands, shape, dt):
        for v in operands:
            if v.kind == "reg" and tuple(v.shape) == tuple(shape):
                return v.layout
        for v in operands:
            if v.kind == "tmem" and tuple(v.shape) == tuple(shape):
                return TmemRows(tuple(shape), self.T)
        return self.default_layout(shape, dt)

    def materialize_elementwise(self, dt, shape, operands, make_expr, layout=None, base="v"):
        """New register tile: element r = make_expr([operand exprs at r])."""
        layout = layout or self.pick_layout(operands, shape, dt)
        ops, maps, straight = self.prepare_operands(operands, layout, shape)
        name = self.fresh(base)
        self.emit(f"{DT.ctype(dt)} {name}[{layout.nreg}];")
        if straight:
            rows = [[self.elem(v, layout, r, m) for v, m in zip(ops, maps)]
                    for r in range(layout.nreg)]
            if isinstance(make_expr, _UniformDivisor) and len({e[1] for e in rows}) == 1:
                self._uniform_division(name, [(str(r), e[0]) for r, e in enumerate(rows)], rows[0][1])
            else:
                for r, exprs in enumerate(rows):
                    self.emit(f"{name}[{r}] = {make_expr(exprs)};")
        else:
            exprs = [self.elem(v, layout, "r") for v in ops]
            if isinstance(make_expr, _UniformDivisor) and not re.search(r"\br\b", exprs[1]):
                self._uniform_division(name, None, exprs[1], exprs[0], layout.nreg)
            elif isinstance(make_expr, (_PackedBin, _PackedFma)) and dt.name == "f32" \
                    and layout.nreg % 2 == 0 and layout.nreg >= 4:
                # two elements per f32x2 instruction
                e0 = [self.elem(v, layout, "(r)") for v in ops]
                e1 = [self.elem(v, layout, "(r + 1)") for v in ops]
                args = ", ".join(f"tila::pk2({a}, {b})" for a, b in zip(e0, e1))
                self.emit("#pragma unroll")
                self.emit(f"for (int r = 0; r < {layout.nreg}; r += 2) {{")
                self.emit(f"  const tila::u64 q_ = tila::{make_expr.fn}({args});")
                self.emit(f"  {name}[r] = tila::lo2(q_); {name}[r + 1] = tila::hi2(q_);")
                self.emit("}")
            else:
                self.emit("#pragma unroll")
                self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
                self.emit(f"  {name}[r] = {make_expr(exprs)};")
                self.emit("}")
        return Val("reg", dt, tuple(shape), name=name, layout=layout)

    def _uniform_division(self, name, rows, divisor, dividend=None, nreg=None):
        """f32 quotients by a divisor shared by all of this thread's elements:
        one reciprocal (tila::udiv_prepare), a range record of the dividends
        (tila::udiv_track), then Markstein-corrected quotients, or IEEE
        division if any dividend leaves the exact range.  Dividends that are
        not plain register reads are computed once into a temporary, so that
        the quotients can take over their registers."""
        ud = self.fresh("ud")
        plain = re.compile(r"\(*\w+\[\(*r\)*\]\)*")
        if rows is not None:
            if not all(re.fullmatch(r"\(*\w+\[\d+\]\)*", a) for _, a in rows):
                tmp = self.fresh("dv")
                self.emit(f"float {tmp}[{len(rows)}];")
                for r, a in rows:
                    self.emit(f"{tmp}[{r}] = {a};")
                rows = [(r, f"{tmp}[{r}]") for r, _ in rows]
        elif not plain.fullmatch(dividend):
            tmp = self.fresh("dv")
            self.emit(f"float {tmp}[{nreg}];")
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {nreg}; ++r) {tmp}[r] = {dividend};")
            dividend = f"{tmp}[r]"
        self.emit(f"const tila::UDiv {ud} = tila::udiv_prepare({divisor});")
        self.emit(f"float {ud}_hi = 0.0f; tila::u32 {ud}_lo = 0xffffffffu;")
        if rows is not None:
            for r, a in rows:
                self.emit(f"tila::udiv_track(({a}), {ud}_hi, {ud}_lo);")
        else:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {nreg}; ++r) tila::udiv_track(({dividend}), {ud}_hi, {ud}_lo);")
        self.emit(f"if (tila::udiv_all_fast({ud}, {ud}_hi, {ud}_lo)) {{")
        if rows is not None:
            for r, a in rows:
                self.emit(f"  {name}[{r}] = tila::udiv_q(({a}), {ud});")
        elif nreg % 2 == 0:
            d0 = re.sub(r"\br\b", "(r)", dividend)
            d1 = re.sub(r"\br\b", "(r + 1)", dividend)
            self.emit("  #pragma unroll")
            self.emit(f"  for (int r = 0; r < {nreg}; r += 2) "
                      f"tila::udiv_q2(({d0}), ({d1}), {ud}, {name}[r], {name}[r + 1]);")
        else:
            self.emit("  #pragma unroll")
            self.emit(f"  for (int r = 0; r < {nreg}; ++r) {name}[r] = tila::udiv_q(({dividend}), {ud});")
        self.emit("} else {")
        if rows is not None:
            for r, a in rows:
                self.emit(f"  {name}[{r}] = (({a}) / ({divisor}));")
        else:
            self.emit(f"  for (int r = 0; r < {nreg}; ++r) {name}[r] = (({dividend}) / ({divisor}));")
        self.emit("}")

    def materialize(self, v: Val, layout=None) -> Val:
        if v.kind == "reg" and (layout is None or v.layout == layout):
            return v
        if v.kind == "tmem" and layout is None:
            return self.tmem_to_reg(v)
        if v.kind == "scalar":
            self.fail("cannot materialise a scalar as a tile")
        if v.kind == "reg":
            return self.convert(v, layout, v.shape)
        layout = layout or self.default_layout(v.shape, v.dt)
        return self.materialize_elementwise(v.dt, v.shape, [v], lambda e: e[0], layout)

    # -- shared-memory redistribution --------------------------------------

    def convert(self, v: Val, layout: Layout, shape) -> Val:
        """Redistribute register tile ``v`` so that ``layout`` (consumer shape
        ``shape``) can read it in place: owners write the tile to shared
        memory, every thread reads back the elements its consumer slots need."""
        key = (v.name, v.layout.key(), layout.key(), tuple(shape))
        if key in self.conv_cache:
            return self.conv_cache[key]
        src = v.layout
        numel = int(np.prod(v.shape)) if v.shape else 1
        ct = DT.ctype(v.dt)
        stype = ct if ct in ("float", "double", "tila::i32", "tila::u32", "tila::i64", "tila::u64") else "tila::i32"
        esize = 8 if stype in ("double", "tila::i64", "tila::u64") else 4
        nbytes = numel * esize
        if nbytes > self.MAX_SCRATCH:
            self.fail(f"tile of {numel} elements too large to redistribute through shared memory")
        self.smem.need_scratch(nbytes)
        dst_layout = self._layout_for_operand(layout, shape, v.shape)
        name = self.fresh("cv")
        self.emit(f"{ct} {name}[{dst_layout.nreg}];")
        self.emit(f"{{ // redistribute {v.name}: {type(src).__name__} -> {type(dst_layout).__name__}")
        self.indent += 1
        buf = self.fresh("xs")
        self.emit("__syncthreads();")
        self.emit(f"{stype}* {buf} = reinterpret_cast<{stype}*>(tila_scratch);")
        sdims = list(v.shape)
        strides = [int(np.prod(sdims[i + 1:])) for i in range(len(sdims))]

        def flat_of(crd):
            return " + ".join(f"({c}) * {st}" for c, st in zip(crd, strides)) or "0"

        own = owner_predicate(src)
        if own == "PER_SLOT" or (isinstance(src, Derived) and not src.reg_affine()):
            for r in range(src.nreg):
                cond = self._owner_cond(src, r)
                pre = f"if ({cond}) " if cond else ""
                self.emit(f"{pre}{buf}[{flat_of(src.coord(r))}] = ({stype}){v.name}[{r}];")
        else:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {src.nreg}; ++r) {{")
            pre = f"if ({own}) " if own else ""
            self.emit(f"  {pre}{buf}[{flat_of(src.coord('r'))}] = ({stype}){v.name}[r];")
            self.emit("}")
        self.emit("__syncthreads();")
        dvalid = dst_layout.valid_expr()
        zero = DT.literal(v.dt, 0)

        def rd(fl):
            return f"({dvalid}) ? ({ct}){buf}[{fl}] : {zero}" if dvalid else f"({ct}){buf}[{fl}]"
        if isinstance(dst_layout, Derived) and not dst_layout.reg_affine():
            for r in range(dst_layout.nreg):
                self.emit(f"{name}[{r}] = {rd(flat_of(dst_layout.coord(r)))};")
        else:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {dst_layout.nreg}; ++r) {name}[r] = {rd(flat_of(dst_layout.coord('r')))};")
        self.indent -= 1
        self.emit("}")
        out = Val("reg", v.dt, tuple(v.shape), name=name, layout=dst_layout)
        self.conv_cache[key] = out
        return out

    def _layout_for_operand(self, consumer: Layout, cshape, oshape) -> Layout:
        """A layout of shape ``oshape`` whose slots line up with ``consumer``
        (shape ``cshape``) under broadcasting, i.e. thread t slot r holds the
        operand element that consumer slot r of thread t needs."""
        oshape = tuple(oshape)
        cshape = tuple(cshape)
        if oshape == cshape:
            return consumer
        return _BroadcastView(consumer, cshape, oshape)

    # -- TMEM --------------------------------------------------------------

    def tmem_to_reg(self, v: Val) -> Val:
        if getattr(v, "pending", None) and self.actx is not None:
            self.emit_acc_wait(v.pending, release=True)
        layout = TmemRows(tuple(v.shape), self.T)
        name = self.fresh("acc")
        n = layout.nreg
        self.emit(f"float {name}[{n}];")
        col = f"tila_tmem + ({v.tmem_col})" + (f" + (tid >> 7) * {layout.cpg}" if layout.groups > 1 else "")
        self.emit(f"tila::tc_fence_after();")
        self.emit(f"tila::tmem_load_row<{n}>({col} + ((tid & 96u) << 16), {name});")
        return Val("reg", v.dt, v.shape, name=name, layout=layout)

    # -- operands -------------------------------------------------------------

    def value(self, x) -> Val:
        if isinstance(x, T_.TName):
            return self.name_value(x.name)
        if isinstance(x, T_.TLit):
            return self.literal(x)
        return self.expr(x)

    def name_value(self, name) -> Val:
        if name in self.env:
            return self.env[name]
        if name in self.consts:
            c = self.consts[name]
            if type(c) is bool:
                return Val("scalar", D.bool_, expr="true" if c else "false", const=c)
            return Val("scalar", D.i32, expr=DT.int_literal(D.i32, c), const=c)
        if name in self.scalar_params:
            p = self.scalar_params[name]
            return Val("scalar", p.dtype, expr=self.scalar_param_expr(p))
        if name in self.ptr_params:
            return Val("ptr", self.ptr_params[name].vtype.elem, ptr=(name, None))
        self.fail(f"unbound name {name!r}")

    def scalar_param_expr(self, p):
        n = f"p_{p.name}"
        if p.dtype.name == "f16":
            return f"tila::h2f({n})"
        if p.dtype.name == "bf16":
            return f"tila::bf2f({n})"
        return n

    def literal(self, x, dt=None) -> Val:
        dt = x.dtype or dt
        v = x.value
        if dt is None:
            if isinstance(v, bool):
                dt = D.bool_
            elif isinstance(v, int):
                dt = D.i32
            else:
                dt = D.f32
        return Val("scalar", dt, expr=DT.literal(dt, v), const=v)

    # -- expressions -------------------------------------------------------

    def expr(self, x) -> Val:
        m = getattr(self, f"e_{type(x).__name__}", None)
        if m is None:
            self.fail(f"unsupported TIR expression {type(x).__name__}", getattr(x, "line", 0))
        return m(x)

    def e_TPid(self, x):
        return Val("scalar", D.i32, expr=self._pid_expr.get(x.axis, f"pid_{x.axis}"))

    def e_TNumPrograms(self, x):
        return Val("scalar", D.i32, expr=f"nprog_{x.axis}")

    def e_TArange(self, x):
        end = self.value(x.end)
        start = int(x.start)
        _, shape, _ = self.vt_info(x.vt)
        return Val("func", D.i32, shape,
                   fn=lambda idx, s=start: f"((tila::i32)({s} + ({idx[0]})))" if s else f"((tila::i32)({idx[0]}))")

    def e_TZeros(self, x):
        dt, shape, _ = self.vt_info(x.vt)
        zero = DT.literal(dt, 0)
        return Val("func", dt, shape, fn=lambda idx, z=zero: z, zero=True)

    def e_TConstant(self, x):
        return Val("scalar", x.dtype, expr=DT.constant_bits(x.dtype, x.bits))

    def e_TExpand(self, x):
        v = self.value(x.operand)
        if v.kind == "scalar":
            self.fail("expand of a scalar")
        ax = int(x.axis)
        if ax < 0:
            ax += len(v.shape) + 1
        if not 0 <= ax <= len(v.shape):
            self.fail(f"expand axis {x.axis} out of range")
        shape = tuple(v.shape[:ax]) + (1,) + tuple(v.shape[ax:])
        if v.kind == "tmem":
            v = self.tmem_to_reg(v)
        if v.kind == "func":
            # the inserted unit axis carries no index
            return Val("func", v.dt, shape, fn=lambda idx, f=v.fn, a=ax: f(tuple(idx[:a]) + tuple(idx[a + 1:])),
                       zero=v.zero)
        if v.kind == "reg":
            lay = Derived(v.layout, ("expand", ax), shape, tuple(range(v.layout.nreg)))
            return Val("reg", v.dt, shape, name=v.name, layout=lay)
        self.fail("expand of this value kind is not supported")

    def e_TReshape(self, x):
        v = self.value(x.operand)
        dt, shape, _ = self.vt_info(x.vt)
        if v.kind == "func":
            old = v.shape
            def fn(idx, f=v.fn, old=old, new=shape):
                flat = " + ".join(f"({i}) * {int(np.prod(new[k + 1:]))}" for k, i in enumerate(idx))
                oidx = tuple(f"((({flat}) / {int(np.prod(old[k + 1:]))}) % {old[k]})"
                             for k in range(len(old)))
                return f(oidx)
            return Val("func", v.dt, shape, fn=fn, zero=v.zero)
        if v.kind == "tmem":
            v = self.tmem_to_reg(v)
        if v.kind == "reg":
            lay = Derived(v.layout, ("reshape", shape), shape, tuple(range(v.layout.nreg)))
            return Val("reg", v.dt, shape, name=v.name, layout=lay)
        self.fail("reshape of this value kind is not supported")

    def e_TCast(self, x):
        v = self.value(x.operand)
        dst = x.dtype
        op = x.operand
        if DT.is_int(dst) and v.kind == "scalar" and type(v.const) is int and (
                isinstance(op, T_.TLit) and type(op.value) is int
                or isinstance(op, T_.TName) and op.name in self.consts
                or isinstance(op, (T_.TBin, T_.TUna)) and getattr(op, "staged", False)):
            # an integer literal, Const or staged constant converts by its exact
            # value modulo 2^bits, not through the dtype the literal carries
            # (cast[i64](-4294967296) is -4294967296; lowering.py:506-510 folds
            # the same way before the tensor conversion)
            return Val("scalar", dst, expr=DT.int_literal(dst, v.const), const=v.const)
        if v.kind == "scalar":
            return Val("scalar", dst, expr=DT.convert(v.dt, dst, v.expr))
        if v.kind == "func":
            return Val("func", dst, v.shape, fn=lambda idx, f=v.fn, s=v.dt: DT.convert(s, dst, f(idx)),
                       zero=v.zero)
        return self.materialize_elementwise(dst, v.shape, [v], lambda e, s=v.dt: DT.convert(s, dst, e[0]))

    def e_TWhere(self, x):
        dt, shape, _ = self.vt_info(x.vt)
        c, a, b = self.value(x.cond), self.value(x.a), self.value(x.b)
        a = self.coerce(a, dt)
        b = self.coerce(b, dt)
        def mk(e):
            return f"(({e[0]}) ? ({e[1]}) : ({e[2]}))"
        return self.combine(dt, shape, [c, a, b], mk)

    def coerce(self, v: Val, dt) -> Val:
        """Literal / differently typed operand -> value of dtype dt."""
        if v.dt is dt or v.dt.name == dt.name:
            return v
        if v.kind == "scalar":
            if v.const is not None and not isinstance(v.const, bool) and v.expr is not None \
                    and not v.expr.startswith("p_"):
                try:
                    return Val("scalar", dt, expr=DT.literal(dt, v.const), const=v.const)
                except (ValueError, OverflowError):
                    pass
            return Val("scalar", dt, expr=DT.convert(v.dt, dt, v.expr))
        if v.kind == "func":
            return Val("func", dt, v.shape, fn=lambda idx, f=v.fn, s=v.dt: DT.convert(s, dt, f(idx)),
                       zero=v.zero)
        return self.materialize_elementwise(dt, v.shape, [v], lambda e, s=v.dt: DT.convert(s, dt, e[0]))

    def combine(self, dt, shape, operands, mk):
        """Element-wise combination: scalar if all scalar, func if no operand
        is materialised, else a new register tile."""
        if not shape:
            if all(o.kind == "scalar" for o in operands):
                return Val("scalar", dt, expr=mk([o.expr for o in operands]))
            self.fail("scalar result from tile operands")
        if all(o.kind in ("scalar", "func") for o in operands):
            def fn(idx, ops=tuple(operands), shape=tuple(shape)):
                es = []
                for o in ops:
                    if o.kind == "scalar":
                        es.append(o.expr)
                    else:
                        es.append(o.fn(self.bcast_idx(idx, o.shape)))
                return mk(es)
            return Val("func", dt, tuple(shape), fn=fn)
        return self.materialize_elementwise(dt, shape, operands, mk)

    def e_TUna(self, x):
        v = self.value(x.operand)
        dt, shape, _ = self.vt_info(x.vt)
        op = x.op
        if op in ("any", "all"):
            return self.reduce_mask(v, op)
        if op in ("exp", "exp2"):
            fn = "exp" if op == "exp" else "exp2"
            if dt.name == "f64":
                mk = lambda e: f"{fn}((double)({e[0]}))"
            elif op == "exp2":
                # ex2.approx.f32: relative error <= 2^-22.5, subnormals kept
                # (tensor-core kernels flush subnormal results; see tila_exp2_f32)
                mk = lambda e: DT.round_to(dt, f"tila_exp2_f32((float)({e[0]}))")
            else:
                mk = lambda e: DT.round_to(dt, f"{fn}f((float)({e[0]}))")
            if v.kind == "scalar":
                return Val("scalar", dt, expr=mk([v.expr]))
            v = self.coerce(v, dt) if v.dt.name != dt.name else v
            # transcendental results are always materialised (no re-evaluation)
            return self.materialize_elementwise(dt, shape, [v], mk)
        if op == "-":
            if DT.is_int(dt) and not x.staged:
                mk = lambda e: f"tila::wneg<{DT.ctype(dt)}>({e[0]})"
            elif DT.is_float(dt):
                mk = lambda e: f"(-({e[0]}))"
            else:
                mk = lambda e: f"(-({e[0]}))"
            if v.kind == "scalar" and v.const is not None and x.staged:
                return Val("scalar", dt, expr=DT.literal(dt, -v.const), const=-v.const)
        elif op == "+":
            mk = lambda e: e[0]
        elif op == "~":
            if dt.name == "bool":
                mk = lambda e: f"(!({e[0]}))"
            else:
                mk = lambda e: f"(({DT.ctype(dt)})(~({e[0]})))"
        elif op == "not":
            mk = lambda e: f"(!({e[0]}))"
        else:
            self.fail(f"unsupported unary op {op}")
        return self.combine(dt, shape, [v], mk)

    @staticmethod
    def _has_effects(node):
        """``node`` contains an atomic or a memory load (evaluating it is observable)."""
        from .pipeline import _walk
        found = [False]
        _walk(node, lambda n: found.__setitem__(0, found[0] or isinstance(n, (T_.TAtomicAdd, T_.TLoad))))
        return found[0]

    def e_TBin(self, x):
        dt, shape, is_ptr = self.vt_info(x.vt)
        op = x.op
        fused = self._try_contract(x, dt, shape)
        if fused is not None:
            return fused
        l = self.value(x.left)
        if op in ("and", "or") and l.kind == "scalar" and l.const is not None:
            if op == "and" and not l.const:
                return Val("scalar", D.bool_, expr="false", const=False)
            if op == "or" and l.const:
                return Val("scalar", D.bool_, expr="true", const=True)
        if op in ("and", "or") and l.kind == "scalar" and not shape and self._has_effects(x.right):
            # Python's short circuit: the right operand (an atomic, a load)
            # runs only when the left one does not decide the result.  The
            # left operand is uniform, so every thread takes the same branch.
            v = self.fresh("sc")
            self.emit(f"bool {v} = ({l.expr});")
            self.emit(f"if ({'' if op == 'and' else '!'}{v}) {{")
            self.indent += 1
            saved_conv = dict(self.conv_cache)      # values made inside the block stay there
            r = self.value(x.right)
            if r.kind != "scalar":
                self.fail("short-circuit operand is not a scalar", getattr(x, "line", 0))
            self.emit(f"{v} = ({r.expr});")
            self.conv_cache = saved_conv
            self.indent -= 1
            self.emit("}")
            return Val("scalar", D.bool_, expr=v)
        r = self.value(x.right)
        if is_ptr:
            self.fail("pointer arithmetic tiles are not supported yet")
        if x.staged and l.const is not None and r.const is not None:
            val = self._py_bin(op, l.const, r.const)
            rdt = dt if dt.name != "bool" or isinstance(val, bool) else D.bool_
            return Val("scalar", rdt, expr=DT.literal(rdt, val), const=val)
        odt = x.operand_dtype or (dt if dt.name != "bool" else None)
        if odt is None:
            odt = l.dt if l.const is None else r.dt
        if op in ("and", "or"):
            mk = (lambda e: f"(({e[0]}) && ({e[1]}))") if op == "and" else (lambda e: f"(({e[0]}) || ({e[1]}))")
            return self.combine(D.bool_, shape, [l, r], mk)
        l = self.coerce(l, odt)
        r = self.coerce(r, odt)
        mode = getattr(self, "_guard_mode", None)
        if mode and op in ("<", "<=") and shape and r.kind == "scalar" and l.kind == "func":
            g = self._bound_guard(x, l, r, op, shape)
            if g is not None:
                if mode == "collect":
                    self._guards.append(g)
                elif g in self._guard_set:
                    return Val("func", D.bool_, tuple(shape), fn=lambda idx: "true")
        mk = self._bin_maker(op, odt, dt)
        return self.combine(dt, shape, [l, r], mk)

    def _try_contract(self, x, dt, shape):
        """In kernels with dots (compiled with multiply-add contraction, like
        nvcc's default), an f32 tile sum whose operand is an unnamed product,
        (a * b) + c, becomes one FMA per element."""
        if x.op != "+" or not self.dot_rows or dt.name != "f32" or not shape or x.staged:
            return None
        for prod, other in ((x.left, x.right), (x.right, x.left)):
            if isinstance(prod, T_.TBin) and prod.op == "*" and not prod.staged:
                pdt, pshape, pptr = self.vt_info(prod.vt)
                if pdt.name != "f32" or pptr or tuple(pshape) != tuple(shape):
                    continue
                a = self.coerce(self.value(prod.left), D.f32)
                b = self.coerce(self.value(prod.right), D.f32)
                c = self.coerce(self.value(other), D.f32)
                self._contracted = True
                return self.combine(dt, shape, [a, b, c], _PackedFma())
        return None

    @staticmethod
    def _py_bin(op, a, b):
        import operator as o
        return {"+": o.add, "-": o.sub, "*": o.mul, "//": o.floordiv, "%": o.mod,
                "<": o.lt, "<=": o.le, ">": o.gt, ">=": o.ge, "==": o.eq, "!=": o.ne,
                "&": o.and_, "|": o.or_, "^": o.xor, "<<": o.lshift, ">>": o.rshift,
                "/": o.truediv}[op](a, b)

    def _bin_maker(self, op, odt, rdt):
        ct = DT.ctype(odt)
        if op in ("<", "<=", ">", ">=", "==", "!="):
            return lambda e: f"(({e[0]}) {op} ({e[1]}))"
        if odt.name == "bool":
            if op in ("&", "|", "^"):
                return lambda e: f"((bool)(({e[0]}) {op} ({e[1]})))"
            self.fail(f"operator {op} on masks")
        if DT.is_float(odt):
            if op == "/" and odt.name == "f32" and rdt.name == "f32":
                return _UniformDivisor()
            if op in ("+", "-", "*") and odt.name == "f32" and rdt.name == "f32":
                return _PackedBin(op)
            if op in ("+", "-", "*", "/"):
                return lambda e: DT.round_to(rdt, f"(({e[0]}) {op} ({e[1]}))")
            if op == "//":
                return lambda e: DT.round_to(rdt, f"tila::py_floordiv(({e[0]}), ({e[1]}))")
            if op == "%":
                return lambda e: DT.round_to(rdt, f"tila::py_mod(({e[0]}), ({e[1]}))")
            self.fail(f"operator {op} on floats")
        # integers: wrapping, floor division (ADR-007)
        if op == "+":
            return lambda e: f"tila::wadd<{ct}>({e[0]}, {e[1]})"
        if op == "-":
            return lambda e: f"tila::wsub<{ct}>({e[0]}, {e[1]})"
        if op == "*":
            return lambda e: f"tila::wmul<{ct}>({e[0]}, {e[1]})"
        if op == "//":
            mn = DT.int_literal(odt, DT.int_min(odt))
            return lambda e: f"tila::floordiv<{ct}>({e[0]}, {e[1]}, {mn})"
        if op == "%":
            mn = DT.int_literal(odt, DT.int_min(odt))
            return lambda e: f"tila::floormod<{ct}>({e[0]}, {e[1]}, {mn})"
        if op in ("&", "|", "^"):
            return lambda e: f"(({ct})(({e[0]}) {op} ({e[1]})))"
        if op == "<<":
            ut = DT.ctype(self._unsigned(odt))
            return lambda e: f"(({ct})(({ut})({e[0]}) << ({e[1]})))"
        if op == ">>":
            return lambda e: f"(({ct})(({e[0]}) >> ({e[1]})))"
        if op == "/":
            return lambda e: f"((float)({e[0]}) / (float)({e[1]}))"
        self.fail(f"unsupported binary op {op}")

    @staticmethod
    def _unsigned(dt):
        return {"i8": D.u8, "i16": D.u16, "i32": D.u32, "i64": D.u64}.get(dt.name, dt)

    # -- reductions ----------------------------------------------------------

    def reduce_mask(self, v: Val, op):
        """any/all of a Mask -> scalar bool (interp.py:261-264)."""
        if v.kind == "scalar":
            return Val("scalar", D.bool_, expr=f"((bool)({v.expr}))")
        m = self.materialize(v)
        as_int = Val("reg", D.i32, m.shape, name=None, layout=m.layout)
        name = self.fresh("mi")
        lay = m.layout
        self.emit(f"tila::i32 {name}[{lay.nreg}];")
        want = "1" if op == "any" else "0"
        self.emit("#pragma unroll")
        self.emit(f"for (int r = 0; r < {lay.nreg}; ++r) {name}[r] = ({m.name}[r] ? 1 : 0) == {want} ? 1 : 0;")
        as_int.name = name
        total = self._full_reduce(as_int, "max", D.i32)
        return Val("scalar", D.bool_, expr=f"(({total.expr}) {'!=' if op == 'any' else '=='} 0)")

    def e_TReduce(self, x):
        v = self.value(x.operand)
        dt, shape, _ = self.vt_info(x.vt)
        acc_dt = x.accumulation_dtype
        if v.kind == "scalar":
            self.fail("reduction of a scalar")
        if v.kind == "tmem":
            v = self.tmem_to_reg(v)
        if v.kind == "func":
            v = self.materialize(v)
        rank = len(v.shape)
        axis = x.axis
        if rank == 1:
            res = self._full_reduce(v, x.op, acc_dt)
            return Val("scalar", dt, expr=DT.convert(acc_dt, dt, res.expr) if acc_dt is not dt else res.expr)
        return self._axis_reduce(v, x.op, axis, acc_dt, dt)

    def _fold(self, op, dt):
        if op == "sum":
            if DT.is_int(dt):
                return lambda a, b: f"tila::wadd<{DT.ctype(dt)}>({a}, {b})"
            return lambda a, b: f"(({a}) + ({b}))"
        if DT.is_float(dt):
            return lambda a, b: f"tila::max_nan({a}, {b})"
        return lambda a, b: f"tila::max_int<{DT.ctype(dt)}>({a}, {b})"

    def _thread_tree(self, op, dt, exprs):
        """In-thread reduction of ``exprs`` (C++ expressions): f32 sums of 8 or
        more terms use two interleaved trees in f32x2 lanes; otherwise a
        balanced pairwise tree (short dependency chains)."""
        fold = self._fold(op, dt)
        if op == "sum" and dt.name == "f32" and len(exprs) % 2 == 0 and len(exprs) >= 8:
            pairs = [f"tila::pk2({exprs[i]}, {exprs[i + 1]})" for i in range(0, len(exprs), 2)]
            t = self.fresh("ps")
            self.emit(f"const tila::u64 {t} = {_tree_fold(pairs, lambda a, b: f'tila::add2({a}, {b})')};")
            return f"((tila::lo2({t})) + (tila::hi2({t})))"
        return _tree_fold(exprs, fold)

    def _identity(self, op, dt):
        if op == "sum":
            return DT.literal(dt, 0)
        if DT.is_float(dt):
            return "(-__int_as_float(0x7f800000))" if dt.name != "f64" else "(-__longlong_as_double(0x7ff0000000000000LL))"
        if DT.is_signed(dt):
            return DT.int_literal(dt, DT.int_min(dt))
        return DT.int_literal(dt, 0)

    def _owner_cond(self, layout, r):
        own = owner_predicate(layout)
        if own is None:
            return None
        if own == "PER_SLOT":
            from .layouts import _tid_set_expr
            coords, owners = layout._tables
            tids = np.nonzero(owners[:, r])[0]
            e = _tid_set_expr(tids, layout.T)
            if e is None:
                e = " || ".join(f"tid == {t}" for t in tids) or "false"
            return e
        return own

    def _full_reduce(self, v: Val, op, acc_dt) -> Val:
        """Reduce every element of a register tile to one uniform scalar."""
        lay = v.layout
        ct = DT.ctype(acc_dt)
        fold = self._fold(op, acc_dt)
        part = self.fresh("part")
        self.emit(f"{ct} {part} = {self._identity(op, acc_dt)};")
        own = owner_predicate(lay)
        src_dt = v.dt
        conv = (lambda e: DT.convert(src_dt, acc_dt, e)) if src_dt.name != acc_dt.name else (lambda e: e)
        if own == "PER_SLOT":
            for r in range(lay.nreg):
                c = self._owner_cond(lay, r)
                self.emit(f"if ({c}) {part} = {fold(part, conv(f'{v.name}[{r}]'))};")
        else:
            # a short tree inside the thread (see _thread_tree)
            self.emit(f"{part} = {self._thread_tree(op, acc_dt, [conv(f'{v.name}[{r}]') for r in range(lay.nreg)])};")
            if own is not None:
                self.emit(f"if (!({own})) {part} = {self._identity(op, acc_dt)};")
        return Val("scalar", acc_dt, expr=self._cta_allreduce(part, op, acc_dt))

    def _cta_allreduce(self, part, op, dt) -> str:
        """All threads' partials -> one value visible to every thread."""
        ct = DT.ctype(dt)
        fold = self._fold(op, dt)
        for m in (16, 8, 4, 2, 1):
            self.emit(f"{part} = {fold(part, f'tila::shfl_xor({part}, {m})')};")
        W = self.T // 32
        if W == 1:
            return part
        esize = 8 if DT.size(dt) == 8 else 4
        self.smem.need_red(W * esize)
        buf = self.fresh("red")
        out = self.fresh("tot")
        self.emit(f"{ct}* {buf} = reinterpret_cast<{ct}*>(tila_red + tila_rsel);")
        self.emit(f"if ((tid & 31) == 0) {buf}[tid >> 5] = {part};")
        self.emit("__syncthreads();")
        self.emit(f"{ct} {out} = {buf}[0];")
        self.emit("#pragma unroll")
        self.emit(f"for (int w = 1; w < {W}; ++w) {out} = {fold(out, f'{buf}[w]')};")
        self.emit("tila_rsel ^= tila_red_half;")
        return out

    def _axis_reduce(self, v: Val, op, axis, acc_dt, out_dt) -> Val:
        lay = v.layout
        if v.shape[axis] == 1:
            # reducing a unit axis: the value itself, re-typed (interp np.sum/np.max)
            keep = tuple(n for i, n in enumerate(v.shape) if i != axis)
            dl = Derived(lay, ("slice", axis), keep, tuple(range(lay.nreg)))
            conv = lambda e: DT.convert(v.dt, out_dt, DT.convert(v.dt, acc_dt, e[0]))
            src = Val("reg", v.dt, keep, name=v.name, layout=dl)
            return self.materialize_elementwise(out_dt, keep, [src], conv, layout=dl)
        if isinstance(lay, Derived) or not hasattr(lay, "reduce_bits"):
            lay2 = self.default_layout(v.shape, v.dt)
            if isinstance(lay2, (Blocked, TmemRows)) and lay2 != lay:
                v = self.materialize(v, lay2)
                lay = lay2
            elif not isinstance(lay, (Blocked, TmemRows)):
                lay = Blocked(tuple(v.shape), self.T, 1)
                v = self.materialize(v, lay)
        coords, owners = lay._tables
        keep_shape = tuple(n for i, n in enumerate(v.shape) if i != axis)
        # group the thread's slots by output coordinate (thread independent)
        t0 = coords[0]
        groups = {}
        for r in range(lay.nreg):
            key = tuple(int(c) for i, c in enumerate(t0[r]) if i != axis)
            groups.setdefault(key, []).append(r)
        outs = list(groups.values())
        # the output slot's representative parent slot
        regs = tuple(g[0] for g in outs)
        ct = DT.ctype(acc_dt)
        fold = self._fold(op, acc_dt)
        ident = self._identity(op, acc_dt)
        conv = (lambda e: DT.convert(v.dt, acc_dt, e)) if v.dt.name != acc_dt.name else (lambda e: e)
        name = self.fresh("rd")
        n = len(outs)
        self.emit(f"{ct} {name}[{n}];")
        own = owner_predicate(lay)
        for k, g in enumerate(outs):
            self.emit(f"{name}[{k}] = {self._thread_tree(op, acc_dt, [conv(f'{v.name}[{r}]') for r in g])};")
        if own is not None and own != "PER_SLOT":
            self.emit(f"if (!({own})) {{")
            self.emit(f"  #pragma unroll")
            self.emit(f"  for (int k = 0; k < {n}; ++k) {name}[k] = {ident};")
            self.emit("}")
        bits = lay.reduce_bits(axis)
        lane_bits = [b for b in bits if b < 5]
        warp_bits = [b for b in bits if b >= 5]
        for b in lane_bits:
            self.emit("#pragma unroll")
            self.emit(f"for (int k = 0; k < {n}; ++k) {name}[k] = {fold(f'{name}[k]', f'tila::shfl_xor({name}[k], {1 << b})')};")
        if warp_bits:
            # shared-memory stage across warps: slot [group][output], so the
            # lanes of a warp (consecutive outputs) touch consecutive words
            G = 1 << len(warp_bits)
            numel_out = int(np.prod(keep_shape))
            esize = 8 if DT.size(acc_dt) == 8 else 4
            self.smem.need_red(numel_out * G * esize)
            buf = self.fresh("rs")
            self.emit(f"{ct}* {buf} = reinterpret_cast<{ct}*>(tila_red + tila_rsel);")
            gexpr = " | ".join(f"(((tid >> {b}) & 1) << {i})" for i, b in enumerate(warp_bits))
            lane_mask = sum(1 << b for b in lane_bits)
            out_lay = Derived(lay, ("slice", axis), keep_shape, regs)
            oc = out_lay.coord("k") if False else None
            self.emit(f"const int {buf}_g = {gexpr};")
            lvalid = lay.valid_expr()
            for k in range(n):
                crd = out_lay.coord(k)
                flat = " + ".join(f"({c}) * {int(np.prod(keep_shape[i + 1:]))}" for i, c in enumerate(crd)) or "0"
                conds = ([f"(tid & {lane_mask}) == 0"] if lane_mask else []) + ([f"({lvalid})"] if lvalid else [])
                cond = f"if ({' && '.join(conds)}) " if conds else ""
                self.emit(f"{cond}{buf}[{buf}_g * {numel_out} + ({flat})] = {name}[{k}];")
            self.emit("__syncthreads();")
            for k in range(n):
                crd = out_lay.coord(k)
                flat = " + ".join(f"({c}) * {int(np.prod(keep_shape[i + 1:]))}" for i, c in enumerate(crd)) or "0"
                acc = f"{buf}[({flat})]"
                for gi in range(1, G):
                    acc = fold(acc, f"{buf}[{gi * numel_out} + ({flat})]")
                pre = f"if ({lvalid}) " if lvalid else ""
                self.emit(f"{pre}{name}[{k}] = {acc};")
            self.emit("tila_rsel ^= tila_red_half;")
        out_lay = Derived(lay, ("slice", axis), keep_shape, regs, owner_fn=dedupe_owner)
        res = Val("reg", acc_dt, keep_shape, name=name, layout=out_lay)
        if acc_dt.name != out_dt.name:
            res = self.materialize_elementwise(out_dt, keep_shape, [res],
                                              lambda e: DT.convert(acc_dt, out_dt, e[0]), layout=out_lay)
        return res

    # -- memory ----------------------------------------------------------------

    def address_terms(self, buffer, coords, layout, r, smaps):
        """Element offset (i64 C++ expr) of a buffer access at slot r."""
        terms = []
        info = self.buffers.get(buffer)
        for i, c in enumerate(coords):
            e = self.elem(c, layout, r, smaps[i]) if layout is not None else c.expr
            if info is not None and info.unit_last and i == len(coords) - 1:
                terms.append(f"(tila::i64)({e})")
            else:
                terms.append(f"(tila::i64)p_{buffer}_stride{i} * (tila::i64)({e})")
        return " + ".join(terms) if terms else "0"

    def _affine_last(self, node, depth=0):
        """Coefficient of the tile's last index in a coordinate expression:
        returns (coef, divisor) where coef in {0, 1, None} and divisor is a
        power of two dividing the index-independent part (lowering.py:374-416
        hints, restated as a structural analysis)."""
        if depth > 40:
            return None, 1
        if isinstance(node, T_.TName):
            if node.name in self.consts:
                c = self.consts[node.name]
                return 0, _pow2_div(c) if type(c) is int else 1
            if node.name in self._defs:
                return self._affine_last(self._defs[node.name], depth + 1)
            if node.name in self._loopvars:
                return 0, self._loopvars[node.name]
            return (0, 1) if node.name in self.scalar_params or node.name in self._pidnames else (None, 1)
        if isinstance(node, T_.TLit):
            return (0, _pow2_div(node.value)) if isinstance(node.value, int) and not isinstance(node.value, bool) else (None, 1)
        if isinstance(node, T_.TPid):
            return 0, 1
        if isinstance(node, T_.TArange):
            return (1, _pow2_div(int(node.start)))
        if isinstance(node, T_.TExpand):
            c, d = self._affine_last(node.operand, depth + 1)
            if c == 1 and node.axis == 1:
                return 0, 1 if True else d   # index moved to rows: no longer along the last dim
            return c, d
        if isinstance(node, T_.TBin):
            if node.op in ("+", "-"):
                c1, d1 = self._affine_last(node.left, depth + 1)
                c2, d2 = self._affine_last(node.right, depth + 1)
                if c1 is None or c2 is None:
                    return None, 1
                c = c1 + c2 if node.op == "+" else c1 - c2
                if c not in (0, 1):
                    return None, 1
                return c, min(d1, d2)
            if node.op == "*":
                c1, d1 = self._affine_last(node.left, depth + 1)
                c2, d2 = self._affine_last(node.right, depth + 1)
                if c1 == 0 and c2 == 0:
                    return 0, min(256, d1 * d2)
                return None, 1
        if isinstance(node, T_.TCast):
            return self._affine_last(node.operand, depth + 1)
        return None, 1

    def _vector_plan(self, buffer, coord_nodes, coords, layout, shape, dt):
        """Decide 128-bit access along the last tile dim.  Returns (width,
        static_aligned) or (1, False)."""
        info = self.buffers.get(buffer)
        if info is None or not shape or layout.vec <= 1:
            return 1, False
        # which coordinate carries the last tile index?
        unit_axis = None
        div = 256
        for i, (node, c) in enumerate(zip(coord_nodes, coords)):
            if c.kind == "scalar":
                d = self._affine_last(node)[1] if node is not None else 1
                div = min(div, d * info.stride_div[i])
                continue
            # a coordinate tile that does not vary along the last dim of the
            # access shape must be a broadcast (size 1 there)
            if c.shape and c.shape[-1] == 1 and len(c.shape) == len(shape):
                d = self._affine_last(node)[1] if node is not None else 1
                div = min(div, max(d, 1) * info.stride_div[i])
                continue
            coef, d = self._affine_last(node) if node is not None else (None, 1)
            if coef != 1 or c.kind not in ("func",):
                return 1, False
            if unit_axis is not None:
                return 1, False
            unit_axis = i
            div = min(div, d)
        if unit_axis is None or unit_axis != len(coords) - 1 or not info.unit_last:
            return 1, False
        esize = DT.size(dt)
        width = min(layout.vec, 16 // esize) if esize <= 16 else 1
        if width < 2:
            return 1, False
        aligned = (info.base_align >= width * esize) and (div % width == 0)
        return width, aligned

    def e_TLoad(self, x):
        dt, shape, _ = self.vt_info(x.vt)
        if x.buffer is None:
            return self.ptr_load(x, dt, shape)
        coords = [self.value(c) for c in x.coords]
        coords = [self.coerce(c, D.i64) if c.dt.name not in ("i32", "i64", "i16", "i8", "u8", "u16", "u32", "u64") else c
                  for c in coords]
        mask = self.value(x.mask) if x.mask is not None else None
        other = self.value(x.other) if x.other is not None else None
        if other is not None:
            other = self.coerce(other, dt)
        if not shape:
            return self._scalar_load(x.buffer, coords, mask, other, dt)
        layout = self.default_layout(shape, dt)
        return self._tile_load(x.buffer, list(x.coords), coords, mask, other, dt, shape, layout,
                               mask_node=x.mask)

    _PREFETCH_NAMES = re.compile(r"\b(?!tid\b|pid_[012]\b|p_\w+\b|nprog_[012]\b|pid_off_[012]\b|"
                                 r"launch_[012]\b|tila\b|r0\b|r\b|g\b|off\b|all\b|a_\b|int\b|bool\b|"
                                 r"const\b|true\b|false\b|return\b|pragma\b|unroll\b|for\b|if\b)"
                                 r"(?<!::)(?<![\w.])[A-Za-z_]\w*")

    def _prefetch_load(self, buffer, layout, groups, width, dt, off, lane_cond):
        """A load at the top level of the program (not in a loop or branch)
        whose addresses and bounds depend only on program ids, thread index
        and kernel parameters: the same groups are prefetched into L2 ahead of
        the grid-dependency wait (one thread per 64 bytes)."""
        if self._loopvars or self.actx is not None or self._guard_mode:
            return
        if DT.size(dt) * width != 16 or groups > 16 or not isinstance(layout, Blocked):
            return
        allc = "true" if lane_cond is None else \
            f"[&] {{ int r = r0; const bool a_ = {lane_cond}; r = r0 + {width - 1}; return a_ && ({lane_cond}); }}()"
        who = "(tid & 3) == 0" if layout.tc >= 4 else "true"
        code = (f"{{ // L2 prefetch of {buffer}\n"
                f"  #pragma unroll\n"
                f"  for (int g = 0; g < {groups}; ++g) {{\n"
                f"    const int r0 = g * {width};\n"
                f"    const tila::i64 off = {off};\n"
                f"    if (({who}) && {allc}) tila::prefetch_l2(p_{buffer} + off);\n"
                f"  }}\n"
                f"}}")
        if self._PREFETCH_NAMES.search(f"{off} {lane_cond or ''}"):
            return
        if len(self._prefetch) < 8:
            self._prefetch.append(code)

    def _scalar_load(self, buffer, coords, mask, other, dt):
        name = self.fresh("ld")
        addr = " + ".join(f"(tila::i64)p_{buffer}_stride{i} * (tila::i64)({c.expr})"
                          for i, c in enumerate(coords)) or "0"
        fill = other.expr if other is not None else DT.literal(dt, 0)
        load = DT.load_conv(dt, f"p_{buffer}[{addr}]")
        if mask is not None:
            self.emit(f"const {DT.ctype(dt)} {name} = ({mask.expr}) ? {load} : {fill};")
        else:
            self.emit(f"const {DT.ctype(dt)} {name} = {load};")
        return Val("scalar", dt, expr=name)

    def _tile_load(self, buffer, coord_nodes, coords, mask, other, dt, shape, layout, mask_node=None):
        top_level = self.indent == 2
        ops = list(coords) + ([mask] if mask is not None else []) + ([other] if other is not None else [])
        ops, maps, straight = self.prepare_operands(ops, layout, shape)
        nc = len(coords)
        coords = ops[:nc]
        mask = ops[nc] if mask is not None else None
        other = ops[nc + (1 if mask is not None else 0)] if other is not None else None
        cm = maps[:nc]
        mm = maps[nc] if mask is not None else None
        om = maps[nc + (1 if mask is not None else 0)] if other is not None else None
        width, aligned = self._vector_plan(buffer, coord_nodes, coords, layout, shape, dt)
        name = self.fresh("ld")
        ct, mt = DT.ctype(dt), DT.memtype(dt)
        self.emit(f"{ct} {name}[{layout.nreg}];")
        # padding lanes of the layout hold no tile element: never touch memory
        valid = layout.valid_expr()

        def cond_at(r, smap=None):
            parts = []
            if valid is not None:
                parts.append(f"({valid})")
            if mask is not None:
                parts.append(f"({self.elem(mask, layout, r, smap)})")
            return " && ".join(parts) if parts else None

        fill0 = DT.literal(dt, 0)
        if width > 1 and not straight:
            groups = layout.nreg // width
            vt = _vec_type(DT.size(dt) * width)
            self.emit("#pragma unroll")
            self.emit(f"for (int g = 0; g < {groups}; ++g) {{")
            self.indent += 1
            self.emit(f"const int r0 = g * {width};")
            off = self.address_terms(buffer, coords, layout, "r0", cm)
            self.emit(f"const tila::i64 off = {off};")
            lane_cond = cond_at("r")
            interval = lane_cond is not None and (mask is None or self._interval_mask(mask_node))
            if interval:
                # the group's lanes where the mask holds are consecutive:
                # the first and the last lane decide the whole group
                self.emit(f"bool all; {{ int r = r0; const bool a_ = {lane_cond}; "
                          f"r = r0 + {width - 1}; all = a_ && ({lane_cond}); }}")
            elif lane_cond is not None:
                self.emit(f"bool m[{width}];")
                self.emit("bool all = true;")
                self.emit("#pragma unroll")
                self.emit(f"for (int j = 0; j < {width}; ++j) {{ const int r = r0 + j; m[j] = {lane_cond}; all = all && m[j]; }}")
            else:
                self.emit("const bool all = true;")
            if top_level and (lane_cond is None or interval):
                self._prefetch_load(buffer, layout, groups, width, dt, off, lane_cond)
            cond = "all" if aligned else f"all && ((reinterpret_cast<unsigned long long>(p_{buffer} + off) & {DT.size(dt) * width - 1}) == 0)"
            self.emit(f"if ({cond}) {{")
            self.emit(f"  const {vt} w = *reinterpret_cast<const {vt}*>(p_{buffer} + off);")
            self.emit(f"  const {mt}* e = reinterpret_cast<const {mt}*>(&w);")
            self.emit("  #pragma unroll")
            self.emit(f"  for (int j = 0; j < {width}; ++j) {name}[r0 + j] = {DT.load_conv(dt, 'e[j]')};")
            self.emit("} else {")
            self.emit("  #pragma unroll")
            self.emit(f"  for (int j = 0; j < {width}; ++j) {{")
            self.emit("    const int r = r0 + j;")
            offr = self.address_terms(buffer, coords, layout, "r", cm)
            fill = self.elem(other, layout, "r") if other is not None else fill0
            mcond = (f"({lane_cond})" if interval else "m[j]") if lane_cond is not None else "true"
            self.emit(f"    {name}[r] = {mcond} ? {DT.load_conv(dt, f'p_{buffer}[{offr}]')} : {fill};")
            self.emit("  }")
            self.emit("}")
            self.indent -= 1
            self.emit("}")
        else:
            rng = range(layout.nreg) if straight else ["r"]
            if not straight:
                self.emit("#pragma unroll")
                self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
                self.indent += 1
            for r in rng:
                off = self.address_terms(buffer, coords, layout, r, cm)
                fill = self.elem(other, layout, r, om) if other is not None else fill0
                ld = DT.load_conv(dt, f"p_{buffer}[{off}]")
                c = cond_at(r, mm)
                if c is not None:
                    self.emit(f"{name}[{r}] = ({c}) ? {ld} : {fill};")
                else:
                    self.emit(f"{name}[{r}] = {ld};")
            if not straight:
                self.indent -= 1
                self.emit("}")
        return Val("reg", dt, tuple(shape), name=name, layout=layout)

    def s_TStore(self, s):
        if s.buffer is None:
            return self.ptr_store(s)
        b = self.buffer_params[s.buffer]
        dt = b.vtype.elem
        coords = [self.value(c) for c in s.coords]
        value = self.value(s.value)
        mask = self.value(s.mask) if s.mask is not None else None
        shapes = [c.shape for c in coords] + [value.shape] + ([mask.shape] if mask is not None else [])
        shape = _broadcast_shapes(shapes)
        value = self.coerce(value, dt) if value.dt.name != dt.name else value
        if not shape:
            addr = " + ".join(f"(tila::i64)p_{s.buffer}_stride{i} * (tila::i64)({c.expr})"
                              for i, c in enumerate(coords)) or "0"
            st = f"p_{s.buffer}[{addr}] = {DT.store_conv(dt, value.expr)};"
            cond = "tid == 0" + (f" && ({mask.expr})" if mask is not None else "")
            self.emit(f"if ({cond}) {st}")
            return
        if value.kind == "tmem":
            value = self.tmem_to_reg(value)
        if self._try_tma_store(s, coords, value, shape, dt):
            return
        if value.kind == "reg" and tuple(value.shape) == tuple(shape):
            layout = value.layout
            if isinstance(layout, Derived) and not layout.reg_affine():
                pass
        else:
            layout = self.default_layout(shape, dt)
        ops = list(coords) + [value] + ([mask] if mask is not None else [])
        ops, maps, straight = self.prepare_operands(ops, layout, shape)
        nc = len(coords)
        coords, value = ops[:nc], ops[nc]
        mask = ops[nc + 1] if mask is not None else None
        cm, vm = maps[:nc], maps[nc]
        mm = maps[nc + 1] if mask is not None else None
        own = owner_predicate(layout)
        width, aligned = self._vector_plan(s.buffer, list(s.coords), coords, layout, shape, dt)
        if own == "PER_SLOT" or (isinstance(layout, Derived) and not layout.reg_affine()):
            straight = True
            width = 1
        mt = DT.memtype(dt)
        self.emit("{")
        self.indent += 1
        if own is not None and own != "PER_SLOT":
            self.emit(f"if ({own}) {{")
            self.indent += 1
        if width > 1 and not straight:
            groups = layout.nreg // width
            vt = _vec_type(DT.size(dt) * width)
            self.emit("#pragma unroll")
            self.emit(f"for (int g = 0; g < {groups}; ++g) {{")
            self.indent += 1
            self.emit(f"const int r0 = g * {width};")
            self.emit(f"const tila::i64 off = {self.address_terms(s.buffer, coords, layout, 'r0', cm)};")
            interval = mask is not None and self._interval_mask(s.mask)
            if interval:
                mexpr = self.elem(mask, layout, "r")
                self.emit(f"bool all; {{ int r = r0; const bool a_ = {mexpr}; "
                          f"r = r0 + {width - 1}; all = a_ && ({mexpr}); }}")
            elif mask is not None:
                self.emit(f"bool m[{width}];")
                self.emit("bool all = true;")
                self.emit("#pragma unroll")
                self.emit(f"for (int j = 0; j < {width}; ++j) {{ const int r = r0 + j; m[j] = {self.elem(mask, layout, 'r')}; all = all && m[j]; }}")
            else:
                self.emit("const bool all = true;")
            cond = "all" if aligned else f"all && ((reinterpret_cast<unsigned long long>(p_{s.buffer} + off) & {DT.size(dt) * width - 1}) == 0)"
            self.emit(f"if ({cond}) {{")
            self.emit(f"  {vt} w;")
            self.emit(f"  {mt}* e = reinterpret_cast<{mt}*>(&w);")
            self.emit("  #pragma unroll")
            self.emit(f"  for (int j = 0; j < {width}; ++j) {{ const int r = r0 + j; e[j] = {DT.store_conv(dt, self.elem(value, layout, 'r'))}; }}")
            self.emit(f"  *reinterpret_cast<{vt}*>(p_{s.buffer} + off) = w;")
            self.emit("} else {")
            self.emit("  #pragma unroll")
            self.emit(f"  for (int j = 0; j < {width}; ++j) {{")
            self.emit("    const int r = r0 + j;")
            offr = self.address_terms(s.buffer, coords, layout, "r", cm)
            mcond = (f"({self.elem(mask, layout, 'r')})" if interval else "m[j]") if mask is not None else "true"
            self.emit(f"    if ({mcond}) p_{s.buffer}[{offr}] = {DT.store_conv(dt, self.elem(value, layout, 'r'))};")
            self.emit("  }")
            self.emit("}")
            self.indent -= 1
            self.emit("}")
        else:
            rng = range(layout.nreg) if straight else ["r"]
            if not straight:
                self.emit("#pragma unroll")
                self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
                self.indent += 1
            for r in rng:
                off = self.address_terms(s.buffer, coords, layout, r, cm)
                val = DT.store_conv(dt, self.elem(value, layout, r, vm))
                conds = []
                if own == "PER_SLOT":
                    conds.append(self._owner_cond(layout, r))
                if mask is not None:
                    conds.append(f"({self.elem(mask, layout, r, mm)})")
                cond = f"if ({' && '.join(conds)}) " if conds else ""
                self.emit(f"{cond}p_{s.buffer}[{off}] = {val};")
            if not straight:
                self.indent -= 1
                self.emit("}")
        if own is not None and own != "PER_SLOT":
            self.indent -= 1
            self.emit("}")
        self.indent -= 1
        self.emit("}")

    def _try_tma_store(self, s, coords, value, shape, dt):
        """Store a 128-row f32 tile held in the tcgen05.ld register image
        (thread = row) with TMA: the rows go to shared memory in the
        SWIZZLE_128B box layout (conflict-free 16-byte writes), one thread
        issues the box stores, and global memory receives whole lines instead
        of 32 scattered 16-byte pieces per warp instruction."""
        from .pipeline import plan_tma_store
        if dt.name != "f32" or value.kind != "reg" or not isinstance(value.layout, TmemRows):
            return False
        lay = value.layout
        if len(shape) != 2 or tuple(value.shape) != tuple(shape) or shape[0] != 128 \
                or shape[1] % 32 or lay.cpg % 4 or self.T not in (128, 256):
            return False
        plan = plan_tma_store(s, tuple(shape), self.pdefs, self.consts, self._uniform_names(),
                              self.buffer_params[s.buffer], self.buffers.get(s.buffer))
        if plan is None or plan.inner != 1 or plan.rank not in (2, 3, 4):
            return False
        if any(c.kind not in ("scalar", "func") for c in coords):
            return False
        # the inner origin must be a multiple of 4 elements (16-byte TMA rule)
        coef, div = self._affine_last(s.coords[plan.col_axis])
        if coef != 1 or div % 4:
            return False
        size = plan.nbox * 128 * 128
        ring = self._store_ring
        if ring is not None and ring["size"] in (None, size) and ring["bytes"] // size >= 2:
            # rotating staging slots: this store waits only for the store that
            # used its slot before (one bulk group per store, in order)
            ring["size"] = size
            nslot = min(4, ring["bytes"] // size)
            slot = ring["next"] % nslot
            ring["next"] += 1
            base = ring["base"] + slot * size
        else:
            ring = None
            base = self._store_staging(size, allocate=False)
        boxes = None
        if base is None and (lay.groups == 1 or lay.cpg % 32 == 0) and len(self._box_slots(16384, 4)) >= 2:
            # freed operand buffers hold at least two boxes: stage through them
            # instead of a new allocation (less shared memory per CTA)
            boxes = self._box_slots(16384, 4)
        elif base is None:
            base = self._store_staging(size)
            if base is None:
                return False
        tm = self.tensor_map_param(plan)
        origin = self._tma_coords(plan, coords)
        if boxes is not None:
            return self._box_ring_store(s, shape, value, lay, plan, tm, origin, boxes)
        col0 = "(tid >> 7) * %d + " % lay.cpg if lay.groups > 1 else ""
        self.emit(f"{{ // TMA store of {s.buffer} ({shape[0]}x{shape[1]} f32) through shared memory")
        self.indent += 1
        if ring is not None:
            self.emit(f"if (tid == 0) tila::bulk_wait_read_n<{nslot - 1}>();   // staging slot {slot} is free")
            self.emit("__syncthreads();")
        self.emit("const int row_ = tid & 127;")
        self.emit("#pragma unroll")
        self.emit(f"for (int r = 0; r < {lay.nreg}; r += 4) {{")
        self.emit(f"  const int c_ = {col0}r;")
        self.emit(f"  *reinterpret_cast<float4*>(tila_smem + {base} + (c_ / 32) * 16384 + row_ * 128 + "
                  f"((((c_ % 32) / 4) ^ (row_ & 7)) * 16)) = "
                  f"make_float4({value.name}[r], {value.name}[r + 1], {value.name}[r + 2], {value.name}[r + 3]);")
        self.emit("}")
        self.emit("tila::fence_proxy_async_smem();")
        self.emit("__syncthreads();")
        self.emit("if (tid == 0) {")
        self.indent += 1
        for b in range(plan.nbox):
            cs = list(origin)
            if b:
                cs[0] = f"({cs[0]} + {32 * b})"
            self.emit(f"tila::tma_store_{plan.rank}d(&{tm}, tila_smem + {base} + {b * 16384}, {', '.join(cs)});")
        self.emit("tila::bulk_commit();")
        if ring is None:
            self.emit("tila::bulk_wait_read();")
        self.indent -= 1
        self.emit("}")
        if ring is None:
            self.emit("__syncthreads();")
        self.indent -= 1
        self.emit("}")
        return True

    def _box_slots(self, size, limit):
        """Up to ``limit`` slots of ``size`` bytes carved from freed regions."""
        slots = []
        for off, n in self._free_smem:
            o = (off + 1023) // 1024 * 1024
            while o + size <= off + n and len(slots) < limit:
                slots.append(o)
                o += size
        return slots

    def _box_ring_store(self, s, shape, value, lay, plan, tm, origin, slots):
        """TMA store staged one 32-column box at a time through a few freed
        16 KB slots: each box waits only for the store that last used its
        slot, so writing box b+1 overlaps the copy-out of box b."""
        k = len(slots)
        self.emit(f"{{ // TMA store of {s.buffer} ({shape[0]}x{shape[1]} f32) through {k} 16 KB staging slots")
        self.indent += 1
        self.emit("const int row_ = tid & 127;")
        for b in range(plan.nbox):
            slot = slots[b % k]
            if b >= k:
                self.emit(f"if (tid == 0) tila::bulk_wait_read_n<{k - 1}>();")
                self.emit("__syncthreads();")
            # the box's 32 columns belong to one thread group (lay.groups
            # groups of 128 threads hold lay.cpg columns of every row each)
            g, c0 = divmod(32 * b, lay.cpg) if lay.groups > 1 else (0, 32 * b)
            if lay.groups > 1:
                self.emit(f"if ((tid >> 7) == {g}) {{")
            self.emit("#pragma unroll")
            self.emit(f"for (int r = {c0}; r < {c0 + 32}; r += 4) {{")
            self.emit(f"  *reinterpret_cast<float4*>(tila_smem + {slot} + row_ * 128 + "
                      f"((((r % 32) / 4) ^ (row_ & 7)) * 16)) = "
                      f"make_float4({value.name}[r], {value.name}[r + 1], {value.name}[r + 2], {value.name}[r + 3]);")
            self.emit("}")
            if lay.groups > 1:
                self.emit("}")
            self.emit("tila::fence_proxy_async_smem();")
            self.emit("__syncthreads();")
            cs = list(origin)
            if b:
                cs[0] = f"({cs[0]} + {32 * b})"
            self.emit(f"if (tid == 0) {{ tila::tma_store_{plan.rank}d(&{tm}, tila_smem + {slot}, {', '.join(cs)}); "
                      f"tila::bulk_commit(); }}")
        self.emit("if (tid == 0) tila::bulk_wait_read();")
        self.emit("__syncthreads();")
        self.indent -= 1
        self.emit("}")
        return True

    def _store_staging(self, size, allocate=True):
        """Shared memory for a TMA store: a region freed by a finished
        pipelined loop when one is large enough, else (``allocate``) a new
        allocation (None when that would not fit)."""
        for off, n in self._free_smem:
            if n >= size:
                return off
        if not allocate or self.smem.top + size > 200 * 1024:
            return None
        return self.smem.alloc(size, 1024)

    # -- Ptr form (interp.py:357-384): a base pointer plus element offsets ------

    def e_TBufPtr(self, x):
        src = self.ptr_params.get(x.buffer) or self.buffer_params[x.buffer]
        return Val("ptr", src.vtype.elem, ptr=(x.buffer, None))

    def e_TPAdd(self, x):
        p = self.value(x.ptr)
        if p.kind != "ptr":
            self.fail("pointer arithmetic on a non-pointer value")
        off = self.coerce(self.value(x.offset), D.i64)
        name, cur = p.ptr
        if cur is not None:
            off = self.combine(D.i64, _broadcast_shapes([cur.shape, off.shape]), [cur, off],
                               lambda e: f"tila::wadd<tila::i64>({e[0]}, {e[1]})")
        return Val("ptr", p.dt, tuple(off.shape), ptr=(name, off))

    def _ptr_target(self, ptr_node):
        p = self.value(ptr_node)
        if p.kind != "ptr":
            self.fail("expected a pointer value")
        name, off = p.ptr
        if off is None:
            off = Val("scalar", D.i64, expr="0", const=0)
        return name, off

    def ptr_load(self, x, dt, shape):
        name, off = self._ptr_target(x.ptr)
        mask = self.value(x.mask) if x.mask is not None else None
        other = self.coerce(self.value(x.other), dt) if x.other is not None else None
        fill0 = DT.literal(dt, 0)
        if not shape:
            fill = other.expr if other is not None else fill0
            ld = DT.load_conv(dt, f"p_{name}[(tila::i64)({off.expr})]")
            v = self.fresh("pl")
            cond = f"({mask.expr})" if mask is not None else "true"
            self.emit(f"const {DT.ctype(dt)} {v} = {cond} ? {ld} : {fill};")
            return Val("scalar", dt, expr=v)
        layout = self.default_layout(shape, dt)
        ops = [off] + ([mask] if mask is not None else []) + ([other] if other is not None else [])
        ops, maps, straight = self.prepare_operands(ops, layout, shape)
        name_v = self.fresh("pl")
        self.emit(f"{DT.ctype(dt)} {name_v}[{layout.nreg}];")
        valid = layout.valid_expr()
        rng = range(layout.nreg) if straight else ["r"]
        if not straight:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
            self.indent += 1
        for r in rng:
            oe = self.elem(ops[0], layout, r, maps[0])
            conds = [f"({valid})"] if valid is not None else []
            if mask is not None:
                conds.append(f"({self.elem(ops[1], layout, r, maps[1])})")
            fill = self.elem(ops[-1], layout, r, maps[-1]) if other is not None else fill0
            ld = DT.load_conv(dt, f"p_{name}[(tila::i64)({oe})]")
            c = " && ".join(conds) if conds else "true"
            self.emit(f"{name_v}[{r}] = ({c}) ? {ld} : {fill};")
        if not straight:
            self.indent -= 1
            self.emit("}")
        return Val("reg", dt, tuple(shape), name=name_v, layout=layout)

    def ptr_store(self, s):
        name, off = self._ptr_target(s.ptr)
        dt = self.ptr_params[name].vtype.elem if name in self.ptr_params else \
            self.buffer_params[name].vtype.elem
        value = self.value(s.value)
        value = self.coerce(value, dt) if value.dt.name != dt.name else value
        mask = self.value(s.mask) if s.mask is not None else None
        shapes = [off.shape, value.shape] + ([mask.shape] if mask is not None else [])
        shape = _broadcast_shapes(shapes)
        if not shape:
            cond = "tid == 0" + (f" && ({mask.expr})" if mask is not None else "")
            self.emit(f"if ({cond}) p_{name}[(tila::i64)({off.expr})] = {DT.store_conv(dt, value.expr)};")
            return
        if value.kind == "tmem":
            value = self.tmem_to_reg(value)
        layout = value.layout if value.kind == "reg" and tuple(value.shape) == tuple(shape) \
            else self.default_layout(shape, dt)
        ops = [off, value] + ([mask] if mask is not None else [])
        ops, maps, straight = self.prepare_operands(ops, layout, shape)
        own = owner_predicate(layout)
        if own == "PER_SLOT":
            straight = True
        valid = layout.valid_expr()
        self.emit("{")
        self.indent += 1
        if own is not None and own != "PER_SLOT":
            self.emit(f"if ({own}) {{")
            self.indent += 1
        rng = range(layout.nreg) if straight else ["r"]
        if not straight:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
            self.indent += 1
        for r in rng:
            conds = [f"({valid})"] if valid is not None else []
            if own == "PER_SLOT":
                conds.append(self._owner_cond(layout, r))
            if mask is not None:
                conds.append(f"({self.elem(ops[2], layout, r, maps[2])})")
            oe = self.elem(ops[0], layout, r, maps[0])
            ve = DT.store_conv(dt, self.elem(ops[1], layout, r, maps[1]))
            c = f"if ({' && '.join(conds)}) " if conds else ""
            self.emit(f"{c}p_{name}[(tila::i64)({oe})] = {ve};")
        if not straight:
            self.indent -= 1
            self.emit("}")
        if own is not None and own != "PER_SLOT":
            self.indent -= 1
            self.emit("}")
        self.indent -= 1
        self.emit("}")

    # -- atomic_add (relaxed, GPU scope; interp.py:334-356) -------------------

    _ATOMIC_CT = {"i32": "int", "u32": "unsigned int", "f32": "float"}

    def e_TAtomicAdd(self, x):
        dt, shape, _ = self.vt_info(x.vt)
        if dt.name not in self._ATOMIC_CT:
            self.fail(f"atomic_add on {dt.name} is not supported (i32, u32, f32)", x.line)
        ct = self._ATOMIC_CT[dt.name]
        if x.buffer is not None:
            coords = [self.value(c) for c in x.coords]
            base = x.buffer
        else:
            base, off = self._ptr_target(x.ptr)
            coords = [off]
        value = self.coerce(self.value(x.value), dt)
        mask = self.value(x.mask) if x.mask is not None else None
        nc = len(coords)

        def addr(exprs):
            if x.buffer is not None:
                terms = [f"(tila::i64)p_{base}_stride{i} * (tila::i64)({e})" for i, e in enumerate(exprs)]
                return " + ".join(terms) or "0"
            return f"(tila::i64)({exprs[0]})"
        res = self.fresh("at")
        if not shape:
            # one thread performs the update; the old value is shared with all
            self.smem.need_scratch(8)
            cond = "tid == 0" + (f" && ({mask.expr})" if mask is not None else "")
            self.emit(f"{DT.ctype(dt)} {res} = {DT.literal(dt, 0)};")
            self.emit(f"if ({cond}) {res} = atomicAdd(reinterpret_cast<{ct}*>(p_{base} + "
                      f"({addr([c.expr for c in coords])})), ({ct})({value.expr}));")
            self.emit("__syncthreads();")
            self.emit(f"if (tid == 0) *reinterpret_cast<{DT.ctype(dt)}*>(tila_scratch) = {res};")
            self.emit("__syncthreads();")
            self.emit(f"{res} = *reinterpret_cast<{DT.ctype(dt)}*>(tila_scratch);")
            self.emit("__syncthreads();")
            return Val("scalar", dt, expr=res)
        layout = self.default_layout(shape, dt)
        ops = list(coords) + [value] + ([mask] if mask is not None else [])
        ops, maps, straight = self.prepare_operands(ops, layout, shape)
        own = owner_predicate(layout)
        if own == "PER_SLOT":
            straight = True
        valid = layout.valid_expr()
        self.emit(f"{DT.ctype(dt)} {res}[{layout.nreg}];")
        rng = range(layout.nreg) if straight else ["r"]
        if not straight:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
            self.indent += 1
        for r in rng:
            conds = [f"({valid})"] if valid is not None else []
            if own is not None:
                conds.append(self._owner_cond(layout, r) if own == "PER_SLOT" else f"({own})")
            if mask is not None:
                conds.append(f"({self.elem(ops[nc + 1], layout, r, maps[nc + 1])})")
            a = addr([self.elem(ops[i], layout, r, maps[i]) for i in range(nc)])
            v = self.elem(ops[nc], layout, r, maps[nc])
            c = " && ".join(conds) if conds else "true"
            self.emit(f"{res}[{r}] = ({c}) ? atomicAdd(reinterpret_cast<{ct}*>(p_{base} + ({a})), ({ct})({v})) "
                      f": {DT.literal(dt, 0)};")
        if not straight:
            self.indent -= 1
            self.emit("}")
        return Val("reg", dt, tuple(shape), name=res, layout=layout)

    # -- dot (tcgen05): see mma.MmaMixin -----------------------------------

    def _stage_operand(self, v: Val, off: int, K: int, transpose: bool):
        """Write an f16 operand into shared memory, K-major, no swizzle.
        A: element (m, k) -> row m; B (K x N): element (k, n) -> row n."""
        if v.kind == "tmem":
            v = self.tmem_to_reg(v)
        if v.kind == "scalar":
            self.fail("dot operand must be a tile")
        if v.kind == "func":
            v = self.materialize(v)
        lay = v.layout
        own = owner_predicate(lay)
        valid = lay.valid_expr()
        coords = lay.coord("r")
        if transpose:
            p, q = coords[1], coords[0]
        else:
            p, q = coords[0], coords[1]
        conv = (lambda e: f"tila::f2h({e})") if v.dt.name == "f16" else (lambda e: f"tila::f2h((float)({e}))")
        straight = isinstance(lay, Derived) and not lay.reg_affine() or own == "PER_SLOT"
        self.emit("__syncthreads();")
        if straight:
            for r in range(lay.nreg):
                c = lay.coord(r)
                pp, qq = (c[1], c[0]) if transpose else (c[0], c[1])
                cond = self._owner_cond(lay, r)
                pre = f"if ({cond}) " if cond else ""
                self.emit(f"{pre}*reinterpret_cast<tila::u16*>(tila_smem + {off} + tila::kmajor_offset({pp}, {qq}, {K})) = {conv(f'{v.name}[{r}]')};")
        else:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {lay.nreg}; ++r) {{")
            pre = f"if ({valid}) " if valid else ""
            self.emit(f"  {pre}*reinterpret_cast<tila::u16*>(tila_smem + {off} + tila::kmajor_offset({p}, {q}, {K})) = {conv(f'{v.name}[r]')};")
            self.emit("}")

    # -- statements ------------------------------------------------------------

    def stmts(self, body):
        for s in body:
            self.stmt(s)

    def stmt(self, s):
        m = getattr(self, f"s_{type(s).__name__}", None)
        if m is None:
            self.fail(f"unsupported TIR statement {type(s).__name__}", getattr(s, "line", 0))
        line = getattr(s, "line", 0)
        if self.source_map and line:
            # source map: the generated code below comes from this Tila line
            self.emit(f"// @tila-line {line}")
        m(s)
        if self.actx is not None:
            self.emit_early_p(s)

    def s_TAssign(self, s):
        v = None
        actx = self.actx
        if actx is not None and s.name in actx.loads:
            v = self.load_smem_val(actx, s.name)
            v.smem_name = s.name
            self.env[s.name] = v
            return
        if actx is not None and s.name in actx.accs:
            if s.value is actx.accs[s.name]["dot"]:
                self.env[s.name] = self.emit_async_acc_dot(s.value, s.name)
                return
            if self.tmem_update_in_place(s.name, s.value):
                return
        if isinstance(s.value, T_.TLoad):
            v = self.try_tma_load(s.value, assigned_name=s.name)
            if v is not None:
                v.smem_name = s.name
        if v is None:
            v = self.value(s.value)
        if v.kind == "scalar" and v.const is None and not _is_simple(v.expr):
            name = self.fresh(f"s_{s.name}")
            self.emit(f"const {DT.ctype(v.dt)} {name} = {v.expr};")
            v = Val("scalar", v.dt, expr=name)
        if v.kind == "tmem":
            v = self.tmem_to_reg(v)
        self.env[s.name] = v
        if isinstance(s.value, T_.TPid):
            self._pidnames.add(s.name)
        self._defs[s.name] = s.value

    def s_TAssume(self, s):
        """ti.assume: a proof fact, free in normal builds.  With TILA_DEBUG=1
        (lowering.py:339-342 emits tl.device_assert there) every thread
        checks its lanes of the predicate; a false lane records the Tila line
        in the launch's error word, and the whole program then stops before
        the accesses the assumption was meant to justify (the host raises).
        Inside a pipelined loop the check only records."""
        if not self.debug:
            return
        v = self.value(s.pred)
        line = int(getattr(s, "line", 0) or 0)
        flag = self.fresh("af")
        if v.kind == "scalar":
            self.emit(f"const bool {flag} = !({v.expr});")
        else:
            if v.kind != "reg":
                v = self.materialize(v)
            lay = v.layout
            valid = lay.valid_expr()
            self.emit(f"bool {flag} = false;")
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {lay.nreg}; ++r) "
                      f"if ({'(' + valid + ') && ' if valid else ''}!({v.name}[r])) {flag} = true;")
        self.emit(f"if ({flag}) tila::report_error(tila_err, tila::kErrAssumption, {line}u);")
        if self.actx is None:
            self.emit(f"if (__syncthreads_or({flag})) goto tila_program_end;")
            self._assume_stop = True
        self._assume_lines.append(line)

    def s_TAtomicStmt(self, s):
        self.e_TAtomicAdd(s.value)

    def s_TReturn(self, s):
        self.emit("break;  // return: leave the program body")

    def s_TStaticIf(self, s):
        c = self._static_cond(s.cond)
        self.stmts(s.then_body if c else s.else_body)

    def _static_cond(self, node):
        ev = tila.runtime._eval_const_operand
        try:
            return bool(ev(node, self.consts))
        except Exception:
            v = self.value(node)
            if v.const is None:
                self.fail("static if condition is not a compile-time constant", getattr(node, "line", 0))
            return bool(v.const)

    def s_TIf(self, s):
        c = self.value(s.cond)
        if c.kind != "scalar":
            self.fail("runtime if needs a scalar condition", s.line)
        if c.const is not None:
            self.stmts(s.then_body if c.const else s.else_body)
            return
        assigned = _stmt_names_assigned(s.then_body) | _stmt_names_assigned(s.else_body)
        merged = [n for n in assigned if n in self.env]
        ends = []
        for body in (s.then_body, s.else_body):
            snap = self._snapshot()
            self.stmts(body)
            ends.append({n: self.env[n] for n in merged})
            self._restore(snap)
        storage = self._declare_merged(merged, [ends[0], ends[1]])
        self.emit(f"if ({c.expr}) {{")
        for body in (s.then_body, s.else_body):
            self.indent += 1
            saved_env = dict(self.env)
            self.stmts(body)
            self._assign_merged(storage)
            self.env = saved_env
            self.indent -= 1
            if body is s.then_body:
                self.emit("} else {")
        self.emit("}")
        for n, st in storage.items():
            self.env[n] = st

    def s_TFor(self, s):
        start = self.value(s.start) if s.start is not None else Val("scalar", D.i64, expr="0", const=0)
        end = self.value(s.end)
        step = self.value(s.step)
        if step.const is None:
            # the checker admits only compile-time steps >= 1 (TILA-TYPE-025)
            self.fail("loop step must be a compile-time constant", s.line)
        stepv = int(step.const)
        if stepv == 0:
            self.fail("loop step is zero", s.line)
        assigned = _stmt_names_assigned(s.body)
        carried = sorted(n for n in assigned if n in self.env and n != s.var)
        # names first assigned inside the body are local to it (their C++
        # variables live in the loop's scope): unbound after the loop
        local = [n for n in assigned if n not in self.env and n != s.var]
        # the loop variable's divisibility (for vector alignment proofs)
        sdiv = _pow2_div(int(start.const)) if start.const is not None else 1
        self._loopvars[s.var] = min(sdiv, _pow2_div(abs(stepv)))
        self.pdefs.scopes.append(self.pdefs.loop_locals(s.body))
        try:
            self._emit_for(s, start, end, stepv, carried)
        finally:
            self.pdefs.scopes.pop()
        self.env.pop(s.var, None)
        for n in local:
            self.env.pop(n, None)

    def _emit_for(self, s, start, end, stepv, carried):
        if self.try_contraction_loop(s, start, end, stepv, carried):
            return
        actx = None
        if self.actx is None:
            actx = self.try_async_loop_setup(s, start, end, stepv, carried)
            if actx is not None:
                carried = [n for n in carried if n not in actx.accs]
        loop_end_vals = None
        # two dry runs reach the fixpoint of the carried layouts
        pre = {n: self.env[n] for n in carried}
        bound = dict(pre)
        for _ in range(2):
            snap = self._snapshot()
            for n, v in bound.items():
                self.env[n] = v
            self.env[s.var] = Val("scalar", D.i32, expr="LOOPVAR")
            self.indent += 1
            self.stmts(s.body)
            self.indent -= 1
            loop_end_vals = {n: self.env[n] for n in carried}
            self._restore(snap)
            bound = {}
            for n in carried:
                bound[n] = self._carried_val(pre[n], loop_end_vals[n], n, dry=True)
        storage = self._declare_carried(carried, pre, loop_end_vals)
        iv = self.fresh("it")
        cmp = "<" if stepv > 0 else ">"
        self.emit(f"for (tila::i64 {iv} = (tila::i64)({start.expr}); {iv} {cmp} (tila::i64)({end.expr}); {iv} += {stepv}) {{")
        self.indent += 1
        lv = self.fresh(f"s_{s.var}")
        self.emit(f"const tila::i32 {lv} = (tila::i32){iv};")
        for n, st in storage.items():
            self.env[n] = st
        self.env[s.var] = Val("scalar", D.i32, expr=lv)
        if actx is not None:
            self._emit_versioned_body(s.body, storage)
        else:
            self.stmts(s.body)
            self._assign_merged(storage)
        self.indent -= 1
        self.emit("}")
        for n, st in storage.items():
            self.env[n] = st
        if actx is not None:
            self.finish_async_loop(actx)

    # -- loop-body versioning on tile bound checks ---------------------------------

    def _emit_versioned_body(self, body, storage):
        """Emit the loop body twice: a general version and one in which every
        bound comparison ``uniform + arange < uniform`` of the body is known
        to hold on the whole tile, selected by one uniform guard per
        iteration (interior tiles skip their mask arithmetic)."""
        if not self.versioning:
            self.stmts(body)
            self._assign_merged(storage)
            return
        env0, cc0 = dict(self.env), dict(self.conv_cache)
        outer = self.lines
        self.lines = []
        self._guard_mode, self._guards = "collect", []
        self.stmts(body)
        self._assign_merged(storage)
        general = self.lines
        guards = list(dict.fromkeys(self._guards))
        if not guards:
            self._guard_mode = None
            self.lines = outer + general
            return
        self.env, self.conv_cache = dict(env0), dict(cc0)
        self.lines = []
        self._guard_mode, self._guard_set = "fast", set(guards)
        self.stmts(body)
        self._assign_merged(storage)
        fast = self.lines
        self._guard_mode = None
        self.lines = outer
        self.env, self.conv_cache = env0, cc0
        self.emit(f"if ({' && '.join(guards)}) {{  // every tile bound check holds")
        self.lines.extend(fast)
        self.emit("} else {")
        self.lines.extend(general)
        self.emit("}")

    def _interval_mask(self, node, depth=0):
        """True when the lanes of any run of consecutive elements along the
        last tile dim on which mask ``node`` holds are themselves consecutive
        (a conjunction of bounds on coordinates that step by 0 or +1 along
        that dim).  Then a vector group is fully inside iff its first and last
        lanes are."""
        from .pipeline import tile_affinity
        if node is None or depth > 16:
            return False
        node = self.pdefs.resolve(node)
        if isinstance(node, T_.TLit):
            return True
        if isinstance(node, T_.TBin):
            if node.op in ("&", "and"):
                return (self._interval_mask(node.left, depth + 1)
                        and self._interval_mask(node.right, depth + 1))
            if node.op in ("<", "<=", ">", ">=", "=="):
                uni = self._uniform_names()
                la = tile_affinity(node.left, self.pdefs, self.consts, uni)
                ra = tile_affinity(node.right, self.pdefs, self.consts, uni)
                if la is None or ra is None:
                    return False
                if la == () and ra == ():
                    return True
                var = la if ra == () else ra if la == () else None
                return var is not None and var[-1] in (0, 1)
            return False
        if isinstance(node, T_.TExpand):
            if node.axis == 1:           # m[:, None]: constant along the last dim
                return True
            return self._interval_mask(node.operand, depth + 1)
        return False

    def _bound_guard(self, x, l, r, op, shape):
        """Uniform condition under which ``l op r`` is true on the whole tile
        (l = uniform + arange along one dim, r uniform), or None."""
        from .pipeline import tile_affinity
        uni = self._uniform_names()
        if tile_affinity(x.right, self.pdefs, self.consts, uni) != ():
            return None
        aff = tile_affinity(x.left, self.pdefs, self.consts, uni)
        if aff is None or sorted(aff) != sorted((1,) + (0,) * (len(aff) - 1)):
            return None
        dim = aff.index(1)
        if len(l.shape) != len(aff) or l.kind != "func":
            return None
        extent = l.shape[dim]
        base = l.fn(("0",) * len(l.shape))
        return f"((tila::i64)({base}) + {extent - 1} {op} (tila::i64)({r.expr}))"

    # -- merge points (loops and runtime ifs) ------------------------------------

    def _snapshot(self):
        return (list(self.lines), dict(self.env), self.counter, self.smem.top, self.smem.scratch,
                self.tmem_cols, dict(self.conv_cache), dict(self._defs), set(self._pidnames),
                dict(self._loopvars), self.uses_tmem, self.uses_mma, self.indent, self.smem.red)

    def _restore(self, snap):
        (self.lines, self.env, _, self.smem.top, self.smem.scratch, self.tmem_cols, self.conv_cache,
         self._defs, self._pidnames, self._loopvars, self.uses_tmem, self.uses_mma, self.indent,
         self.smem.red) = snap
        # keep the counter monotonic so names never collide

    def _carried_val(self, pre, end, name, dry=False):
        """Representation of a carried variable inside the loop."""
        if not pre.shape and not end.shape:
            return Val("scalar", end.dt, expr=f"c_{name}")
        shape = end.shape or pre.shape
        dt = end.dt
        if end.kind == "reg":
            lay = end.layout
        elif pre.kind == "reg":
            lay = pre.layout
        else:
            lay = self.default_layout(shape, dt)
        if isinstance(lay, Derived) and not lay.reg_affine():
            lay = self.default_layout(shape, dt)
        return Val("reg", dt, tuple(shape), name=f"c_{name}", layout=lay)

    def _declare_carried(self, carried, pre, end):
        storage = {}
        for n in carried:
            proto = self._carried_val(pre[n], end[n], n)
            var = self.fresh(f"c_{n}")
            if not proto.shape:
                dt = proto.dt
                src = self.coerce(pre[n], dt) if pre[n].dt.name != dt.name else pre[n]
                self.emit(f"{DT.ctype(dt)} {var} = {src.expr};")
                storage[n] = Val("scalar", dt, expr=var)
            else:
                lay = proto.layout
                src = pre[n]
                if src.kind == "tmem":
                    src = self.tmem_to_reg(src)
                if src.dt.name != proto.dt.name:
                    src = self.coerce(src, proto.dt)
                self.emit(f"{DT.ctype(proto.dt)} {var}[{lay.nreg}];")
                ops, maps, straight = self.prepare_operands([src], lay, proto.shape)
                self._copy_into(var, lay, ops[0], maps[0], straight)
                storage[n] = Val("reg", proto.dt, proto.shape, name=var, layout=lay)
        return storage

    def _declare_merged(self, names, ends):
        storage = {}
        for n in names:
            a, b = ends[0][n], ends[1][n]
            cur = self.env[n]
            proto = self._carried_val(cur, a if a.kind == "reg" else b, n)
            var = self.fresh(f"m_{n}")
            if not proto.shape:
                self.emit(f"{DT.ctype(proto.dt)} {var} = {self.coerce(cur, proto.dt).expr};")
                storage[n] = Val("scalar", proto.dt, expr=var)
            else:
                lay = proto.layout
                self.emit(f"{DT.ctype(proto.dt)} {var}[{lay.nreg}];")
                src = cur if cur.kind != "tmem" else self.tmem_to_reg(cur)
                ops, maps, straight = self.prepare_operands([self.coerce(src, proto.dt)], lay, proto.shape)
                self._copy_into(var, lay, ops[0], maps[0], straight)
                storage[n] = Val("reg", proto.dt, proto.shape, name=var, layout=lay)
        return storage

    def _assign_merged(self, storage):
        for n, st in storage.items():
            cur = self.env[n]
            if cur.kind == st.kind and cur.name == st.name and cur.expr == st.expr:
                continue
            if not st.shape:
                src = self.coerce(cur, st.dt) if cur.dt.name != st.dt.name else cur
                self.emit(f"{st.expr} = {src.expr};")
                continue
            if cur.kind == "tmem":
                cur = self.tmem_to_reg(cur)
            if cur.dt.name != st.dt.name:
                cur = self.coerce(cur, st.dt)
            ops, maps, straight = self.prepare_operands([cur], st.layout, st.shape)
            self._copy_into(st.name, st.layout, ops[0], maps[0], straight)

    def _copy_into(self, var, lay, src, smap, straight):
        if straight or (isinstance(lay, Derived) and not lay.reg_affine()):
            for r in range(lay.nreg):
                self.emit(f"{var}[{r}] = {self.elem(src, lay, r, smap)};")
        else:
            self.emit("#pragma unroll")
            self.emit(f"for (int r = 0; r < {lay.nreg}; ++r) {var}[r] = {self.elem(src, lay, 'r')};")

    # -- kernel ----------------------------------------------------------------

    def generate(self) -> KernelSpec:
        self._defs = {}
        self._pidnames = set()
        self._loopvars = {}
        self._need_barrier_init = []
        self._phase_vars = []
        self.tmem_scratch_need = 0
        self._init_mma()
        if self._small_program():
            self.T = 64
        tk = self.tk
        params = []
        sig = []
        for b in tk.buffers:
            dt = b.vtype.elem
            const = "const " if b.vtype.access is TY.READ_ONLY else ""
            sig.append(f"{const}{DT.memtype(dt)}* __restrict__ p_{b.name}" if b.vtype.access is TY.READ_ONLY
                       else f"{DT.memtype(dt)}* p_{b.name}")
            params.append(("buffer", b.name, "ptr"))
        for p in tk.ptr_params:
            dt = p.vtype.elem
            sig.append(f"{DT.memtype(dt)}* p_{p.name}")
            params.append(("ptr", p.name, "ptr"))
        for s in tk.scalars:
            sig.append(f"{DT.memtype(s.dtype)} p_{s.name}")
            params.append(("scalar", s.name, s.dtype.name))
        # strides appear as scalars already (x_stride0 ...): also accessible as p_<buf>_stride<i>
        for ax in range(3):
            sig.append(f"tila::i32 nprog_{ax}")
            params.append(("nprog", ax, "i32"))
        for ax in range(3):
            sig.append(f"tila::i32 pid_off_{ax}")
            params.append(("pid_off", ax, "i32"))
        sig.append("tila::u32* __restrict__ tila_err")
        params.append(("err", None, "ptr"))
        self.lines = []
        self.indent = 2
        if not self.try_fused_kernel():
            self.stmts(tk.body)
        body = self.lines
        # shared-memory plan and tensor-memory columns of one program
        scratch_off = (self.smem.top + 127) // 128 * 128
        scratch_col = self.tmem_next
        total_cols = self.tmem_next + self.tmem_scratch_need
        if self.uses_tmem:
            if total_cols > 512:
                self.fail(f"kernel needs {total_cols} tensor-memory columns (limit 512)")
            self.tmem_cols = _pow2_at_least(max(32, total_cols))
        # cross-warp reductions alternate between two halves of their own
        # region (tila_rsel): the barrier after a reduction's writes also
        # orders the previous reduction's reads before the next writes there
        red_off = scratch_off + (self.smem.scratch + 127) // 128 * 128
        prog_bytes = red_off + 2 * self.smem.red
        per_prog = -(-prog_bytes // 1024) * 1024
        # two programs of axis 0 per CTA, one per warpgroup (see _pingpong_ok)
        wg = (self._wg_candidate and not self.fuse and self.T == 128 and self.uses_tmem
              and self.tmem_cols <= 256 and 2 * per_prog + 64 <= 232448 and self._uneven_loops <= 3
              and not self._assume_lines)
        # the warp-specialised form also takes programs of 8 warps (one per
        # pair of warpgroups), which the two-program hand-off does not
        found = self.ws_ready() if self._ws is None else None
        ws_fit = (found is not None and not self.fuse and self.T in (128, 256)
                  and self.uses_tmem and self.tmem_cols <= 256 and not self._assume_lines)
        if ws_fit and os.environ.get("TILA_B200_WS", "1") != "0":
            # the loops have the flash-attention shape: generate the
            # warp-specialised kernel instead (this pass's plan is the fallback)
            # (always 4-warp programs: the thread layout is the backend's
            # choice and does not change results; see wspec.ws_budget)
            try:
                return KernelEmitter(self.tk, self.consts, self.buffers, num_warps=4,
                                     entry_name=self.entry, debug=self.debug,
                                     versioning=self.versioning, source_map=self.source_map,
                                     ws=found).generate()
            except CodegenError:
                pass
        if self._ws is not None:
            if not (self.T == 128 and self.uses_tmem and self.tmem_cols <= 256 and not self.fuse):
                self.fail("warp-specialised loop: two programs per CTA do not fit")
            wg = True
        if wg:
            self.fuse = {0: 2}
        for ax in sorted(self.fuse or {}):
            sig.append(f"tila::i32 launch_{ax}")
            params.append(("launch", ax, "i32"))
        if self.persistent:
            # workspace and flags of the split tiles (one slot per CTA)
            sig.append("float* __restrict__ tila_sk_ws")
            params.append(("skws", None, "ptr"))
            sig.append("tila::u32* __restrict__ tila_sk_flags")
            params.append(("skflags", None, "ptr"))
        for tm in self.tensor_maps:
            sig.append(f"const __grid_constant__ tila::TensorMap {tm['param']}")
            params.append(("tensormap", tm["param"], tm))
        threads = 2 * self.T if wg else self.T
        cta_cols = 2 * self.tmem_cols if wg else self.tmem_cols
        if self._ws is not None:
            return self._ws_generate(sig, params, per_prog, body, scratch_off, red_off, scratch_col,
                                     cta_cols)
        out = ['#include "tila_tile.cuh"', ""]
        # f32 exp2: tensor-core kernels (compared within a tolerance, compiled
        # with multiply-add contraction) use the flush-to-zero form, which
        # returns 0 instead of a subnormal below 2^-126 and the same values
        # elsewhere; all other kernels keep subnormal results.
        out.append("#define tila_exp2_f32 tila::" + ("exp2_ftz" if self.uses_mma else "exp2_fast"))
        out.append("")
        out.append(f'extern "C" __global__ void __launch_bounds__({threads}) {self.entry}(')
        out.append(",\n".join("    " + x for x in sig) + ") {")
        if wg:
            out.append("  extern __shared__ __align__(1024) unsigned char tila_smem_all[];")
            out.append("  // two programs of grid axis 0 per CTA: warpgroup w runs program 2*blockIdx.x + w")
            out.append("  const int tila_wg = threadIdx.x >> 7;")
            out.append("  const int tid = threadIdx.x & 127;")
            out.append(f"  unsigned char* const tila_smem = tila_smem_all + tila_wg * {per_prog};")
            out.append("  const tila::i32 pid_0 = (tila::i32)(blockIdx.x * 2 + tila_wg + pid_off_0);")
            out.append("  const bool tila_live = (tila::i32)(blockIdx.x * 2 + tila_wg) < launch_0;")
            out.append("  const bool tila_partner_live = (tila::i32)(blockIdx.x * 2 + (tila_wg ^ 1)) < launch_0;")
            out.append(f"  tila::u64* const tila_tok = reinterpret_cast<tila::u64*>(tila_smem_all + {2 * per_prog});")
            out.append(f"  volatile tila::i64* const tila_trips = reinterpret_cast<volatile tila::i64*>(tila_smem_all + {2 * per_prog + 16});")
            out.append("  (void)tila_trips;")
            out.append("  tila::u32 tila_tok_ph = 0, tila_tok_n = 0;")
            out.append("  (void)tila_partner_live; (void)tila_tok; (void)tila_tok_ph; (void)tila_tok_n;")
        else:
            out.append("  extern __shared__ __align__(1024) unsigned char tila_smem[];")
            out.append("  const int tid = threadIdx.x;")
            out.append("  const tila::i32 pid_0 = (tila::i32)(blockIdx.x + pid_off_0);")
        out.append("  const tila::i32 pid_1 = (tila::i32)(blockIdx.y + pid_off_1);")
        out.append("  const tila::i32 pid_2 = (tila::i32)(blockIdx.z + pid_off_2);")
        if self.uses_mma:
            # shared-memory matrix descriptors are built from this base (tila::sdesc)
            out.append("  const tila::u32 tila_sb4 = tila::smem_u32(tila_smem) >> 4;")
        # fixed shared-memory head: mbarrier, tmem slot, dead flag; scratch follows the plan
        out.append(f"  tila::u64* tila_mma_bar = reinterpret_cast<tila::u64*>(tila_smem);")
        out.append(f"  tila::u32* tila_tmem_slot = reinterpret_cast<tila::u32*>(tila_smem + 8);")
        out.append(f"  volatile int& tila_dead = *reinterpret_cast<volatile int*>(tila_smem + 12);")
        out.append(f"  unsigned char* tila_scratch = tila_smem + {scratch_off};")
        out.append("  (void)tila_scratch; (void)tila_mma_bar; (void)tila_tmem_slot;")
        if self.smem.red:
            out.append(f"  unsigned char* const tila_red = tila_smem + {red_off};")
            out.append(f"  constexpr tila::u32 tila_red_half = {self.smem.red};")
            out.append("  tila::u32 tila_rsel = 0;")
        out.append("  tila::u32 tila_mma_phase = 0; (void)tila_mma_phase;")
        for v in self._phase_vars:
            out.append(f"  tila::u32 {v} = 0;")
        if self.uses_tmem or self._need_barrier_init:
            inits = " ".join(f"tila::mbar_init(reinterpret_cast<tila::u64*>(tila_smem + {o}), 1);"
                             for o in self._need_barrier_init)
            out.append(f"  if (tid == 0) {{ tila::mbar_init(tila_mma_bar, 1); {inits} tila::mbar_fence_init(); tila_dead = 0; }}")
            for tm in self.tensor_maps:
                out.append(f"  if (tid == 0) tila::tma_prefetch_desc(&{tm['param']});")
        if wg:
            out.append("  if (threadIdx.x == 0) { tila::mbar_init(&tila_tok[0], 128); "
                       "tila::mbar_init(&tila_tok[1], 128); tila::mbar_fence_init(); }")
        # everything above touches only shared memory and kernel parameters;
        # global memory (and tensor memory) only after the previous grid ends,
        # except for L2 prefetch hints of the program's first loads
        if self._prefetch:
            # only programs that exist (two-program CTAs may hold one past the grid)
            out.append("  if (tila_live) {" if wg else "  {")
            for code in self._prefetch:
                out.extend("    " + ln for ln in code.split("\n"))
            out.append("  }")
        out.append("  tila::grid_dep_wait();")
        out.append("  tila::grid_dep_release();")
        if self.uses_tmem:
            out.append(f"  if (threadIdx.x < 32) tila::tmem_alloc("
                       + ("reinterpret_cast<tila::u32*>(tila_smem_all + 8)" if wg else "tila_tmem_slot")
                       + f", {cta_cols});")
            out.append("  tila::tc_fence_before();")
            out.append("  __syncthreads();")
            out.append("  tila::tc_fence_after();")
            if wg:
                out.append(f"  const tila::u32 tila_tmem = *reinterpret_cast<tila::u32*>(tila_smem_all + 8) "
                           f"+ (tila::u32)(tila_wg * {self.tmem_cols});")
            else:
                out.append("  const tila::u32 tila_tmem = *tila_tmem_slot;")
            out.append(f"  const tila::u32 tila_tmem_scratch_col = {scratch_col}; (void)tila_tmem_scratch_col;")
        elif self._need_barrier_init:
            out.append("  __syncthreads();")
        out.append("  do {")
        if wg:
            from .mma import WG_ACQUIRE, WG_RELEASE, WG_TRIPS, WG_TURNS
            acquire = ("if (tila_partner_live && (tila_wg == 1 || tila_tok_n > 0)) { "
                       "tila::mbar_wait(&tila_tok[tila_wg], tila_tok_ph, tila_err, __LINE__, &tila_dead); "
                       "tila_tok_ph ^= 1u; } ++tila_tok_n;")
            release = "if (tila_partner_live) tila::mbar_arrive(&tila_tok[tila_wg ^ 1]);"
            out.append("    if (!tila_live) break;")
            for line in body:
                st = line.strip()
                ind = line[:len(line) - len(line.lstrip())]
                if st.startswith(WG_TRIPS):
                    # both programs reach this point (no early exits); a CTA-wide
                    # barrier orders the exchange (the partner is live, so both run)
                    k = int(st.split()[-1])
                    out.append(f"{ind}tila::i64 tila_ptrip_{k} = 0;")
                    out.append(f"{ind}if (tila_partner_live) {{")
                    out.append(f"{ind}  if (tid == 0) tila_trips[{2 * k} + tila_wg] = tila_trip_{k};")
                    out.append(f"{ind}  tila::cta_sync();")
                    out.append(f"{ind}  tila_ptrip_{k} = tila_trips[{2 * k} + (tila_wg ^ 1)];")
                    out.append(f"{ind}}}")
                    continue
                if st.startswith(WG_TURNS):
                    k = int(st.split()[-1])
                    out.append(f"{ind}for (tila::i64 t_ = tila_trip_{k}; t_ < tila_ptrip_{k}; ++t_) {{ {acquire} {release} }}")
                    continue
                line = line.replace("__syncthreads();", "tila::wg_sync(tila_wg);")
                line = line.replace(WG_ACQUIRE, acquire).replace(WG_RELEASE, release)
                out.append(line)
        else:
            from .mma import WG_ACQUIRE, WG_RELEASE, WG_TRIPS, WG_TURNS
            out.extend(l for l in body if l.strip() not in (WG_ACQUIRE, WG_RELEASE)
                       and not l.strip().startswith((WG_TRIPS, WG_TURNS)))
        out.append("  } while (0);")
        if self._assume_stop:
            out.append("  tila_program_end: ;")
        if self.uses_tmem:
            out.append("  tila::tc_fence_before();")
            out.append("  __syncthreads();")
            out.append(f"  if (threadIdx.x < 32) tila::tmem_dealloc(tila_tmem, {cta_cols});")
        out.append("}")
        src = "\n".join(out) + "\n"
        smem = 2 * per_prog + 64 if wg else prog_bytes
        if self.uses_tmem:
            # keep (resident CTAs) x (TMEM columns) within the SM's 512 columns
            max_ctas = max(1, 512 // cta_cols)
            floor_bytes = 233472 // (max_ctas + 1) - 1024 + 1
            smem = max(smem, floor_bytes)
        self.tmem_cols = cta_cols
        return KernelSpec(self.entry, src, threads, smem, params, fp_contract=self.uses_mma or self._contracted,
                          assume_lines=list(self._assume_lines),
                          tmem_cols=self.tmem_cols,
                          tensor_maps=list(self.tensor_maps), fuse=dict(self.fuse or {}),
                          persistent=self.persistent)


def _ws_generate_impl(self, sig, params, per_prog, body, scratch_off, red_off, scratch_col, cta_cols):
    """Kernel text of the warp-specialised two-program kernel (wspec.py):
    warpgroups 0 and 1 run the consumer body of programs 2 * blockIdx.x + w,
    thread 256 the producer."""
    from .mma import WG_ACQUIRE, WG_RELEASE, WG_TRIPS, WG_TURNS
    from .wspec import RING
    T = self.T
    threads, launch_regs, regs_producer, regs_consumer = ws_budget(T)
    ring_off = -(-(2 * per_prog) // 1024) * 1024
    kp, vp = self._ws["k"], self._ws["v"]
    ring_bytes = RING * sum(c["plan"].nbox * max(c["plan"].outer_extent, 128) * 128 for c in (kp, vp))
    bars_off = ring_off + ring_bytes
    prod, nbars, _ = self.ws_producer(per_prog, ring_off, bars_off, scratch_col)
    dead_off = bars_off + 8 * nbars
    total = dead_off + 16
    if total > 232448:
        self.fail(f"warp-specialised kernel needs {total} bytes of shared memory")
    out = ['#include "tila_tile.cuh"', "",
           "#define tila_exp2_f32 tila::" + ("exp2_ftz" if self.uses_mma else "exp2_fast"), "",
           f'extern "C" __global__ void __launch_bounds__({threads}, 1) {self.entry}(',
           ",\n".join("    " + x for x in sig) + ") {"]
    e = out.append
    e("  extern __shared__ __align__(1024) unsigned char tila_smem_all[];")
    e("  // warpgroups 0 and 1: programs 2*blockIdx.x + w (softmax side); warpgroup 2: thread 256 copies, thread 288 issues the MMAs")
    e(f"  const bool tila_producer = threadIdx.x >= {2 * T};")
    e(f"  const int tila_wg = tila_producer ? 0 : (int)(threadIdx.x / {T});")
    e(f"  const int tid = threadIdx.x & {T - 1};")
    e(f"  unsigned char* const tila_smem = tila_smem_all + tila_wg * {per_prog};")
    e("  const tila::i32 pid_0 = (tila::i32)(blockIdx.x * 2 + tila_wg + pid_off_0);")
    e("  const bool tila_live = !tila_producer && (tila::i32)(blockIdx.x * 2 + tila_wg) < launch_0;")
    e("  const tila::i32 pid_1 = (tila::i32)(blockIdx.y + pid_off_1);")
    e("  const tila::i32 pid_2 = (tila::i32)(blockIdx.z + pid_off_2);")
    e("  (void)pid_0; (void)pid_1; (void)pid_2;")
    e("  const tila::u32 tila_sb4 = tila::smem_u32(tila_smem) >> 4; (void)tila_sb4;")
    e("  tila::u64* tila_mma_bar = reinterpret_cast<tila::u64*>(tila_smem);")
    e("  tila::u32* tila_tmem_slot = reinterpret_cast<tila::u32*>(tila_smem_all + 8);")
    e(f"  volatile int& tila_dead = *reinterpret_cast<volatile int*>(tila_smem_all + {dead_off});")
    e(f"  unsigned char* tila_scratch = tila_smem + {scratch_off};")
    e("  (void)tila_scratch; (void)tila_mma_bar; (void)tila_tmem_slot;")
    if self.smem.red:
        e(f"  unsigned char* const tila_red = tila_smem + {red_off};")
        e(f"  constexpr tila::u32 tila_red_half = {self.smem.red};")
        e("  tila::u32 tila_rsel = 0;")
    e("  tila::u32 tila_mma_phase = 0; (void)tila_mma_phase;")
    for v in self._phase_vars:
        e(f"  tila::u32 {v} = 0;")
    q = self._ws["q_load"]
    per_region = [(0, 1), (q["bar_off"], 1), (self._ws["acc_bar"], 1), (self._ws["p_full"], T)]
    per_region += [(o, 1) for o in self._need_barrier_init]
    inits = " ".join(f"tila::mbar_init(reinterpret_cast<tila::u64*>(tila_smem_all + {w * per_prog + o}), {c});"
                     for w in range(2) for o, c in per_region)
    inits += " " + " ".join(f"tila::mbar_init(reinterpret_cast<tila::u64*>(tila_smem_all + {bars_off + 8 * i}), 1);"
                            for i in range(nbars))
    e(f"  if (threadIdx.x == 0) {{ {inits} tila::mbar_fence_init(); tila_dead = 0; }}")
    for tm in self.tensor_maps:
        e(f"  if (threadIdx.x == 0) tila::tma_prefetch_desc(&{tm['param']});")
    if self._prefetch:
        e("  if (tila_live) {")
        for code in self._prefetch:
            out.extend("    " + ln for ln in code.split("\n"))
        e("  }")
    e("  tila::grid_dep_wait();")
    e("  tila::grid_dep_release();")
    e(f"  if (threadIdx.x < 32) tila::tmem_alloc(tila_tmem_slot, {cta_cols});")
    e("  tila::tc_fence_before();")
    e("  __syncthreads();")
    e("  tila::tc_fence_after();")
    e(f"  const tila::u32 tila_tmem = *tila_tmem_slot + (tila::u32)(tila_wg * {self.tmem_cols});")
    e(f"  const tila::u32 tila_tmem_scratch_col = {scratch_col}; (void)tila_tmem_scratch_col;")
    e("  if (tila_producer) {")
    e(f"    tila::reg_dealloc<{regs_producer}>();")
    copy_lines, mma_lines = prod
    e(f"    if (threadIdx.x == {2 * T}) {{")
    out.extend("  " + ln for ln in copy_lines)
    e(f"    }} else if (threadIdx.x == {2 * T + 32}) {{")
    e("    const tila::u32 tila_tmem_base = *tila_tmem_slot;")
    out.extend("  " + ln for ln in mma_lines)
    e("    }")
    e("    __syncwarp();   // each producer warp reconverges before the final barrier")
    e("  } else {")
    e(f"  tila::reg_alloc<{regs_consumer}>();")
    e("  do {")
    e("    if (!tila_live) break;")
    for line in body:
        st = line.strip()
        if st in (WG_ACQUIRE, WG_RELEASE) or st.startswith((WG_TRIPS, WG_TURNS)):
            continue
        out.append(line.replace("__syncthreads();", f"tila::wg_sync_n(tila_wg, {T});"))
    e("  } while (0);")
    e("  }")
    e("  tila::tc_fence_before();")
    e("  __syncthreads();")
    e(f"  if (threadIdx.x < 32) tila::tmem_dealloc(*tila_tmem_slot, {cta_cols});")
    e("}")
    src = "\n".join(out) + "\n"
    if self._ws.get("heavy_last") is not None:
        from .wspec import cta_order_prelude
        decl = "  extern __shared__ __align__(1024) unsigned char tila_smem_all[];\n"
        head, body = src.split(decl, 1)
        body = body.replace("blockIdx.x", "tila_bx").replace("blockIdx.y", "tila_by").replace("blockIdx.z", "tila_bz")
        src = head + decl + cta_order_prelude(self._ws["heavy_last"]) + body
    self.fuse = {0: 2}
    tmem_cols = cta_cols
    return KernelSpec(self.entry, src, threads, max(total, 233472 // 2 - 1024 + 1), params,
                      fp_contract=True, assume_lines=list(self._assume_lines), tmem_cols=tmem_cols,
                      tensor_maps=list(self.tensor_maps), fuse={0: 2}, launch_regs=launch_regs)


KernelEmitter._ws_generate = _ws_generate_impl


class _PackedBin:
    """Expression maker of an f32 +, - or *; register tiles with an even
    number of slots are materialised two elements per f32x2 instruction."""

    def __init__(self, op):
        self.op = op
        self.fn = {"+": "add2", "-": "sub2", "*": "mul2"}[op]

    def __call__(self, e):
        return f"(({e[0]}) {self.op} ({e[1]}))"


class _PackedFma:
    """Expression maker of a contracted f32 a * b + c (one rounding); packed
    two elements per f32x2 FMA like _PackedBin."""
    fn = "fma2"

    def __call__(self, e):
        return f"__fmaf_rn(({e[0]}), ({e[1]}), ({e[2]}))"


class _UniformDivisor:
    """Expression maker of an f32 division (IEEE).  When a register tile is
    materialised and every element of a thread divides by the same value (a
    scalar, or a row value broadcast along the thread's elements), the
    emitter replaces it with the shared-reciprocal path
    (``KernelEmitter._uniform_division``), which yields the same quotients."""

    def __call__(self, e):
        return f"(({e[0]}) / ({e[1]}))"


class _BroadcastView(Layout):
    """Layout of a broadcast operand that mirrors a consumer layout slot by
    slot: slot r holds the operand element the consumer's slot r needs."""

    def __init__(self, consumer: Layout, cshape, oshape):
        self.consumer = consumer
        self.cshape = tuple(cshape)
        self.shape = tuple(oshape)
        self.rank = len(oshape)
        self.T = consumer.T
        self.nreg = consumer.nreg
        self.vec = 1

    def key(self):
        return ("bview", self.consumer.key(), self.cshape, self.shape)

    def valid_expr(self):
        return self.consumer.valid_expr()

    def coord(self, r):
        c = self.consumer.coord(r)
        c = tuple(c)[len(c) - self.rank:]
        return tuple("0" if n == 1 else i for i, n in zip(c, self.shape))

    def table(self):
        coords, owner = self.consumer._tables
        coords = coords[..., coords.shape[-1] - self.rank:]
        out = coords.copy()
        for i, n in enumerate(self.shape):
            if n == 1:
                out[..., i] = np.where(coords[..., i] >= 0, 0, -1)
        return out, np.zeros_like(owner)


def _tree_fold(terms, fold):
    """Pairwise combination of ``terms`` (depth log2(n))."""
    terms = list(terms)
    while len(terms) > 1:
        nxt = [fold(terms[i], terms[i + 1]) for i in range(0, len(terms) - 1, 2)]
        if len(terms) % 2:
            nxt.append(terms[-1])
        terms = nxt
    return terms[0]


def _affine_map(m):
    """(a, b) when slot map m is m[r] = a + b * r, else None."""
    if not m:
        return (0, 1)
    a = m[0]
    b = m[1] - m[0] if len(m) > 1 else 1
    if all(x == a + b * i for i, x in enumerate(m)):
        return (a, b)
    return None


def _pow2_div(v):
    v = int(v)
    if v == 0:
        return 256
    d = 1
    while v % (d * 2) == 0 and d < 256:
        d *= 2
    return d


def _pow2_at_least(n):
    p = 1
    while p < n:
        p *= 2
    return p


def _broadcast_shapes(shapes):
    shapes = [tuple(s) for s in shapes if s]
    if not shapes:
        return ()
    rank = max(len(s) for s in shapes)
    out = [1] * rank
    for s in shapes:
        s = (1,) * (rank - len(s)) + s
        for i, n in enumerate(s):
            if n != 1:
                out[i] = n
    return tuple(out)


def _vec_type(nbytes):
    return {16: "uint4", 8: "uint2", 4: "unsigned int", 2: "unsigned short"}[nbytes]


def _is_simple(expr):
    return expr.replace("_", "").isalnum()
