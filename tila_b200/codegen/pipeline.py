"""Analyses behind the TMA-fed, software-pipelined tensor-core path.

* :func:`tile_affinity` - how a coordinate expression depends on the tile
  indices: ``(c0, c1)`` with each coefficient 0 or 1 (None: not affine).
* :func:`plan_tma` - when a 2-D f16 ``load`` can be a TMA box copy: one
  buffer axis follows tile rows with unit step, one follows tile columns,
  every other coordinate is uniform, the tile's column-or-row axis is the
  buffer's contiguous axis, ``other`` is zero, and the mask is a
  conjunction of exactly the in-bounds conditions of the coordinates.  TMA
  fills out-of-bounds elements with zero, so the copy then produces exactly
  the masked load of the interpreter (interp.py:167-197): masked lanes read
  ``other`` = 0 and active lanes are in bounds by the proven obligations.
* :func:`match_contraction_loop` - a ``for`` loop whose carried tiles are
  only updated by ``acc = dot(a, b, acc=acc)`` with TMA-loadable (or
  loop-invariant shared-memory) operands: it lowers to a TMA ring plus
  asynchronous ``tcgen05.mma`` accumulating in tensor memory.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .._reference import tila

T_ = tila.tir
TY = tila.types


# ---------------------------------------------------------------------------
# name resolution and canonical forms
# ---------------------------------------------------------------------------

class Defs:
    """Single-assignment view of names: name -> defining TIR expression, for
    names assigned exactly once in the whole kernel (index math, masks)."""

    def __init__(self, body):
        self.defs = {}
        self.count = {}
        self.scopes = []          # loop-local definitions of the bodies being emitted
        self._collect(body)

    def _collect(self, body):
        for s in body:
            if isinstance(s, T_.TAssign):
                self.count[s.name] = self.count.get(s.name, 0) + 1
                self.defs[s.name] = s.value
            elif isinstance(s, (T_.TIf, T_.TStaticIf)):
                self._collect(s.then_body)
                self._collect(s.else_body)
            elif isinstance(s, T_.TFor):
                self.count[s.var] = self.count.get(s.var, 0) + 2   # never resolve loop vars
                self._collect(s.body)

    def resolve(self, node):
        seen = 0
        while isinstance(node, T_.TName) and seen < 64:
            for scope in reversed(self.scopes):
                if node.name in scope:
                    node = scope[node.name]
                    break
            else:
                if self.count.get(node.name) != 1:
                    break
                node = self.defs[node.name]
            seen += 1
        return node

    @staticmethod
    def loop_locals(body):
        """Names assigned exactly once in ``body`` (a loop's statement list,
        nested statements included) and never read in it before that
        assignment: their value inside the body is that single definition
        (names reused by another loop resolve per loop)."""
        order = []

        def flat(stmts):
            for st in stmts:
                order.append(st)
                if isinstance(st, (T_.TIf, T_.TStaticIf)):
                    flat(st.then_body)
                    flat(st.else_body)
                elif isinstance(st, T_.TFor):
                    flat(st.body)
        flat(body)
        count = {}
        for st in order:
            if isinstance(st, T_.TAssign):
                count[st.name] = count.get(st.name, 0) + 1
        out, defined, read_early = {}, set(), set()
        for st in order:
            names = []
            for fld in getattr(st, "__dataclass_fields__", {}):
                if fld in ("vt", "definition", "effect", "body", "then_body", "else_body", "name"):
                    continue
                _walk(getattr(st, fld), lambda n: names.append(n.name) if isinstance(n, T_.TName) else None)
            for n in names:
                if n not in defined:
                    read_early.add(n)
            if isinstance(st, T_.TAssign):
                defined.add(st.name)
                if count[st.name] == 1 and st.name not in read_early:
                    out[st.name] = st.value
        return out


def canon(node, defs: Defs, expand=None) -> str:
    """Canonical text of an index/mask expression with single-assignment
    names inlined and ``expand`` pushed down to the 1-D leaves."""
    node = defs.resolve(node)
    if isinstance(node, T_.TName):
        return node.name
    if isinstance(node, T_.TLit):
        return repr(node.value)
    if isinstance(node, T_.TPid):
        return f"pid{node.axis}"
    if isinstance(node, T_.TNumPrograms):
        return f"nprog{node.axis}"
    if isinstance(node, T_.TArange):
        e = f"arange({node.start},{canon(node.end, defs)})"
        return e if expand is None else f"x{expand}[{e}]"
    if isinstance(node, T_.TExpand):
        return canon(node.operand, defs, node.axis)
    if isinstance(node, T_.TBin):
        return f"({canon(node.left, defs, expand)} {node.op} {canon(node.right, defs, expand)})"
    if isinstance(node, T_.TUna):
        return f"({node.op} {canon(node.operand, defs, expand)})"
    if isinstance(node, T_.TCast):
        return f"cast_{node.dtype.name}({canon(node.operand, defs, expand)})"
    return f"?{type(node).__name__}@{id(node)}"


def tile_affinity(node, defs: Defs, consts, uniform_names, rank_hint=None):
    """Coefficients of a coordinate on the tile indices.

    Returns ``()`` for a uniform scalar, ``(c,)`` for a 1-D tile expression,
    ``(c0, c1)`` for a 2-D one (each 0 or 1), or None when the expression is
    not an affine function with unit coefficients.
    """
    node = defs.resolve(node)
    if isinstance(node, T_.TName):
        if node.name in consts or node.name in uniform_names:
            return ()
        return None
    if isinstance(node, (T_.TLit, T_.TPid, T_.TNumPrograms, T_.TConstant)):
        return ()
    if isinstance(node, T_.TArange):
        return (1,) if int(node.start) == 0 else None
    if isinstance(node, T_.TExpand):
        a = tile_affinity(node.operand, defs, consts, uniform_names)
        if a is None or len(a) != 1:
            return None
        return (a[0], 0) if node.axis == 1 else (0, a[0])
    if isinstance(node, T_.TCast):
        return tile_affinity(node.operand, defs, consts, uniform_names)
    if isinstance(node, T_.TBin):
        l = tile_affinity(node.left, defs, consts, uniform_names)
        r = tile_affinity(node.right, defs, consts, uniform_names)
        if l is None or r is None:
            return None
        if node.op in ("+", "-"):
            n = max(len(l), len(r))
            l = l + (0,) * (n - len(l)) if len(l) < n and len(l) == 0 else l
            r = r + (0,) * (n - len(r)) if len(r) < n and len(r) == 0 else r
            if len(l) == 0:
                l = (0,) * n
            if len(r) == 0:
                r = (0,) * n
            if len(l) != len(r):
                return None
            out = tuple(a + b if node.op == "+" else a - b for a, b in zip(l, r))
            if any(c not in (0, 1) for c in out):
                return None
            return out
        if node.op == "*":
            if l == () and r == ():
                return ()
            return None
        return None
    return None


# ---------------------------------------------------------------------------
# TMA plans
# ---------------------------------------------------------------------------

SWIZZLE_BYTES = 128          # 128-byte swizzle: inner box of 64 f16


@dataclass
class TmaPlan:
    """A 2-D tile copied between global and shared memory as TMA boxes.

    ``row_axis``/``col_axis``: buffer axes following tile dims 0 / 1.
    ``inner``: tile dim (0 or 1) lying along the buffer's contiguous axis.
    The tile is copied as ``nbox`` boxes of 128 contiguous bytes (64 f16 or
    32 f32 elements); box b covers inner indices [E b, E b + E) and lands
    ``outer * 128`` bytes after box b - 1 (the UMMA SWIZZLE_128B canonical
    layout for f16 operands).
    """
    buffer: str
    rank: int
    shape: tuple
    row_axis: int
    col_axis: int
    inner: int
    coord_nodes: tuple
    elem_bytes: int = 2

    @property
    def outer_extent(self):
        return self.shape[1 - self.inner]

    @property
    def inner_extent(self):
        return self.shape[self.inner]

    @property
    def box_elems(self):
        """Elements of the innermost box dim: 128 bytes (the swizzle span)."""
        return 128 // self.elem_bytes

    @property
    def nbox(self):
        return self.inner_extent // self.box_elems

    @property
    def box_bytes(self):
        return self.outer_extent * 128

    @property
    def bytes(self):
        return self.shape[0] * self.shape[1] * self.elem_bytes

    def box_dims(self):
        """Tensor-map box per buffer axis, innermost axis first."""
        dims = []
        for ax in reversed(range(self.rank)):
            if ax == self.rank - 1:
                dims.append(self.box_elems)
            elif ax == self.row_axis:
                dims.append(self.shape[0])
            elif ax == self.col_axis:
                dims.append(self.shape[1])
            else:
                dims.append(1)
        return tuple(dims)

    def key(self):
        return (self.buffer, self.rank, self.shape, self.row_axis, self.col_axis, self.inner)


def _mask_atoms(node, defs, out):
    node = defs.resolve(node)
    if isinstance(node, T_.TExpand):
        inner = defs.resolve(node.operand)
        if isinstance(inner, T_.TBin) and inner.op in ("&", "and"):
            _mask_atoms(T_.TExpand(node.vt, inner.left, node.axis), defs, out)
            _mask_atoms(T_.TExpand(node.vt, inner.right, node.axis), defs, out)
            return
        out.append(node)
        return
    if isinstance(node, T_.TBin) and node.op in ("&", "and"):
        _mask_atoms(node.left, defs, out)
        _mask_atoms(node.right, defs, out)
        return
    out.append(node)


def _split_cmp(atom, defs):
    """(op, left, right, expand_axis) of a comparison atom."""
    axis = None
    node = defs.resolve(atom)
    if isinstance(node, T_.TExpand):
        axis = node.axis
        node = defs.resolve(node.operand)
    if isinstance(node, T_.TBin) and node.op in ("<", ">=", "<=", ">"):
        return node.op, node.left, node.right, axis
    return None


def plan_tma_store(store, dims, defs: Defs, consts, uniform_names, buffer_param, facts):
    """TMA plan for a 2-D f32 tile ``store`` (TStore), or None: the same
    conditions as a load (affine tile coordinates, mask = bounds of the
    tiled coordinates), since a TMA store skips the box's out-of-bounds
    elements exactly like the masked store."""
    from types import SimpleNamespace
    view = SimpleNamespace(buffer=store.buffer, ptr=None, coords=store.coords, other=None,
                           mask=store.mask)
    return plan_tma(view, dims, defs, consts, uniform_names, buffer_param, facts,
                    dtypes=("f32",))


def plan_tma(load, dims, defs: Defs, consts, uniform_names, buffer_param, facts,
             dtypes=("f16",)) -> TmaPlan | None:
    """TMA plan for ``load`` (a TLoad with a 2-D result of one of ``dtypes``), or None."""
    if load.buffer is None or load.ptr is not None:
        return None
    if facts is None or not getattr(facts, "tma_ok", False):
        return None
    if len(dims) != 2:
        return None
    ename = buffer_param.vtype.elem.name
    if ename not in dtypes:
        return None
    elem_bytes = 2 if ename == "f16" else 4
    R, C = dims
    rank = len(load.coords)
    rows = cols = None
    for ax, c in enumerate(load.coords):
        a = tile_affinity(c, defs, consts, uniform_names)
        if a is None:
            return None
        if a in ((), (0,), (0, 0)):
            continue
        if a == (1, 0) and rows is None:
            rows = ax
        elif a == (0, 1) and cols is None:
            cols = ax
        else:
            return None
    if rows is None or cols is None:
        return None
    last = rank - 1
    if last == cols:
        inner = 1
    elif last == rows:
        inner = 0
    else:
        return None
    inner_extent = dims[inner]
    outer_extent = dims[1 - inner]
    if inner_extent % (128 // elem_bytes) or outer_extent > 256 or outer_extent < 8:
        return None
    # other must be zero (TMA fills out-of-bounds elements with zero)
    if load.other is not None:
        o = defs.resolve(load.other)
        if not (isinstance(o, T_.TLit) and o.value == 0):
            return None
    # mask: conjunction of in-bounds conditions on the tiled coordinates
    if load.mask is not None:
        atoms = []
        _mask_atoms(load.mask, defs, atoms)
        coord_canon = {}
        for ax in (rows, cols):
            coord_canon[canon(load.coords[ax], defs)] = ax
        bdims = buffer_param.vtype.dims
        for atom in atoms:
            cmp = _split_cmp(atom, defs)
            if cmp is None:
                return None
            op, left, right, axis = cmp
            if op == ">=":
                r = defs.resolve(right)
                if isinstance(r, T_.TLit) and r.value == 0 and \
                        tile_affinity(left, defs, consts, uniform_names) in ((1,), (1, 0), (0, 1)):
                    continue   # arange-based coordinates are never negative
                return None
            if op != "<":
                return None
            lc = canon(left, defs, axis)
            ax = coord_canon.get(lc)
            if ax is None:
                return None
            d = bdims[ax]
            r = defs.resolve(right)
            if not (isinstance(r, T_.TName) and getattr(d, "name", None) == r.name):
                return None
    return TmaPlan(load.buffer, rank, (R, C), rows, cols, inner, tuple(load.coords), elem_bytes)


# ---------------------------------------------------------------------------
# contraction loops
# ---------------------------------------------------------------------------

@dataclass
class DotSite:
    acc: str                 # carried accumulator name
    dot: object              # the TDot node
    a: object                # operand nodes (TLoad inside the loop, or outer names)
    b: object
    a_name: str | None
    b_name: str | None


@dataclass
class ContractionLoop:
    dots: list
    loads: dict = field(default_factory=dict)        # name -> TLoad (TMA in the ring)
    functional: list = field(default_factory=list)   # index/mask assignments


def match_contraction_loop(loop, defs: Defs, is_tma_load, is_smem_name, carried):
    """Match ``for k: <index math>; x = load(...); ...; acc = dot(x, y, acc=acc)``.

    ``is_tma_load(load_node)`` tells whether a load has a TMA plan;
    ``is_smem_name(name)`` whether an outer name already lives in shared
    memory (a loop-invariant operand loaded by TMA before the loop).
    """
    body = loop.body
    if not body or any(not isinstance(s, T_.TAssign) for s in body):
        return None
    assigned = {}
    for s in body:
        if s.name in assigned:
            return None      # reassigned inside the body: not a simple pipeline
        assigned[s.name] = s.value
    dots = []
    loads = {}
    functional = []
    used_as_operand = set()
    for s in body:
        v = s.value
        if isinstance(v, T_.TDot):
            if v.acc is None or not (isinstance(v.acc, T_.TName) and v.acc.name == s.name):
                return None
            if s.name not in carried:
                return None
            ops = []
            for op in (v.a, v.b):
                if isinstance(op, T_.TName) and op.name in assigned:
                    ld = assigned[op.name]
                    if not (isinstance(ld, T_.TLoad) and is_tma_load(ld)):
                        return None
                    loads[op.name] = ld
                    used_as_operand.add(op.name)
                    ops.append((ld, op.name))
                elif isinstance(op, T_.TName) and is_smem_name(op.name):
                    ops.append((op, op.name))
                else:
                    return None
            dots.append(DotSite(s.name, v, ops[0][0], ops[1][0], ops[0][1], ops[1][1]))
        elif isinstance(v, T_.TLoad):
            continue
        else:
            functional.append(s)
    if not dots:
        return None
    # every carried name must be a dot accumulator; loads only feed dots
    if set(carried) - {d.acc for d in dots}:
        return None
    for s in body:
        if isinstance(s.value, T_.TLoad) and s.name not in used_as_operand:
            return None
    # functional statements must not read loads, dots or accumulators
    banned = set(loads) | {d.acc for d in dots}

    def reads(node):
        if isinstance(node, T_.TName):
            return {node.name}
        out = set()
        if hasattr(node, "__dataclass_fields__"):
            for f in node.__dataclass_fields__:
                if f in ("vt", "definition", "effect"):
                    continue
                x = getattr(node, f)
                if isinstance(x, list):
                    for y in x:
                        out |= reads(y)
                elif hasattr(x, "__dataclass_fields__"):
                    out |= reads(x)
        return out
    for s in functional:
        if reads(s.value) & banned:
            return None
    for name in used_as_operand:
        # the operand tile must be consumed by the dots only
        for s in body:
            if isinstance(s.value, T_.TDot):
                continue
            if name in reads(s.value):
                return None
    return ContractionLoop(dots, loads, functional)


# ---------------------------------------------------------------------------
# asynchronous accumulator loops (online-softmax attention and relatives)
# ---------------------------------------------------------------------------

@dataclass
class AsyncLoop:
    """A loop whose carried accumulators stay in tensor memory.

    ``accs``: accumulator name -> its ``acc = dot(x, y, acc=acc)`` node; the
    dot runs asynchronously and is waited for lazily.  ``loads``: in-body
    loads that feed only dots and are TMA-copyable; each is copied one
    iteration ahead, as soon as the MMA that read it has completed.
    """
    accs: dict
    loads: dict
    # loads consumed only through cast[f16](...) as the A operand of an
    # accumulating dot: copied by TMA, read into registers, re-copied as soon
    # as every thread has read them
    cast_loads: set = field(default_factory=set)


def _walk(node, fn):
    fn(node)
    if hasattr(node, "__dataclass_fields__"):
        for f in node.__dataclass_fields__:
            if f in ("vt", "definition", "effect"):
                continue
            x = getattr(node, f)
            if isinstance(x, list):
                for y in x:
                    _walk(y, fn)
            elif hasattr(x, "__dataclass_fields__"):
                _walk(x, fn)


def match_async_loop(loop, defs: Defs, is_tma_load, is_smem_name, carried, acc_shape_ok,
                     is_tma_cast_load=None):
    body = loop.body
    if not body or any(not isinstance(s, T_.TAssign) for s in body):
        return None
    assigned = {}
    for s in body:
        assigned.setdefault(s.name, []).append(s.value)
    loads = {}
    for name, vals in assigned.items():
        if len(vals) == 1 and isinstance(vals[0], T_.TLoad) and is_tma_load(vals[0]):
            loads[name] = vals[0]
    # candidates read only through a cast feeding an accumulating dot's A
    cast_cands = {}
    if is_tma_cast_load is not None:
        for name, vals in assigned.items():
            if name not in loads and len(vals) == 1 and isinstance(vals[0], T_.TLoad) \
                    and is_tma_cast_load(vals[0]):
                cast_cands[name] = vals[0]
    # how every name is used inside the body
    uses = {}

    def record(parent):
        if not hasattr(parent, "__dataclass_fields__"):
            return
        for f in parent.__dataclass_fields__:
            if f in ("vt", "definition", "effect"):
                continue
            x = getattr(parent, f)
            for y in (x if isinstance(x, list) else [x]):
                if isinstance(y, T_.TName):
                    uses.setdefault(y.name, []).append((type(parent).__name__, f))
    for s in body:
        _walk(s.value, record)
    for name in list(loads):
        if not uses.get(name) or any(p != "TDot" or f not in ("a", "b") for p, f in uses[name]):
            del loads[name]
    cast_loads = set()
    for s in body:
        v = s.value
        if isinstance(v, T_.TDot) and isinstance(v.acc, T_.TName) and v.acc.name == s.name \
                and isinstance(v.a, T_.TCast) and isinstance(v.a.operand, T_.TName):
            n = v.a.operand.name
            if n in cast_cands and uses.get(n) == [("TCast", "operand")]:
                loads[n] = cast_cands[n]
                cast_loads.add(n)
    accs = {}
    for s in body:
        v = s.value
        if isinstance(v, T_.TDot) and isinstance(v.acc, T_.TName) and v.acc.name == s.name:
            if s.name not in carried or not acc_shape_ok(v):
                return None
            if not (isinstance(v.b, T_.TName) and v.b.name in loads):
                return None
            a = v.a
            ok_a = (isinstance(a, T_.TName) and (a.name in loads or is_smem_name(a.name))) or \
                (isinstance(a, T_.TCast) and a.dtype.name == "f16" and isinstance(a.operand, T_.TName)
                 and (a.operand.name not in loads or a.operand.name in cast_loads))
            if not ok_a or s.name in accs:
                return None
            accs[s.name] = v
    if not accs:
        return None
    # accumulators: besides their dot, only element-wise updates that read them
    for name in accs:
        for val in assigned[name]:
            if isinstance(val, T_.TDot):
                continue
            if not isinstance(val, (T_.TBin, T_.TUna, T_.TWhere, T_.TCast)):
                return None
        for p, f in uses.get(name, []):
            if p == "TDot" and f != "acc":
                return None
    # the other dots of the body: synchronous, operands in shared memory
    for s in body:
        def check(node):
            if isinstance(node, T_.TDot) and not (isinstance(node.acc, T_.TName) and node.acc.name in accs):
                for op in (node.a, node.b):
                    if not (isinstance(op, T_.TName) and (op.name in loads or is_smem_name(op.name))):
                        raise ValueError
        try:
            _walk(s.value, check)
        except ValueError:
            return None
    return AsyncLoop(accs, loads, cast_loads)
