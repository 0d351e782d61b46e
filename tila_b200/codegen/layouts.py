"""Register layouts of tile values inside one CTA (one Tila program).

A layout says which thread holds which element of a tile and in which
register slot.  Every layout can

* emit, for register slot ``r`` (an int or the C++ loop variable ``"r"``),
  the C++ index expression of each tile dimension in terms of ``tid``;
* produce the same mapping as a NumPy table ``coords[T, nreg, rank]`` with a
  boolean ``owner[T, nreg]`` (exactly one owner per element; other holders are
  replicas that never store or contribute to reductions twice).

The tables are what the code generator uses to decide whether a value can be
read in place by a consumer with another layout (same thread, slot known at
compile time) or must be redistributed through shared memory.  Tile dims are
powers of two (the verifier enforces it, verifier.py:106-120), so all the
index arithmetic below is exact.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import cached_property

import numpy as np


class Layout:
    rank: int
    shape: tuple
    T: int
    nreg: int
    vec: int = 1          # consecutive slots r..r+vec-1 hold consecutive last-dim indices

    def coord(self, r) -> tuple:
        raise NotImplementedError

    def owner_expr(self, r) -> str | None:
        """C++ predicate true when this thread owns slot r (None: always)."""
        return None

    def valid_expr(self) -> str | None:
        """C++ predicate true when this thread's slots hold tile elements at
        all (False for padding lanes); memory accesses are guarded by it."""
        return None

    def table(self):
        raise NotImplementedError

    def key(self):
        raise NotImplementedError

    def __eq__(self, other):
        return isinstance(other, Layout) and self.key() == other.key()

    def __hash__(self):
        return hash(self.key())

    @cached_property
    def _tables(self):
        return self.table()


def _tid_table(T):
    return np.arange(T, dtype=np.int64)


@dataclass(eq=False)
class Blocked(Layout):
    """Row-major blocked distribution of an (R, C) tile (1-D tiles: R = 1, rank 1;
    rank >= 3: R is the product of the leading dimensions, row-major).

    Threads form a ``tr x tc`` grid with columns fastest (coalesced).  Each
    thread holds ``RA`` rows (strided by ``tr``) and ``CB`` chunks of ``V``
    consecutive columns (chunks strided by ``tc * V``).  Threads beyond
    ``tr * tc`` replicate the first ``tr * tc`` threads.
    """
    shape: tuple
    T: int
    V: int

    def __post_init__(self):
        self.rank = len(self.shape)
        if self.rank == 1:
            R, C = 1, self.shape[0]
        else:
            R, C = int(np.prod(self.shape[:-1])), self.shape[-1]
        self.R, self.C = R, C
        V = min(self.V, C)
        self.V = V
        self.vec = V
        self.tc = min(C // V, self.T)
        self.tr = min(R, self.T // self.tc)
        self.RA = R // self.tr
        self.CB = C // (self.tc * V)
        self.nreg = self.RA * self.CB * V
        self.active = self.tr * self.tc

    def key(self):
        return ("blocked", self.shape, self.T, self.V)

    def _parts(self, r):
        V, CB = self.V, self.CB
        if isinstance(r, int):
            j, b, a = r % V, (r // V) % CB, r // (V * CB)
            return str(a), str(b), str(j)
        return f"(({r}) / {V * CB})", f"((({r}) / {V}) % {CB})", f"(({r}) % {V})"

    def coord(self, r):
        a, b, j = self._parts(r)
        tcol = f"(tid % {self.tc})" if self.tc > 1 else "0"
        trow = f"((tid / {self.tc}) % {self.tr})" if self.tr > 1 else "0"
        col = f"(({tcol} + {self.tc} * {b}) * {self.V} + {j})"
        if self.rank == 1:
            return (col,)
        row = f"({trow} + {self.tr} * {a})"
        if self.rank == 2:
            return (row, col)
        lead = self.shape[:-1]
        out = []
        for k in range(len(lead)):
            stride = int(np.prod(lead[k + 1:]))
            e = f"({row} / {stride})" if stride > 1 else row
            out.append(f"({e} % {lead[k]})" if k else e)
        return (*out, col)

    def owner_expr(self, r):
        return None if self.active >= self.T else f"(tid < {self.active})"

    def table(self):
        T = self.T
        tid = _tid_table(T)[:, None]
        r = np.arange(self.nreg)[None, :]
        V, CB = self.V, self.CB
        j, b, a = r % V, (r // V) % CB, r // (V * CB)
        tcol = tid % self.tc
        trow = (tid // self.tc) % self.tr
        col = (tcol + self.tc * b) * V + j
        row = trow + self.tr * a
        owner = np.broadcast_to(tid < self.active, (T, self.nreg))
        if self.rank == 1:
            coords = col[..., None]
        elif self.rank == 2:
            coords = np.stack(np.broadcast_arrays(row, col), axis=-1)
        else:
            lead = self.shape[:-1]
            parts = [(row // int(np.prod(lead[k + 1:]))) % lead[k] for k in range(len(lead))]
            coords = np.stack(np.broadcast_arrays(*parts, col), axis=-1)
        return np.broadcast_to(coords, (T, self.nreg, self.rank)).copy(), owner.copy()

    # thread-index bits that separate the partial results of a reduction
    def reduce_bits(self, axis):
        import math
        lc, lr = int(math.log2(self.tc)), int(math.log2(self.tr))
        if self.rank == 1 or axis == self.rank - 1:
            return list(range(0, lc))
        if self.rank == 2:
            return list(range(lc, lc + lr))
        # a leading axis occupies bits [lo, hi) of the flattened row index; the
        # thread's row (tid bits lc..lc+lr) holds the row index's low lr bits
        lead = self.shape[:-1]
        lo = int(math.log2(int(np.prod(lead[axis + 1:]))))
        hi = lo + int(math.log2(lead[axis]))
        return [lc + b for b in range(lo, min(hi, lr))]


@dataclass(eq=False)
class TmemRows(Layout):
    """The tcgen05.ld 32x32b register image of an (M, N) tile: warp w, lane l
    holds row ``32 * (w % 4) + l``; with T = 128 * G threads the N columns are
    split into G contiguous groups, group ``w / 4``.  Rows >= M are padding."""
    shape: tuple
    T: int

    def __post_init__(self):
        self.rank = 2
        M, N = self.shape
        self.G = self.T // 128
        self.cpg = max(N // self.G, 1)
        self.groups = N // self.cpg
        self.nreg = self.cpg
        self.vec = self.cpg

    def key(self):
        return ("tmemrows", self.shape, self.T)

    def coord(self, r):
        row = "((tid & 127))"
        if self.groups > 1:
            col = f"((tid >> 7) * {self.cpg} + ({r}))"
        else:
            col = f"({r})"
        return (row, col)

    def valid_expr(self):
        return self.owner_expr(0)

    def owner_expr(self, r):
        M = self.shape[0]
        conds = []
        if M < 128:
            conds.append(f"((tid & 127) < {M})")
        if self.groups < self.G:
            conds.append(f"((tid >> 7) < {self.groups})")
        return " && ".join(conds) if conds else None

    def table(self):
        T = self.T
        tid = _tid_table(T)[:, None]
        r = np.arange(self.nreg)[None, :]
        row = np.broadcast_to(tid & 127, (T, self.nreg))
        grp = tid >> 7
        col = np.broadcast_to(grp * self.cpg + r, (T, self.nreg))
        M = self.shape[0]
        owner = (row < M) & (np.broadcast_to(grp, (T, self.nreg)) < self.groups)
        coords = np.stack([np.where(owner, row, -1), np.where(owner, col, -1)], axis=-1)
        return coords, owner

    def reduce_bits(self, axis):
        import math
        if axis == 1:
            return list(range(7, 7 + int(math.log2(self.G))))
        return list(range(0, 7))


@dataclass(eq=False)
class Derived(Layout):
    """A layout obtained from a parent by slicing out a reduced axis,
    inserting a unit axis (expand) or reshaping.  ``regs`` lists the parent
    slots kept (for slices) so that slot r of this layout is parent slot
    ``regs[r]``; its coordinates are the parent's, transformed by ``kind``.

    kinds: ("slice", axis) drops ``axis``; ("expand", axis) inserts a unit
    axis at ``axis``; ("reshape", new_shape) re-indexes the flat position.
    Replicas of a slice (threads that hold the same reduced element) are
    owners only when they are the first of their reduction group.
    """
    parent: Layout
    kind: tuple
    shape: tuple
    regs: tuple
    owner_fn: object = None     # optional callable(table_owner) -> owner

    def __post_init__(self):
        self.rank = len(self.shape)
        self.T = self.parent.T
        self.nreg = len(self.regs)
        self.vec = 1
        if self.kind[0] == "expand" and self.kind[1] != self.rank - 1:
            self.vec = self._parent_vec_kept()
        elif self.kind[0] == "slice" and self.kind[1] != self.parent.rank - 1:
            self.vec = self._parent_vec_kept()

    def _parent_vec_kept(self):
        pv = self.parent.vec
        regs = list(self.regs)
        if pv <= 1 or len(regs) % pv:
            return 1
        for g in range(0, len(regs), pv):
            if regs[g:g + pv] != list(range(regs[g], regs[g] + pv)) or regs[g] % pv:
                return 1
        return pv

    def key(self):
        return ("derived", self.parent.key(), self.kind, self.shape, self.regs)

    def coord(self, r):
        if isinstance(r, int):
            pr = self.regs[r]
        else:
            pr = self._reg_expr(r)
        pc = self.parent.coord(pr)
        kind = self.kind[0]
        if kind == "slice":
            ax = self.kind[1]
            return tuple(c for i, c in enumerate(pc) if i != ax)
        if kind == "expand":
            ax = self.kind[1]
            out = list(pc)
            out.insert(ax, "0")
            return tuple(out)
        if kind == "reshape":
            old = self.parent.shape
            flat = " + ".join(f"({c}) * {int(np.prod(old[i + 1:]))}" for i, c in enumerate(pc))
            new = self.shape
            outs = []
            for i in range(len(new)):
                inner = int(np.prod(new[i + 1:]))
                outs.append(f"((({flat}) / {inner}) % {new[i]})")
            return tuple(outs)
        raise AssertionError(kind)

    def _reg_expr(self, r):
        regs = list(self.regs)
        if regs == list(range(len(regs))):
            return r
        # regs is an arithmetic progression in the common slice cases
        if len(regs) > 1:
            step = regs[1] - regs[0]
            if all(regs[i] == regs[0] + i * step for i in range(len(regs))):
                return f"({regs[0]} + {step} * ({r}))"
            # groups of consecutive slots
        raise ValueError("non-affine register subset needs straight-line emission")

    def reg_affine(self) -> bool:
        try:
            self._reg_expr("r")
            return True
        except ValueError:
            return False

    def owner_expr(self, r):
        return self._owner_expr

    _owner_expr = None

    def valid_expr(self):
        return self.parent.valid_expr()

    def table(self):
        pcoords, powner = self.parent._tables
        sel = pcoords[:, list(self.regs), :]
        kind = self.kind[0]
        if kind == "slice":
            ax = self.kind[1]
            coords = np.delete(sel, ax, axis=-1)
        elif kind == "expand":
            ax = self.kind[1]
            coords = np.insert(sel, ax, 0, axis=-1)
            coords = np.where(sel[..., :1] < 0, -1, coords)
        else:
            old = self.parent.shape
            strides = [int(np.prod(old[i + 1:])) for i in range(len(old))]
            flat = sum(sel[..., i] * strides[i] for i in range(len(old)))
            new = self.shape
            coords = np.stack([(flat // int(np.prod(new[i + 1:]))) % new[i]
                               for i in range(len(new))], axis=-1)
            coords = np.where(sel[..., :1] < 0, -1, coords)
        owner = powner[:, list(self.regs)]
        if self.owner_fn is not None:
            owner = self.owner_fn(coords, owner)
        return coords.copy(), owner.copy()


def dedupe_owner(coords, owner):
    """Keep one owner per element: the lowest thread (then slot) holding it."""
    T, n, rank = coords.shape
    seen = set()
    out = np.zeros_like(owner)
    for t in range(T):
        for r in range(n):
            c = tuple(coords[t, r])
            if c[0] < 0 or not owner[t, r]:
                continue
            if c not in seen:
                seen.add(c)
                out[t, r] = True
    return out


def owner_predicate(layout: Layout):
    """Owner predicate of a derived layout as per-thread C++ condition, or None.

    Returns (expr, per_slot) where per_slot is False when one condition on
    ``tid`` covers every slot.
    """
    coords, owner = layout._tables
    if owner.all():
        return None
    # common case: ownership depends on the thread only
    per_thread = owner.all(axis=1) | (~owner).all(axis=1)
    if per_thread.all():
        tids = np.nonzero(owner.all(axis=1))[0]
        return _tid_set_expr(tids, layout.T)
    return "PER_SLOT"


def _tid_set_expr(tids, T):
    tids = [int(t) for t in tids]
    if not tids:
        return "false"
    s = set(tids)
    if len(s) == T:
        return None
    # try a bitmask form: tid & mask == value
    for mask in range(1, 1 << max(1, (T - 1).bit_length())):
        vals = {t & mask for t in tids}
        if len(vals) == 1:
            v = vals.pop()
            if s == {t for t in range(T) if (t & mask) == v}:
                return f"((tid & {mask}) == {v})"
    if tids == list(range(len(tids))):
        return f"(tid < {len(tids)})"
    return None


def source_slot_map(src: Layout, dst: Layout, dst_shape, need_owner_only=False):
    """For consumer ``dst`` reading a value laid out as ``src`` (shape
    broadcast to ``dst_shape``), return the list of source slots per
    consumer slot, or None when some thread does not hold what it needs at a
    thread-independent slot."""
    scoords, _ = src._tables
    dcoords, downer = dst._tables
    T = dst.T
    if src.T != T:
        return None
    srank, drank = src.rank, len(dst_shape)
    sshape = tuple(src.shape)
    if srank < drank:
        sshape = (1,) * (drank - srank) + sshape
    # flatten source coordinates to element indices
    sdims = [int(d) for d in sshape]
    strides = [int(np.prod(sdims[i + 1:])) for i in range(drank)]
    sc = scoords
    if srank < drank:
        pad = np.zeros(sc.shape[:2] + (drank - srank,), dtype=sc.dtype)
        sc = np.concatenate([pad, sc], axis=-1)
    valid = sc[..., 0] >= 0
    sflat = np.where(valid, sum(sc[..., i] * strides[i] for i in range(drank)), -1)
    numel = int(np.prod(sdims))
    lookup = np.full((T, numel), -1, dtype=np.int64)
    tt, rr = np.nonzero(valid)
    lookup[tt, sflat[tt, rr]] = rr
    dc = dcoords
    need = dc[..., 0] >= 0
    if need_owner_only:
        need = need & downer
    nflat = sum(np.where(np.array(sdims[i]) == 1, 0, dc[..., i]) * strides[i]
                for i in range(drank))
    nflat = np.where(need, nflat, 0)
    found = np.take_along_axis(lookup, nflat, axis=1)
    found = np.where(need, found, -2)
    out = []
    for r in range(dst.nreg):
        col = found[:, r]
        col = col[col != -2]
        if col.size == 0:
            out.append(0)
            continue
        if (col < 0).any() or (col != col[0]).any():
            return None
        out.append(int(col[0]))
    return out
