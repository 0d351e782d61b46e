"""Tensor-core lowering of ``dot``: TMA-fed operands, asynchronous
``tcgen05.mma`` into tensor memory, and pipelined contraction loops.

Mixed into :class:`tila_b200.codegen.emitter.KernelEmitter`.

Shared-memory operand layouts (the UMMA canonical layouts):

* TMA-loaded tiles use SWIZZLE_128B: the tile is cut into boxes of 64
  contiguous f16 elements; box b holds ``outer`` rows of 128 bytes and sits
  ``outer * 128`` bytes after box b - 1.  K-major operands advance 32 bytes
  per 16-element K step inside a box (SBO = 1024 bytes between 8-row groups);
  MN-major operands advance 2048 bytes (16 rows) per K step with
  LBO = box stride and SBO = 1024 bytes.
* Register tiles (computed operands) are written K-major without swizzle
  (core matrices of 8 rows x 16 bytes, LBO = 128 bytes, SBO = K * 16 bytes).

The instruction shape is always M = 128 (cta_group::1); tiles with fewer
rows leave padding rows that are never read back.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import numpy as np

from .._reference import tila
from . import dtypes as DT
from .layouts import TmemRows, owner_predicate
from .pipeline import Defs, TmaPlan, match_contraction_loop, plan_tma

T_ = tila.tir
D = tila.dtypes


@dataclass
class SmemOperand:
    """A tile in shared memory.  One-shot TMA loads carry their mbarrier, the
    per-thread phase bit of that barrier and a per-thread "already waited for
    this issue" flag, so a consumer inside a loop waits exactly once per copy."""
    plan: TmaPlan
    base: str                  # smem byte offset expression (relative to tila_smem)
    bar: str | None = None     # mbarrier of a one-shot load (None: ready by construction)
    phase: str = "0u"
    flag: str | None = None
    nbytes: int = 0            # size of a one-shot load's buffer (0: not a one-shot load)


class MmaMixin:

    # -- set-up ---------------------------------------------------------------

    def _init_mma(self):
        self.pdefs = Defs(self.tk.body)
        self.uses = {}
        self._collect_uses(self.tk.body, None, None)
        self.tma_plans = {}
        self.tensor_maps = []          # [(param, buffer, box, plan)]
        self._tm_index = {}
        self.tmem_next = 0             # bump allocator of TMEM columns for carried accumulators
        self.tmem_scratch_col = None

    def _collect_uses(self, node, parent, fld):
        if isinstance(node, list):
            for x in node:
                self._collect_uses(x, parent, fld)
            return
        if isinstance(node, T_.TName):
            self.uses.setdefault(node.name, []).append((type(parent).__name__, fld))
            return
        if dataclasses.is_dataclass(node):
            for f in dataclasses.fields(node):
                if f.name in ("vt", "definition", "effect"):
                    continue
                self._collect_uses(getattr(node, f.name), node, f.name)

    def _dot_only(self, name):
        uses = self.uses.get(name, [])
        return bool(uses) and all(p == "TDot" and f in ("a", "b") for p, f in uses)

    def _uniform_names(self):
        return set(self.scalar_params) | set(self._loopvars)

    def tma_plan(self, load, cast=False):
        """TMA plan of a tile load: f16 MMA operands, or with ``cast`` also
        f32 tiles that are read into registers."""
        key = (id(load), cast)
        if key in self.tma_plans:
            return self.tma_plans[key]
        plan = None
        if load.buffer is not None and load.buffer in self.buffer_params:
            dt, shape, _ = self.vt_info(load.vt)
            plan = plan_tma(load, shape, self.pdefs, self.consts, self._uniform_names(),
                            self.buffer_params[load.buffer], self.buffers.get(load.buffer),
                            dtypes=("f16", "f32") if cast else ("f16",))
        self.tma_plans[key] = plan
        return plan

    # -- tensor maps --------------------------------------------------------------

    def tensor_map_param(self, plan: TmaPlan) -> str:
        key = (plan.buffer, plan.box_dims())
        if key not in self._tm_index:
            name = f"tm_{len(self._tm_index)}"
            self._tm_index[key] = name
            self.tensor_maps.append({"param": name, "buffer": plan.buffer,
                                     "box": list(plan.box_dims()), "swizzle": 128,
                                     "dtype": "f16" if plan.elem_bytes == 2 else "f32"})
        return self._tm_index[key]

    def _tma_coords(self, plan: TmaPlan, coords):
        """Innermost-first TMA coordinates (uniform tile origin per axis)."""
        origin = []
        zero = ("0", "0")
        for c in coords:
            if c.kind == "scalar":
                origin.append(f"(int)({c.expr})")
            elif c.kind == "func":
                origin.append(f"(int)({c.fn(self.bcast_idx(zero, c.shape))})")
            else:
                self.fail("TMA coordinate is not an index expression")
        return list(reversed(origin))

    def _emit_tma(self, plan: TmaPlan, coords_if, dst: str, bar: str):
        tm = self.tensor_map_param(plan)
        rank = plan.rank
        if rank not in (2, 3, 4):
            self.fail("TMA loads support buffers of rank 2 to 4")
        for b in range(plan.nbox):
            cs = list(coords_if)
            if b:
                cs[0] = f"({cs[0]} + {plan.box_elems * b})"
            args = ", ".join(cs)
            self.emit(f"tila::tma_load_{rank}d(tila_smem + {dst} + {b * plan.box_bytes}, &{tm}, {bar}, {args});")

    # -- one-shot TMA loads -----------------------------------------------------------

    def try_tma_load(self, x, assigned_name=None):
        """Lower a dot-operand load to a TMA copy into shared memory."""
        if assigned_name is None or not self._dot_only(assigned_name):
            return None
        plan = self.tma_plan(x)
        if plan is None:
            return None
        coords = [self.value(c) for c in x.coords]
        if any(c.kind not in ("scalar", "func") for c in coords):
            return None
        if self._ws is not None and assigned_name == self._ws["q"]:
            return self.ws_oneshot(x, assigned_name, plan, coords)
        size = plan.nbox * max(plan.outer_extent, 128) * 128
        off = self.smem.alloc(size, 1024)
        bar_off = self.smem.alloc(8, 8)
        bar = f"reinterpret_cast<tila::u64*>(tila_smem + {bar_off})"
        self._need_barrier_init.append(bar_off)
        self.emit(f"// TMA load of {x.buffer} ({plan.shape[0]}x{plan.shape[1]}) into shared memory")
        self.emit("if (tid == 0) {")
        self.indent += 1
        self.emit(f"tila::mbar_arrive_expect_tx({bar}, {plan.bytes}u);")
        self._emit_tma(plan, self._tma_coords(plan, coords), str(off), bar)
        self.indent -= 1
        self.emit("}")
        phase = self._tma_state_var(f"tila_ph_{bar_off}")
        flag = self._tma_state_var(f"tila_w_{bar_off}")
        self.emit(f"{flag} = 0u;")
        dt, shape, _ = self.vt_info(x.vt)
        return self._smem_val(dt, shape, SmemOperand(plan, str(off), bar, phase, flag, nbytes=size))

    def _tma_state_var(self, name):
        """Per-thread state of a one-shot TMA barrier (declared at kernel entry)."""
        if name not in self._phase_vars:
            self._phase_vars.append(name)
        return name

    def emit_smem_wait(self, v):
        """Every thread waits (once per issue) for a one-shot TMA tile."""
        op = v.smem
        if op.bar is None:
            return
        self.emit(f"if (!{op.flag}) {{ tila::mbar_wait({op.bar}, {op.phase}, tila_err, __LINE__, &tila_dead);"
                  f" {op.phase} ^= 1u; {op.flag} = 1u; }}")

    def _smem_val(self, dt, shape, op: SmemOperand):
        from .emitter import Val
        v = Val("smem", dt, tuple(shape))
        v.smem = op
        return v

    # -- descriptors ------------------------------------------------------------------

    def _operand_desc(self, v, role, kk):
        """(descriptor C++ expr, mn_major) for K step kk of an operand."""
        op = v.smem
        plan = op.plan
        R, C = plan.shape
        if role == "A":
            k_major = plan.inner == 1
        else:
            k_major = plan.inner == 0
        k0 = 16 * kk
        if k_major:
            box, within = divmod(k0, 64)
            off = f"{op.base} + {box * plan.box_bytes + within * 2}"
            return (f"tila::sdesc<16, 1024, 2>(tila_sb4, (tila::u32)({off}))", 0)
        off = f"{op.base} + {k0 * 128}"
        return (f"tila::sdesc<{plan.box_bytes}, 1024, 2>(tila_sb4, (tila::u32)({off}))", 1)

    # -- dot ----------------------------------------------------------------------------

    def tmem_alloc_cols(self, n):
        col = self.tmem_next
        self.tmem_next += n
        return col

    def e_TDot(self, x):
        dt, shape, _ = self.vt_info(x.vt)
        ctx = self.actx
        if ctx is not None and getattr(ctx, "ws", False) and x.acc is None:
            return self.ws_sync_dot(x)
        # In an asynchronous loop whose synchronous dot reads two TMA tiles,
        # that dot's MMAs for the next iteration are issued right behind the
        # accumulating dot (see emit_async_acc_dot); tila_s_pre records it.
        hoist = (ctx is not None and getattr(ctx, "pingpong", False) and x.acc is None
                 and isinstance(x.a, T_.TName) and isinstance(x.b, T_.TName)
                 and getattr(self.env.get(x.a.name), "kind", None) == "smem"
                 and getattr(self.env.get(x.b.name), "kind", None) == "smem")
        if hoist:
            self.emit(f"if (!{self._s_pre_var()}) {{")
            self.indent += 1
        if ctx is not None:
            self.wait_all_accs(release=True)
        a = self.value(x.a)
        b = self.value(x.b)
        acc = self.value(x.acc) if x.acc is not None else None
        M, K = a.shape
        K2, N = b.shape
        if K != K2 or (M, N) != tuple(shape):
            self.fail("dot shape mismatch")
        if M > 128:
            self.fail("dot with more than 128 rows is not supported yet")
        if N > 256:
            self.fail("dot with more than 256 columns is not supported yet")
        Npad = max(16, N)
        if Npad % 16:
            self.fail("dot N must be a multiple of 16 or smaller than 16")
        self.uses_mma = True
        self.uses_tmem = True
        self.tmem_scratch_need = max(self.tmem_scratch_need, Npad)
        col = "tila_tmem_scratch_col"
        descs = {}
        if a.kind == "smem":
            if a.smem.plan.shape[0] != 128 and a.smem.plan.inner == 0:
                a = self.smem_to_reg(a)
            elif a.smem.plan.shape[0] < 128:
                a = self.smem_to_reg(a)
        if b.kind == "smem" and b.smem.plan.shape[1] != Npad:
            b = self.smem_to_reg(b)
        if a.kind != "smem":
            a_off = self.smem.alloc(128 * K * 2, 1024)
            self._stage_operand(a, a_off, K, transpose=False)
            descs["A"] = lambda kk, o=a_off: (f"tila::sdesc<128, {K * 16}, 0>(tila_sb4, (tila::u32)({o} + {kk} * 256))", 0)
        else:
            descs["A"] = lambda kk, v=a: self._operand_desc(v, "A", kk)
        if b.kind != "smem":
            b_off = self.smem.alloc(Npad * K * 2, 1024)
            self._stage_operand(b, b_off, K, transpose=True)
            descs["B"] = lambda kk, o=b_off: (f"tila::sdesc<128, {K * 16}, 0>(tila_sb4, (tila::u32)({o} + {kk} * 256))", 0)
        else:
            descs["B"] = lambda kk, v=b: self._operand_desc(v, "B", kk)
        accumulate = "0"
        if acc is not None and not (acc.kind == "func" and acc.zero):
            accv = acc if acc.kind != "tmem" else self.tmem_to_reg(acc)
            if accv.dt.name != "f32":
                accv = self.coerce(accv, D.f32)
            lay = TmemRows((M, N), self.T)
            if accv.kind == "scalar":
                accv = self.materialize_elementwise(D.f32, (M, N), [accv], lambda e: e[0], layout=lay)
            accv = self.materialize(accv, lay) if not (accv.kind == "reg" and accv.layout == lay) else accv
            self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {col}"
                      + (f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else "")
                      + f" + ((tid & 96u) << 16), {accv.name});")
            accumulate = "1"
        for v in (a, b):
            if v.kind == "smem":
                self.emit_smem_wait(v)
        self.emit("tila::fence_proxy_async_smem();")
        self.emit("tila::tc_fence_before();")
        self.emit("__syncthreads();")
        self.emit("tila::tc_fence_after();")
        issue_at = len(self.lines)
        issue_indent = self.indent
        self.emit("if (tid == 0) {")
        self.indent += 1
        a_mn = descs["A"](0)[1]
        b_mn = descs["B"](0)[1]
        idesc = f"tila::idesc_f16_f32(128, {Npad}, {a_mn}, {b_mn})"
        for kk in range(K // 16):
            da, _ = descs["A"](kk)
            db, _ = descs["B"](kk)
            acc_flag = "1u" if kk > 0 else f"{accumulate}u"
            self.emit(f"tila::mma_f16_ss(tila_tmem + {col}, {da}, {db}, {idesc}, {acc_flag});")
        self.emit("tila::mma_commit(tila_mma_bar);")
        self.indent -= 1
        self.emit("}")
        if hoist:
            pad = "  " * issue_indent
            ctx.s_issue = [l[len(pad):] if l.startswith(pad) else l.lstrip() for l in self.lines[issue_at:]]
            ctx.s_operands = [v for v in (a, b) if v.kind == "smem"]
            self.indent -= 1
            self.emit("}")
            self.emit(f"{self._s_pre_var()} = 0u;")
        self.emit("tila::mbar_wait(tila_mma_bar, tila_mma_phase, tila_err, __LINE__, &tila_dead);")
        self.emit("tila_mma_phase ^= 1u;")
        self.emit("tila::tc_fence_after();")
        if ctx is None and not self._loopvars:
            # one-shot TMA operands read only by this dot are dead once its MMAs
            # completed: their shared memory can stage later stores
            for v in (a, b):
                name = getattr(v, "smem_name", None)
                op = getattr(v, "smem", None)
                if v.kind == "smem" and name and len(self.uses.get(name, [])) == 1 \
                        and op.nbytes and op.base.isdigit():
                    self._free_smem.append((int(op.base), op.nbytes))
        if ctx is not None:
            if hoist:
                # MMAs complete in issue order: the accumulating dot issued
                # before this one is done too (its buffers can be refilled)
                self.wait_all_accs(release=True)
            # refill the operands this dot consumed before waiting for the
            # hand-off, so the copies overlap the wait
            self.release_after_sync_dot([a, b])
            if getattr(ctx, "pingpong", False):
                # start of the CUDA-core phase of the iteration (see WG_ACQUIRE)
                self.emit(WG_ACQUIRE)
        from .emitter import Val
        res = Val("tmem", D.f32, (M, N), tmem_col=col)
        reg = self.tmem_to_reg(res)
        if dt.name == "f16":
            reg = self.materialize_elementwise(dt, (M, N), [reg], lambda e: f"tila::round_f16({e[0]})",
                                               layout=reg.layout)
        self.emit("tila::tc_fence_before();")
        return reg

    def smem_rows_to_reg(self, v, lay):
        """Read a TMA-copied (SWIZZLE_128B) tile whose columns run along the
        buffer's contiguous axis into the row-per-thread register image
        ``lay`` (TmemRows): 16-byte shared loads, four lanes per bank group."""
        from .emitter import Val
        plan = v.smem.plan
        if plan.inner != 1 or plan.shape[0] != 128 or not isinstance(lay, TmemRows):
            self.fail("row read of a shared-memory tile needs 128 rows with contiguous columns")
        self.emit_smem_wait(v)
        name = self.fresh("sr")
        eb = plan.elem_bytes
        per = 16 // eb                    # elements per 16-byte chunk
        be = plan.box_elems
        col0 = f"(tid >> 7) * {lay.cpg} + " if lay.groups > 1 else ""
        self.emit(f"float {name}[{lay.nreg}];")
        self.emit("{")
        self.indent += 1
        self.emit("const int row_ = tid & 127;")
        self.emit("#pragma unroll")
        self.emit(f"for (int r = 0; r < {lay.nreg}; r += {per}) {{")
        self.indent += 1
        self.emit(f"const int c_ = {col0}r;")
        addr = (f"tila_smem + {v.smem.base} + (c_ / {be}) * {plan.box_bytes} + row_ * 128 + "
                f"((((c_ % {be}) / {per}) ^ (row_ & 7)) * 16)")
        if eb == 4:
            self.emit(f"const float4 q_ = *reinterpret_cast<const float4*>({addr});")
            self.emit(f"{name}[r] = q_.x; {name}[r + 1] = q_.y; {name}[r + 2] = q_.z; {name}[r + 3] = q_.w;")
        else:
            self.emit(f"const uint4 q_ = *reinterpret_cast<const uint4*>({addr});")
            self.emit("const tila::u32 w_[4] = {q_.x, q_.y, q_.z, q_.w};")
            self.emit("#pragma unroll")
            self.emit(f"for (int j = 0; j < 4; ++j) {{ {name}[r + 2 * j] = tila::h2f((tila::u16)(w_[j] & 0xffffu)); "
                      f"{name}[r + 2 * j + 1] = tila::h2f((tila::u16)(w_[j] >> 16)); }}")
        self.indent -= 1
        self.emit("}")
        self.indent -= 1
        self.emit("}")
        return Val("reg", v.dt, tuple(v.shape), name=name, layout=lay)

    def smem_to_reg(self, v):
        """Read a TMA-loaded (SWIZZLE_128B) tile from shared memory into registers."""
        plan = v.smem.plan
        layout = self.default_layout(v.shape, v.dt)
        self.emit_smem_wait(v)
        name = self.fresh("sm")
        self.emit(f"float {name}[{layout.nreg}];")
        self.emit("#pragma unroll")
        self.emit(f"for (int r = 0; r < {layout.nreg}; ++r) {{")
        i, j = layout.coord("r")
        inner, outer = (i, j) if plan.inner == 0 else (j, i)
        # box = inner / 64, row = outer, 16-byte chunk = (inner % 64) / 8 xor (row % 8)
        addr = (f"{v.smem.base} + (({inner}) / 64) * {plan.box_bytes} + ({outer}) * 128 + "
                f"(((((({inner}) % 64) / 8) ^ (({outer}) % 8))) * 16) + ((({inner}) % 8) * 2)")
        valid = layout.valid_expr()
        load = f"tila::h2f(*reinterpret_cast<const tila::u16*>(tila_smem + {addr}))"
        self.emit(f"  {name}[r] = {('(' + valid + ') ? ' + load + ' : 0.0f') if valid else load};")
        self.emit("}")
        from .emitter import Val
        return Val("reg", v.dt, tuple(v.shape), name=name, layout=layout)

    # -- pipelined contraction loops ------------------------------------------------

    def try_contraction_loop(self, s, start, end, stepv, carried):
        if stepv <= 0:
            return False

        def is_tma(ld):
            p = self.tma_plan(ld)
            return p is not None

        def is_smem(name):
            v = self.env.get(name)
            return v is not None and v.kind == "smem"
        cl = match_contraction_loop(s, self.pdefs, is_tma, is_smem, carried)
        if cl is None:
            return False
        # shape constraints of the instruction: M = 128, 16 <= N <= 256
        for d in cl.dots:
            dt, shape, _ = self.vt_info(d.dot.vt)
            M, N = shape
            if M != 128 or N % 16 or N > 256 or dt.name != "f32":
                return False
            for role, node, name in (("A", d.a, d.a_name), ("B", d.b, d.b_name)):
                plan = self.tma_plan(node) if isinstance(node, T_.TLoad) else self.env[name].smem.plan
                if role == "A" and plan.shape[0] != 128:
                    return False
                if role == "B" and plan.shape[1] != N:
                    return False
        self._emit_contraction(s, cl, start, end, stepv)
        return True

    def _emit_contraction(self, s, cl, start, end, stepv):
        self.uses_mma = True
        self.uses_tmem = True
        var = s.var
        loads = list(cl.loads.items())
        plans = {n: self.tma_plan(ld) for n, ld in loads}
        # stage layout
        offs, stage = {}, 0
        for n, _ in loads:
            offs[n] = stage
            stage += (plans[n].nbox * plans[n].box_bytes + 1023) // 1024 * 1024
        tx = sum(plans[n].bytes for n, _ in loads)
        budget = 110 * 1024
        S = max(2, min(6, budget // max(stage, 1)))
        ring = self.smem.alloc(S * stage, 1024)
        bars = self.smem.alloc(8 * (2 * S + 1), 8)
        full = lambda i: f"reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * ({i}))"
        empty = lambda i: f"reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * ({S} + ({i})))"
        accbar = f"reinterpret_cast<tila::u64*>(tila_smem + {bars + 16 * S})"
        # accumulators into tensor memory
        acc_cols = {}
        for d in cl.dots:
            dt, (M, N), _ = self.vt_info(d.dot.vt)
            col = self.tmem_alloc_cols(N)
            acc_cols[d.acc] = (col, N)
            pre = self.env[d.acc]
            if pre.kind == "tmem" and pre.tmem_col == col:
                continue
            lay = TmemRows((M, N), self.T)
            if pre.kind == "tmem":
                pre = self.tmem_to_reg(pre)
            if pre.dt.name != "f32":
                pre = self.coerce(pre, D.f32)
            if pre.kind == "scalar":
                pre = self.materialize_elementwise(D.f32, (M, N), [pre], lambda e: e[0], layout=lay)
            pre = self.materialize(pre, lay)
            self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {col}"
                      + (f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else "")
                      + f" + ((tid & 96u) << 16), {pre.name});")
        self.emit(f"{{ // pipelined contraction loop over {var}: {S}-stage TMA ring, tcgen05.mma into TMEM")
        self.indent += 1
        self.emit(f"const tila::i64 cl_start = (tila::i64)({start.expr});")
        self.emit(f"const tila::i64 cl_end = (tila::i64)({end.expr});")
        self.emit(f"const tila::i64 cl_n = cl_end > cl_start ? (cl_end - cl_start + {stepv - 1}) / {stepv} : 0;")
        self.emit("if (tid == 0) {")
        self.emit(f"  for (int i = 0; i < {2 * S + 1}; ++i) tila::mbar_init(reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * i), 1);")
        self.emit("  tila::mbar_fence_init();")
        self.emit("}")
        self.emit("tila::tc_fence_before();")
        self.emit("__syncthreads();")
        self.emit("tila::tc_fence_after();")
        # loop-invariant shared-memory operands must have landed
        for d in cl.dots:
            for name in (d.a_name, d.b_name):
                if name not in cl.loads:
                    self.emit_smem_wait(self.env[name])
        def issue(jexpr, stage_expr):
            self.emit("{")
            self.indent += 1
            lv = self.fresh(f"s_{var}")
            self.emit(f"const tila::i32 {lv} = (tila::i32)(cl_start + ({jexpr}) * {stepv});")
            saved = dict(self.env)
            self.env[var] = self._scalar(D.i32, lv)
            for st in cl.functional:
                self.s_TAssign(st)
            self.emit(f"tila::mbar_arrive_expect_tx({full(stage_expr)}, {tx}u);")
            for n, ld in loads:
                coords = [self.value(c) for c in ld.coords]
                dst = f"{ring} + ({stage_expr}) * {stage} + {offs[n]}"
                self._emit_tma(plans[n], self._tma_coords(plans[n], coords), dst, full(stage_expr))
            self.env = saved
            self.indent -= 1
            self.emit("}")

        def mmas():
            for d in cl.dots:
                col, N = acc_cols[d.acc]
                ops = {}
                for role, node, name in (("A", d.a, d.a_name), ("B", d.b, d.b_name)):
                    if name in cl.loads:
                        sv = self._smem_val(D.f16, plans[name].shape,
                                            SmemOperand(plans[name], f"{ring} + st * {stage} + {offs[name]}"))
                    else:
                        sv = self.env[name]
                    ops[role] = sv
                K = ops["A"].shape[1]
                a_mn = self._operand_desc(ops["A"], "A", 0)[1]
                b_mn = self._operand_desc(ops["B"], "B", 0)[1]
                idesc = f"tila::idesc_f16_f32(128, {N}, {a_mn}, {b_mn})"
                for kk in range(K // 16):
                    da, _ = self._operand_desc(ops["A"], "A", kk)
                    db, _ = self._operand_desc(ops["B"], "B", kk)
                    self.emit(f"tila::mma_f16_ss(tila_tmem + {col}, {da}, {db}, {idesc}, 1u);")
            self.emit(f"tila::mma_commit({empty('st')});")

        if self.T >= 64:
            # copy producer (thread 32) refills a stage as soon as its MMAs have
            # completed; the MMA issuer (thread 0) never waits on a refill
            self.emit("if (tid == 32) {")
            self.indent += 1
            self.emit("for (tila::i64 j = 0; j < cl_n; ++j) {")
            self.indent += 1
            self.emit(f"const int sj = (int)(j % {S});")
            self.emit(f"if (j >= {S}) tila::mbar_wait({empty('sj')}, (tila::u32)(((j / {S}) - 1) & 1), tila_err, __LINE__, &tila_dead);")
            issue("j", "sj")
            self.indent -= 1
            self.emit("}")
            self.indent -= 1
            self.emit("}")
            self.emit("if (tid == 0) {")
            self.indent += 1
            self.emit("for (tila::i64 i = 0; i < cl_n; ++i) {")
            self.indent += 1
            self.emit(f"const int st = (int)(i % {S});")
            self.emit(f"tila::mbar_wait({full('st')}, (tila::u32)((i / {S}) & 1), tila_err, __LINE__, &tila_dead);")
            self.emit("tila::tc_fence_after();")
            mmas()
            self.indent -= 1
            self.emit("}")
        else:
            self.emit("if (tid == 0) {")
            self.indent += 1
            self.emit(f"for (tila::i64 j = 0; j < cl_n && j < {S - 1}; ++j) {{")
            self.indent += 1
            issue("j", "j")
            self.indent -= 1
            self.emit("}")
            self.emit("for (tila::i64 i = 0; i < cl_n; ++i) {")
            self.indent += 1
            self.emit(f"const int st = (int)(i % {S});")
            self.emit(f"tila::mbar_wait({full('st')}, (tila::u32)((i / {S}) & 1), tila_err, __LINE__, &tila_dead);")
            self.emit("tila::tc_fence_after();")
            mmas()
            self.emit(f"const tila::i64 j = i + {S - 1};")
            self.emit("if (j < cl_n) {")
            self.indent += 1
            self.emit(f"const int sj = (int)(j % {S});")
            self.emit(f"if (j >= {S}) tila::mbar_wait({empty('sj')}, (tila::u32)(((j / {S}) - 1) & 1), tila_err, __LINE__, &tila_dead);")
            issue("j", "sj")
            self.indent -= 1
            self.emit("}")
            self.indent -= 1
            self.emit("}")
        self.emit(f"tila::mma_commit({accbar});")
        self.indent -= 1
        self.emit("}")
        self.emit(f"tila::mbar_wait({accbar}, 0u, tila_err, __LINE__, &tila_dead);")
        self.emit("tila::tc_fence_after();")
        self.indent -= 1
        self.emit("}")
        # every copy into the ring has been consumed by a completed MMA
        self._free_smem.append((ring, S * stage))
        from .emitter import Val
        for d in cl.dots:
            col, N = acc_cols[d.acc]
            self.env[d.acc] = Val("tmem", D.f32, (128, N), tmem_col=f"{col}")
        self.env.pop(var, None)

    def _scalar(self, dt, expr):
        from .emitter import Val
        return Val("scalar", dt, expr=expr)


# ---------------------------------------------------------------------------
# asynchronous accumulator loops
# ---------------------------------------------------------------------------

# Placeholders for the warpgroup hand-off of an asynchronous accumulator loop
# (filled in, or dropped, when the kernel is assembled): a warpgroup acquires
# the CUDA-core phase of its iteration once its synchronous dot has completed
# and releases it when it issues the accumulating dot.
WG_ACQUIRE = "/*@wg_acquire*/"
WG_RELEASE = "/*@wg_release*/"
# loops whose trip count depends on program_id(0): "WG_TRIPS k" before the
# loop (exchange of the two programs' trip counts), "WG_TURNS k" after it (the
# program with fewer iterations takes the partner's remaining hand-off turns)
WG_TRIPS = "/*@wg_trips*/"
WG_TURNS = "/*@wg_turns*/"


@dataclass
class AsyncCtx:
    """Code-generation state of one asynchronous accumulator loop."""
    loop: object
    var: str
    stepv: int
    end: str
    loads: dict          # name -> dict(plan, node, base, bar, phase, flag)
    accs: dict           # name -> dict(col, N, bar, phase, pend, releases)
    p_col: str = "tila_tmem_scratch_col"


class AsyncLoopMixin:

    def try_async_loop_setup(self, s, start, end, stepv, carried):
        from .pipeline import match_async_loop
        if stepv <= 0:
            return None

        def is_tma(ld):
            plan = self.tma_plan(ld)
            return plan is not None and plan.outer_extent >= 64

        def is_smem(name):
            v = self.env.get(name)
            return v is not None and v.kind == "smem"

        def acc_ok(dot):
            dt, shape, _ = self.vt_info(dot.vt)
            return (dt.name == "f32" and len(shape) == 2 and shape[0] == 128 and
                    shape[1] % 16 == 0 and 16 <= shape[1] <= 256)
        def is_cast_tma(ld):
            plan = self.tma_plan(ld, cast=True)
            return plan is not None and plan.inner == 1 and plan.shape[0] == 128
        al = match_async_loop(s, self.pdefs, is_tma, is_smem, carried, acc_ok, is_cast_tma)
        if al is None:
            return None
        if self._ws is not None:
            return self.ws_loop_setup(s, start, end, stepv, al)
        # B operands must be laid out for an N that the instruction accepts
        for name, dot in al.accs.items():
            _, (M, N), _ = self.vt_info(dot.vt)
            bplan = self.tma_plan(al.loads[dot.b.name])
            if bplan.shape[1] != N:
                return None
        self.uses_mma = True
        self.uses_tmem = True
        ctx = AsyncCtx(al, s.var, stepv, f"(tila::i64)({end.expr})", {}, {})
        ctx.body = s.body
        ctx.cast_loads = set(al.cast_loads)
        ctx.p_early_after = self._early_p_points(s.body, al)
        ctx.p_early = False
        for name, ld in al.loads.items():
            plan = self.tma_plan(ld, cast=name in al.cast_loads)
            size = plan.nbox * max(plan.outer_extent, 128) * 128
            base = self._reuse_smem(size)
            bar_off = self.smem.alloc(8, 8)
            ctx.loads[name] = dict(plan=plan, node=ld, base=str(base),
                                   bar=f"reinterpret_cast<tila::u64*>(tila_smem + {bar_off})",
                                   bar_off=bar_off,
                                   phase=self._tma_state_var(f"tila_ph_{bar_off}"),
                                   flag=self._tma_state_var(f"tila_w_{bar_off}"))
        for name, dot in al.accs.items():
            _, (M, N), _ = self.vt_info(dot.vt)
            pre = self.env.get(name)
            if pre is not None and pre.kind == "tmem" and (str(pre.tmem_col), N) in self._loop_acc_cols:
                # the accumulator of an earlier loop continues in place
                col = int(pre.tmem_col)
            else:
                col = self.tmem_alloc_cols(N)
                self._loop_acc_cols.add((str(col), N))
            bar_off = self.smem.alloc(8, 8)
            releases = [op.name for op in (dot.a, dot.b)
                        if isinstance(op, T_.TName) and op.name in al.loads]
            ctx.accs[name] = dict(col=col, N=N, bar_off=bar_off,
                                  bar=f"reinterpret_cast<tila::u64*>(tila_smem + {bar_off})",
                                  phase=self._tma_state_var(f"tila_ph_{bar_off}"),
                                  pend=self._tma_state_var(f"tila_p_{bar_off}"),
                                  releases=releases, dot=dot)
        # TS operands (register P) live in the dot scratch columns
        for name, dot in al.accs.items():
            if isinstance(dot.a, T_.TCast):
                K = self.vt_info(dot.a.vt)[1][1]
                self.tmem_scratch_need = max(self.tmem_scratch_need, K // 2)
        # prologue: accumulators into TMEM, barriers, first copies
        from .emitter import Val
        for name, a in ctx.accs.items():
            pre = self.env[name]
            lay = TmemRows((128, a["N"]), self.T)
            if pre.kind == "tmem" and str(pre.tmem_col) == str(a["col"]):
                continue
            if pre.kind == "tmem":
                pre = self.tmem_to_reg(pre)
            if pre.dt.name != "f32":
                pre = self.coerce(pre, D.f32)
            if pre.kind == "scalar":
                pre = self.materialize_elementwise(D.f32, (128, a["N"]), [pre], lambda e: e[0], layout=lay)
            pre = self.materialize(pre, lay)
            self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {a['col']}"
                      + (f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else "")
                      + f" + ((tid & 96u) << 16), {pre.name});")
        self.emit(f"// asynchronous accumulator loop over {s.var}: TMEM accumulators "
                  f"{', '.join(ctx.accs)}; copies one iteration ahead: {', '.join(ctx.loads)}")
        inits = " ".join(f"tila::mbar_init({x['bar']}, 1);" for x in list(ctx.loads.values()) + list(ctx.accs.values()))
        self.emit(f"if (tid == 0) {{ {inits} tila::mbar_fence_init(); }}")
        for x in ctx.loads.values():
            self.emit(f"{x['phase']} = 0u; {x['flag']} = 1u;")
        for x in ctx.accs.values():
            self.emit(f"{x['phase']} = 0u; {x['pend']} = 0u;")
        self.emit("tila::tc_fence_before();")
        self.emit("__syncthreads();")
        self.emit("tila::tc_fence_after();")
        self.emit(f"if ((tila::i64)({start.expr}) < {ctx.end}) {{")
        self.indent += 1
        self._emit_loop_copies(ctx, list(ctx.loads), f"(tila::i64)({start.expr})")
        self.indent -= 1
        self.emit("}")
        for name, a in ctx.accs.items():
            v = Val("tmem", D.f32, (128, a["N"]), tmem_col=str(a["col"]))
            self.env[name] = v
        ctx.pingpong = self._pingpong_ok(s, start, al)
        ctx.turns = None
        if ctx.pingpong:
            self._wg_candidate = True
            if any(node is not None and not self._pid0_free(node) for node in (s.start, s.end)):
                # the partner program may run a different number of iterations:
                # exchange trip counts, and let the shorter one take its
                # remaining hand-off turns after its loop (see WG_TRIPS)
                k = self._uneven_loops
                self._uneven_loops += 1
                ctx.turns = k
                self.emit(f"const tila::i64 tila_trip_{k} = ((tila::i64)({end.expr}) > (tila::i64)({start.expr})) ? "
                          f"((tila::i64)({end.expr}) - (tila::i64)({start.expr}) + {stepv - 1}) / {stepv} : 0;")
                self.emit(f"{WG_TRIPS} {k}")
        self.ws_detect(s, start, end, stepv, al, ctx)
        self.actx = ctx
        return ctx

    def _early_p_points(self, body, al):
        """{id(statement): (acc name, register tile name)}: for an accumulating
        dot whose A operand is cast[f16](R) of a register tile R, the last
        statement of the loop body before the dot that mentions R.  P is
        packed and stored into tensor memory right after it, so R's
        registers are free for the rest of the iteration (the dot then only
        issues the MMAs)."""
        points = {}
        for name, dot in al.accs.items():
            if not (isinstance(dot.a, T_.TCast) and isinstance(dot.a.operand, T_.TName)):
                continue
            r = dot.a.operand.name
            if r in al.loads:
                continue
            d = next((i for i, st in enumerate(body)
                      if isinstance(st, T_.TAssign) and st.value is dot), None)
            if d is None:
                continue

            def mentions(node, found=None):
                found = found if found is not None else [False]
                if isinstance(node, T_.TName) and node.name == r:
                    found[0] = True
                if isinstance(node, T_.TAssign) and node.name == r:
                    found[0] = True
                if dataclasses.is_dataclass(node):
                    for f in dataclasses.fields(node):
                        if f.name in ("vt", "definition", "effect"):
                            continue
                        v = getattr(node, f.name)
                        for x in (v if isinstance(v, list) else [v]):
                            if dataclasses.is_dataclass(x):
                                mentions(x, found)
                return found[0]
            k = max((i for i in range(d) if mentions(body[i])), default=None)
            if k is None or not (isinstance(body[k], T_.TAssign) or any(
                    isinstance(body[i], T_.TAssign) and body[i].name == r for i in range(k))):
                continue
            points[id(body[k])] = (name, r)
        return points

    def emit_early_p(self, st):
        """Called after each statement of an asynchronous loop body."""
        ctx = self.actx
        if ctx is None or id(st) not in getattr(ctx, "p_early_after", {}):
            return
        name, r = ctx.p_early_after[id(st)]
        v = self.env.get(r)
        if v is None or v.kind not in ("reg", "func", "tmem"):
            return
        self.wait_all_accs(release=True)
        self._store_p(v, ctx)
        ctx.p_early = True

    def _store_p(self, pv, ctx):
        """cast[f16](R): round and pack pairs from R and store them into the
        P columns of tensor memory (one cvt per pair)."""
        K = pv.shape[1]
        play = TmemRows((128, K), self.T)
        if pv.dt.name not in ("f32", "f16"):
            pv = self.coerce(pv, D.f32)
        pv = self.materialize(pv, play) if not (pv.kind == "reg" and pv.layout == play) else pv
        half = play.nreg // 2
        self.emit("{")
        self.indent += 1
        self.emit(f"float pk[{half}];")
        self.emit("#pragma unroll")
        self.emit(f"for (int c = 0; c < {half}; ++c) pk[c] = __uint_as_float(tila::pack_f16x2({pv.name}[2 * c], {pv.name}[2 * c + 1]));")
        goff = f" + (tid >> 7) * {play.cpg // 2}" if play.groups > 1 else ""
        # no store wait here: the P@V issue below waits once for every TMEM
        # store of the iteration (P and the accumulator rescale)
        self.emit(f"tila::tmem_store_row_async<{half}>(tila_tmem + {ctx.p_col}{goff} + ((tid & 96u) << 16), pk);")
        self.indent -= 1
        self.emit("}")

    def _reuse_smem(self, size):
        """1024-aligned shared memory for a loop buffer: part of a region a
        finished pipelined loop released, else a new allocation."""
        for i, (off, n) in enumerate(self._free_smem):
            if n >= size:
                self._free_smem[i] = (off + size, n - size)
                return off
        return self.smem.alloc(size, 1024)

    def _pingpong_ok(self, s, start, al, any_T=False):
        """Two programs of grid axis 0 may share a CTA, one per warpgroup,
        handing the CUDA-core phase of each iteration back and forth, when
        both are sure to run the same iterations: the loop is a top-level
        statement of a kernel without early returns, its bounds do not depend
        on program_id(0), and each iteration has exactly one synchronous and
        one accumulating dot."""
        from .pipeline import _walk
        if (self.T != 128 and not any_T) or id(s) not in {id(st) for st in self.tk.body}:
            return False
        has_return = [False]
        for st in self.tk.body:
            _walk(st, lambda n: has_return.__setitem__(0, has_return[0] or isinstance(n, T_.TReturn)))
        if has_return[0] or len(al.accs) != 1:
            return False
        # bounds that depend on program_id(0) are allowed (the two programs then
        # run different trip counts; see the token turns in generate())
        if s.step is not None and not self._pid0_free(s.step):
            return False
        dots = []
        for st in s.body:
            _walk(st, lambda n: dots.append(n) if isinstance(n, T_.TDot) else None)
        acc_dots = {id(d) for d in al.accs.values()}
        return len(dots) == 2 and sum(1 for d in dots if id(d) not in acc_dots) == 1

    def _pid0_free(self, node, depth=0):
        """``node`` provably has the same value in every program of grid axis 0."""
        from .pipeline import _walk
        if depth > 32:
            return False
        ok = [True]
        uni = set(self.scalar_params)

        def chk(n):
            if isinstance(n, T_.TPid) and n.axis == 0:
                ok[0] = False
            elif isinstance(n, T_.TName) and n.name not in uni and n.name not in self.consts:
                d = self.pdefs.resolve(n)
                if d is n or not self._pid0_free(d, depth + 1):
                    ok[0] = False
        _walk(node, chk)
        return ok[0]

    def _functional_prefix(self, ctx, loop_value):
        """Bind the loop variable to ``loop_value`` and evaluate the body's
        pure index assignments: no loads, dots, reductions or transcendental
        math, and reading only the loop variable, Consts, scalars, names set
        before the loop and earlier pure assignments."""
        from .emitter import Val
        from .pipeline import _walk
        assigned = {st.name for st in ctx.body if isinstance(st, T_.TAssign)}
        pure_names = set()

        def pure(node):
            ok = [True]

            def chk(n):
                if isinstance(n, (T_.TLoad, T_.TDot, T_.TReduce, T_.TAtomicAdd)) or \
                        (isinstance(n, T_.TUna) and n.op in ("exp", "exp2")):
                    ok[0] = False
                elif isinstance(n, T_.TName) and n.name != ctx.var and n.name in assigned \
                        and n.name not in pure_names:
                    ok[0] = False
            _walk(node, chk)
            return ok[0]
        self.env[ctx.var] = Val("scalar", D.i32, expr=f"((tila::i32)({loop_value}))")
        saved_mode, self._guard_mode = self._guard_mode, None
        for st in ctx.body:
            if isinstance(st, T_.TAssign) and st.name not in ctx.loads and st.name not in ctx.accs \
                    and st.name not in pure_names and pure(st.value):
                self.env[st.name] = self.value(st.value)
                pure_names.add(st.name)
        self._guard_mode = saved_mode

    def _emit_loop_copies(self, ctx, names, iter_value):
        """tid 0 issues the TMA copies of ``names`` for loop value ``iter_value``;
        every thread marks them not yet waited for."""
        if not names or getattr(ctx, "ws", False):
            return
        saved = dict(self.env)
        self.emit("{")
        self.indent += 1
        lv = self.fresh(f"s_{ctx.var}")
        self.emit(f"const tila::i32 {lv} = (tila::i32)({iter_value});")
        self._functional_prefix(ctx, lv)
        for n in names:
            self.emit(f"{ctx.loads[n]['flag']} = 0u;")
        self.emit("if (tid == 0) {")
        self.indent += 1
        for n in names:
            x = ctx.loads[n]
            coords = [self.value(c) for c in x["node"].coords]
            self.emit(f"tila::mbar_arrive_expect_tx({x['bar']}, {x['plan'].bytes}u);")
            self._emit_tma(x["plan"], self._tma_coords(x["plan"], coords), x["base"], x["bar"])
        self.indent -= 1
        self.emit("}")
        self.indent -= 1
        self.emit("}")
        self.env = saved

    def load_smem_val(self, ctx, name):
        x = ctx.loads[name]
        dt, shape, _ = self.vt_info(x["node"].vt)
        return self._smem_val(dt, shape, SmemOperand(x["plan"], x["base"], x["bar"], x["phase"], x["flag"]))

    def emit_acc_wait(self, name, release=True):
        ctx = self.actx
        a = ctx.accs[name]
        self.emit(f"if ({a['pend']}) {{")
        self.indent += 1
        self.emit(f"tila::mbar_wait({a['bar']}, {a['phase']}, tila_err, __LINE__, &tila_dead);")
        self.emit(f"{a['phase']} ^= 1u; {a['pend']} = 0u;")
        self.emit("tila::tc_fence_after();")
        if release and a["releases"]:
            # the MMA that read these buffers is done: copy the current iteration's tiles
            cur = self.env[ctx.var].expr
            self._emit_loop_copies(ctx, a["releases"], f"(tila::i64)({cur})")
        self.indent -= 1
        self.emit("}")

    def wait_all_accs(self, release=True):
        if self.actx is None:
            return
        for name in self.actx.accs:
            self.emit_acc_wait(name, release)

    def release_after_sync_dot(self, operands):
        """A synchronous dot completed: copy the next iteration's tiles of its
        in-loop TMA operands into the freed buffers."""
        ctx = self.actx
        if ctx is None:
            return
        names = [v.smem_name for v in operands if getattr(v, "smem_name", None) in ctx.loads]
        if not names:
            return
        cur = self.env[ctx.var].expr
        nxt = f"((tila::i64)({cur}) + {ctx.stepv})"
        self.emit(f"if ({nxt} < {ctx.end}) {{")
        self.indent += 1
        self._emit_loop_copies(ctx, names, nxt)
        self.indent -= 1
        self.emit("}")

    def emit_async_acc_dot(self, x, name):
        """acc = dot(a, b, acc=acc) with acc in TMEM: issue and leave pending."""
        from .emitter import Val
        ctx = self.actx
        if getattr(ctx, "ws", False):
            return self.ws_acc_dot(x, name)
        a = ctx.accs[name]
        N = a["N"]
        # the previous accumulation and any TS operand reader must be finished
        self.wait_all_accs(release=True)
        acc = self.env[name]
        lay = TmemRows((128, N), self.T)
        if acc.kind != "tmem":
            accv = acc if acc.dt.name == "f32" else self.coerce(acc, D.f32)
            accv = self.materialize(accv, lay) if not (accv.kind == "reg" and accv.layout == lay) else accv
            self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {a['col']}"
                      + (f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else "")
                      + f" + ((tid & 96u) << 16), {accv.name});")
        bv = self.value(x.b)
        K = bv.shape[0]
        ts = isinstance(x.a, T_.TCast)
        cast_src = None
        if ts and ctx.p_early:
            # P was packed into tensor memory right after its last other use
            ctx.p_early = False
            adesc = None
        elif ts:
            # cast[f16](R): round and pack pairs straight from R (one cvt per pair)
            pv = self.value(x.a.operand)
            play = TmemRows((128, K), self.T)
            if pv.kind == "smem":
                cast_src = getattr(pv, "smem_name", None)
                pv = self.smem_rows_to_reg(pv, play)
            self._store_p(pv, ctx)
            adesc = None
        else:
            av = self.value(x.a)
            if av.kind != "smem":
                self.fail("asynchronous dot needs its A operand in shared or tensor memory")
        self.emit_smem_wait(bv)
        if not ts:
            self.emit_smem_wait(av)
        else:
            self.emit("tila::tmem_wait_st();")
        self.emit("tila::fence_proxy_async_smem();")
        self.emit("tila::tc_fence_before();")
        self.emit("__syncthreads();")
        self.emit("tila::tc_fence_after();")
        if getattr(ctx, "pingpong", False):
            self.emit(WG_RELEASE)
        if cast_src is not None and cast_src in ctx.cast_loads:
            # every thread has read the tile into registers: copy the next one
            cur = self.env[ctx.var].expr
            nxt = f"((tila::i64)({cur}) + {ctx.stepv})"
            self.emit(f"if ({nxt} < {ctx.end}) {{")
            self.indent += 1
            self._emit_loop_copies(ctx, [cast_src], nxt)
            self.indent -= 1
            self.emit("}")
        b_mn = self._operand_desc(bv, "B", 0)[1]
        self.emit("if (tid == 0) {")
        self.indent += 1
        for kk in range(K // 16):
            db, _ = self._operand_desc(bv, "B", kk)
            if ts:
                idesc = f"tila::idesc_f16_f32(128, {N}, 0, {b_mn})"
                self.emit(f"tila::mma_f16_ts(tila_tmem + {a['col']}, tila_tmem + {ctx.p_col} + {kk * 8}, {db}, {idesc}, 1u);")
            else:
                da, a_mn = self._operand_desc(av, "A", kk)
                idesc = f"tila::idesc_f16_f32(128, {N}, {a_mn}, {b_mn})"
                self.emit(f"tila::mma_f16_ss(tila_tmem + {a['col']}, {da}, {db}, {idesc}, 1u);")
        self.emit(f"tila::mma_commit({a['bar']});")
        self.indent -= 1
        self.emit("}")
        self.emit(f"{a['pend']} = 1u;")
        if getattr(ctx, "s_issue", None):
            # issue the next iteration's synchronous dot now: the tensor pipe
            # executes it right after this accumulation (in issue order; it
            # overwrites the TMEM columns this accumulation reads only after
            # that MMA has consumed them)
            cur = self.env[ctx.var].expr
            nxt = f"((tila::i64)({cur}) + {ctx.stepv})"
            self.emit(f"if ({nxt} < {ctx.end}) {{")
            self.indent += 1
            for op in ctx.s_operands:
                self.emit_smem_wait(op)
            for line in ctx.s_issue:
                self.emit(line)
            self.emit(f"{self._s_pre_var()} = 1u;")
            self.indent -= 1
            self.emit("}")
        v = Val("tmem", D.f32, (128, N), tmem_col=str(a["col"]))
        v.pending = name
        return v

    def _s_pre_var(self):
        return self._tma_state_var("tila_s_pre")

    def tmem_update_in_place(self, name, node):
        """acc = acc <op> rowvec (or scalar): update the TMEM accumulator in
        32-column chunks instead of materialising the whole tile."""
        if not isinstance(node, T_.TBin) or node.op not in ("*", "+", "-", "/"):
            return False
        l, r = node.left, node.right
        if isinstance(l, T_.TName) and l.name == name:
            other_node, acc_left = r, True
        elif isinstance(r, T_.TName) and r.name == name:
            other_node, acc_left = l, False
        else:
            return False
        a = self.actx.accs[name]
        N = a["N"]
        dt, shape, _ = self.vt_info(node.vt)
        if dt.name != "f32" or tuple(shape) != (128, N):
            return False
        other = self.value(other_node)
        if other.kind == "tmem" or other.kind == "smem":
            return False
        if other.shape and other.shape[-1] != 1:
            return False
        if other.dt.name != "f32":
            other = self.coerce(other, D.f32)
        lay = TmemRows((128, N), self.T)
        if other.kind == "reg":
            m = self.slot_map(other.layout, lay, (128, N))
            if m is None:
                other = self.convert(other, lay, (128, N))
                m = self.slot_map(other.layout, lay, (128, N))
            if len(set(m)) != 1:
                return False
            oexpr = f"{other.name}[{m[0]}]"
        elif other.kind == "func":
            oexpr = other.fn(("((tid & 127))", "0") if len(other.shape) == 2 else ("0",))
        else:
            oexpr = other.expr
        mk = self._bin_maker(node.op, D.f32, D.f32)
        self.wait_all_accs(release=True)
        chunk = 32 if lay.cpg % 32 == 0 else 8
        base = f"tila_tmem + {a['col']}" + (f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else "") + " + ((tid & 96u) << 16)"
        if chunk == 32 and lay.cpg >= 64 and getattr(mk, "fn", None):
            # software-pipelined: the next chunk's load is in flight while this
            # chunk is scaled and stored; one wait for the stores at the end
            nch = lay.cpg // 32
            xt, xo = ("tila::pk2(t_[c & 1][j], t_[c & 1][j + 1])", "tila::pk2(o_, o_)")
            args = f"{xt}, {xo}" if acc_left else f"{xo}, {xt}"
            self.emit("{ // in-place TMEM update of " + name + " (loads one chunk ahead)")
            self.indent += 1
            self.emit(f"const float o_ = {oexpr};")
            self.emit("float t_[2][32];")
            self.emit(f"tila::tmem_ld32({base}, t_[0]);")
            self.emit("tila::tmem_wait_ld();")
            self.emit("#pragma unroll")
            self.emit(f"for (int c = 0; c < {nch}; ++c) {{")
            self.indent += 1
            self.emit(f"if (c + 1 < {nch}) tila::tmem_ld32({base} + (c + 1) * 32, t_[(c + 1) & 1]);")
            self.emit("#pragma unroll")
            self.emit(f"for (int j = 0; j < 32; j += 2) {{ const tila::u64 q_ = tila::{mk.fn}({args}); "
                      f"t_[c & 1][j] = tila::lo2(q_); t_[c & 1][j + 1] = tila::hi2(q_); }}")
            self.emit(f"tila::tmem_st32({base} + c * 32, t_[c & 1]);")
            self.emit(f"if (c + 1 < {nch}) tila::tmem_wait_ld();")
            self.indent -= 1
            self.emit("}")
            self.emit("tila::tmem_wait_st();")
            self.indent -= 1
            self.emit("}")
            from .emitter import Val
            self.env[name] = Val("tmem", D.f32, (128, N), tmem_col=str(a["col"]))
            return True
        self.emit("{ // in-place TMEM update of " + name)
        self.indent += 1
        self.emit(f"const float o_ = {oexpr};")
        self.emit(f"for (int ch = 0; ch < {lay.cpg}; ch += {chunk}) {{")
        self.indent += 1
        self.emit(f"float t_[{chunk}];")
        self.emit(f"tila::tmem_load_row<{chunk}>({base} + ch, t_);")
        self.emit("#pragma unroll")
        if getattr(mk, "fn", None) and chunk % 2 == 0:
            # two columns per f32x2 instruction
            xt, xo = ("tila::pk2(t_[j], t_[j + 1])", "tila::pk2(o_, o_)")
            args = f"{xt}, {xo}" if acc_left else f"{xo}, {xt}"
            self.emit(f"for (int j = 0; j < {chunk}; j += 2) {{ const tila::u64 q_ = tila::{mk.fn}({args}); "
                      f"t_[j] = tila::lo2(q_); t_[j + 1] = tila::hi2(q_); }}")
        else:
            e = mk(["t_[j]", "o_"] if acc_left else ["o_", "t_[j]"])
            self.emit(f"for (int j = 0; j < {chunk}; ++j) t_[j] = {e};")
        self.emit(f"tila::tmem_store_row<{chunk}>({base} + ch, t_);")
        self.indent -= 1
        self.emit("}")
        self.indent -= 1
        self.emit("}")
        from .emitter import Val
        self.env[name] = Val("tmem", D.f32, (128, N), tmem_col=str(a["col"]))
        return True

    def finish_async_loop(self, ctx):
        from .emitter import Val
        if getattr(ctx, "turns", None) is not None:
            self.emit(f"{WG_TURNS} {ctx.turns}")
        for name in ctx.accs:
            self.emit_acc_wait(name, release=False)
        if getattr(ctx, "ws", False):
            self.ws_finish(ctx)
        # all loop copies were consumed (the last iteration issues none)
        spans = [(int(x["base"]), x["plan"].nbox * max(x["plan"].outer_extent, 128) * 128)
                 for x in ctx.loads.values() if x["base"] is not None]
        if spans:
            lo = min(b for b, _ in spans)
            hi = max(b + n for b, n in spans)
            self._free_smem.append((lo, hi - lo))
        for name, a in ctx.accs.items():
            self.env[name] = Val("tmem", D.f32, (128, a["N"]), tmem_col=str(a["col"]))
        self.actx = None
