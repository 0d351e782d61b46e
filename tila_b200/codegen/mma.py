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

    def tma_plan(self, load):
        key = id(load)
        if key in self.tma_plans:
            return self.tma_plans[key]
        plan = None
        if load.buffer is not None and load.buffer in self.buffer_params:
            dt, shape, _ = self.vt_info(load.vt)
            plan = plan_tma(load, shape, self.pdefs, self.consts, self._uniform_names(),
                            self.buffer_params[load.buffer], self.buffers.get(load.buffer))
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
                                     "dtype": "f16"})
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
                cs[0] = f"({cs[0]} + {64 * b})"
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
        return self._smem_val(dt, shape, SmemOperand(plan, str(off), bar, phase, flag))

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
            return (f"tila::smem_desc(tila::smem_u32(tila_smem + {off}), 16, 1024, 2)", 0)
        off = f"{op.base} + {k0 * 128}"
        return (f"tila::smem_desc(tila::smem_u32(tila_smem + {off}), {plan.box_bytes}, 1024, 2)", 1)

    # -- dot ----------------------------------------------------------------------------

    def tmem_alloc_cols(self, n):
        col = self.tmem_next
        self.tmem_next += n
        return col

    def e_TDot(self, x):
        dt, shape, _ = self.vt_info(x.vt)
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
            descs["A"] = lambda kk, o=a_off: (f"tila::smem_desc(tila::smem_u32(tila_smem + {o}) + {kk} * 256, 128, {K * 16}, 0)", 0)
        else:
            descs["A"] = lambda kk, v=a: self._operand_desc(v, "A", kk)
        if b.kind != "smem":
            b_off = self.smem.alloc(Npad * K * 2, 1024)
            self._stage_operand(b, b_off, K, transpose=True)
            descs["B"] = lambda kk, o=b_off: (f"tila::smem_desc(tila::smem_u32(tila_smem + {o}) + {kk} * 256, 128, {K * 16}, 0)", 0)
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
        self.emit("tila::mbar_wait(tila_mma_bar, tila_mma_phase, tila_err, __LINE__, &tila_dead);")
        self.emit("tila_mma_phase ^= 1u;")
        self.emit("tila::tc_fence_after();")
        from .emitter import Val
        res = Val("tmem", D.f32, (M, N), tmem_col=col)
        reg = self.tmem_to_reg(res)
        if dt.name == "f16":
            reg = self.materialize_elementwise(dt, (M, N), [reg], lambda e: f"tila::round_f16({e[0]})",
                                               layout=reg.layout)
        self.emit("tila::tc_fence_before();")
        return reg

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
        self.emit("if (tid == 0) {")
        self.indent += 1

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
        from .emitter import Val
        for d in cl.dots:
            col, N = acc_cols[d.acc]
            self.env[d.acc] = Val("tmem", D.f32, (128, N), tmem_col=f"{col}")
        self.env.pop(var, None)

    def _scalar(self, dt, expr):
        from .emitter import Val
        return Val("scalar", dt, expr=expr)
