"""CTA coarsening of contraction kernels: one CTA runs a block of programs.

Tila programs are independent instances of the kernel body, so a CTA may run
several of them.  For kernels of the form

    <index math>;  for k: acc = dot(load_a, load_b, acc=acc);  <epilogue>

where the A tile depends on one program axis and the B tile on another
(matmul: A on the row-tile axis, B on the column-tile axis), running a 2 x 2
block of programs in one CTA loads every A tile once for the two programs
that share it and every B tile once for the two programs that share it.
That halves the L2 -> shared-memory operand traffic, which is what bounds a
128 x 128 tile on B200, and lets two adjacent MN-major B tiles form one
N = 256 MMA.  Results are those of the individual programs: each program's
accumulator lives in its own 128 TMEM columns and its epilogue runs with its
own ``program_id`` values; programs beyond the launched grid store nothing.
"""

from __future__ import annotations

from .._reference import tila
from .layouts import TmemRows
from .pipeline import _walk, canon, match_contraction_loop

T_ = tila.tir
D = tila.dtypes

FUSE = 2     # programs per CTA along each of the two fused axes


def _pure_index(node):
    ok = [True]

    def chk(n):
        if isinstance(n, (T_.TLoad, T_.TDot, T_.TReduce, T_.TAtomicAdd)) or \
                (isinstance(n, T_.TUna) and n.op in ("exp", "exp2")):
            ok[0] = False
    _walk(node, chk)
    return ok[0]


def _pid_axes(text):
    return {ax for ax in range(3) if f"pid{ax}" in text}


class FusedContractionMixin:

    def try_fused_kernel(self):
        """Emit the whole kernel body as a 2 x 2 block of programs per CTA
        when the kernel is a single pipelined contraction; False otherwise."""
        body = self.tk.body
        if self.T < 64:      # thread 32 is the copy producer
            return False
        loops = [i for i, s in enumerate(body) if isinstance(s, T_.TFor)]
        if len(loops) != 1:
            return False
        li = loops[0]
        loop, prefix, suffix = body[li], body[:li], body[li + 1:]
        if any(not isinstance(s, T_.TAssign) or not _pure_index(s.value) for s in prefix):
            return False
        for s in suffix:
            bad = [isinstance(s, (T_.TFor, T_.TIf, T_.TReturn))]

            def chk(n):
                if isinstance(n, (T_.TDot, T_.TFor, T_.TAtomicAdd, T_.TAtomicStmt)):
                    bad[0] = True
            _walk(s, chk)
            if bad[0]:
                return False
        for part in (loop.start, loop.end, loop.step):
            if part is not None and _pid_axes(canon(part, self.pdefs)):
                return False
        # bind the prefix once to check that the loop is a plain contraction
        saved_env, saved_lines = dict(self.env), self.lines
        self.lines = []
        for s in prefix:
            self.s_TAssign(s)
        self._loopvars[loop.var] = 1
        carried = sorted(n for n in {s.name for s in loop.body if isinstance(s, T_.TAssign)}
                         if n in self.env)
        cl = match_contraction_loop(loop, self.pdefs, lambda ld: self.tma_plan(ld) is not None,
                                    lambda n: False, carried)
        self.env, self.lines = saved_env, saved_lines
        self._loopvars.pop(loop.var, None)
        if cl is None or len(cl.dots) != 1:
            return False
        d = cl.dots[0]
        if d.a_name not in cl.loads or d.b_name not in cl.loads:
            return False
        dt, (M, N), _ = self.vt_info(d.dot.vt)
        pa, pb = self.tma_plan(cl.loads[d.a_name]), self.tma_plan(cl.loads[d.b_name])
        if M != 128 or N != 128 or dt.name != "f32" or pa.shape[0] != 128 or pb.shape[1] != 128:
            return False
        if any(p.outer_extent > 256 for p in (pa, pb)):
            return False
        ya = set().union(*[_pid_axes(canon(c, self.pdefs)) for c in cl.loads[d.a_name].coords])
        xb = set().union(*[_pid_axes(canon(c, self.pdefs)) for c in cl.loads[d.b_name].coords])
        if len(ya) != 1 or len(xb) != 1 or ya == xb:
            return False
        ay, ax = ya.pop(), xb.pop()
        if ay == 2 or ax == 2:
            return False
        self._emit_fused(prefix, loop, suffix, cl, d, ay, ax, pa, pb, N)
        return True

    def _emit_fused(self, prefix, loop, suffix, cl, d, ay, ax, pa, pb, N):
        from .emitter import Val
        if self._streamk_ok(prefix, d, ay, ax):
            return self._emit_fused_streamk(prefix, loop, suffix, cl, d, ay, ax, pa, pb, N)
        fy = fx = FUSE
        self.fuse = {ay: fy, ax: fx}
        self.uses_mma = True
        self.uses_tmem = True
        inst = [(i, j) for i in range(fy) for j in range(fx)]
        for ax_, f in ((ay, fy), (ax, fx)):
            blk = "xyz"[ax_]
            for k in range(f):
                self.emit(f"const tila::i32 pid_{ax_}_{k} = (tila::i32)(blockIdx.{blk} * {f} + {k} + pid_off_{ax_});")
                self.emit(f"const bool live_{ax_}_{k} = (tila::i32)(blockIdx.{blk} * {f} + {k}) < launch_{ax_};")
        envs = {}
        base_env = dict(self.env)
        for (i, j) in inst:
            self.env = dict(base_env)
            self._pid_expr = {ay: f"pid_{ay}_{i}", ax: f"pid_{ax}_{j}"}
            for s in prefix:
                self.s_TAssign(s)
            envs[(i, j)] = dict(self.env)
        self._pid_expr = {}
        self.env = dict(envs[(0, 0)])
        start = self.value(loop.start) if loop.start is not None else Val("scalar", D.i64, expr="0", const=0)
        end = self.value(loop.end)
        stepv = int(self.value(loop.step).const)
        # shared-memory ring: A_0..A_{fy-1} then B_0..B_{fx-1} (B tiles adjacent)
        a_bytes = (pa.nbox * pa.box_bytes + 1023) // 1024 * 1024
        b_bytes = (pb.nbox * pb.box_bytes + 1023) // 1024 * 1024
        stage = fy * a_bytes + fx * b_bytes
        tx = fy * pa.bytes + fx * pb.bytes
        S = max(2, min(6, (200 * 1024) // stage))
        ring = self.smem.alloc(S * stage, 1024)
        bars = self.smem.alloc(8 * (2 * S + 1), 8)
        full = lambda e: f"reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * ({e}))"
        empty = lambda e: f"reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * ({S} + ({e})))"
        accbar = f"reinterpret_cast<tila::u64*>(tila_smem + {bars + 16 * S})"
        cols = {(i, j): self.tmem_alloc_cols(N) for (i, j) in inst}
        lay = TmemRows((128, N), self.T)
        for (i, j) in inst:
            self.env = dict(envs[(i, j)])
            pre = self.env[d.acc]
            if pre.dt.name != "f32":
                pre = self.coerce(pre, D.f32)
            if pre.kind == "scalar":
                pre = self.materialize_elementwise(D.f32, (128, N), [pre], lambda e: e[0], layout=lay)
            pre = self.materialize(pre, lay)
            self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {cols[(i, j)]} + ((tid & 96u) << 16), {pre.name});")
        self.emit(f"{{ // {fy}x{fx} programs per CTA: {S}-stage TMA ring, tcgen05.mma into TMEM")
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
        def issue(jexpr, st):
            self.emit("{")
            self.indent += 1
            lv = self.fresh(f"s_{loop.var}")
            self.emit(f"const tila::i32 {lv} = (tila::i32)(cl_start + ({jexpr}) * {stepv});")
            self.emit(f"tila::mbar_arrive_expect_tx({full(st)}, {tx}u);")
            for role, plan, nm, count, offset in (("A", pa, d.a_name, fy, 0), ("B", pb, d.b_name, fx, fy * a_bytes)):
                for k in range(count):
                    self.env = dict(envs[(k, 0)] if role == "A" else envs[(0, k)])
                    self.env[loop.var] = Val("scalar", D.i32, expr=lv)
                    for s2 in cl.functional:
                        self.s_TAssign(s2)
                    coords = [self.value(c) for c in cl.loads[nm].coords]
                    size = a_bytes if role == "A" else b_bytes
                    self._emit_tma(plan, self._tma_coords(plan, coords),
                                   f"{ring} + ({st}) * {stage} + {offset + k * size}", full(st))
            self.indent -= 1
            self.emit("}")

        # producer (thread 32): refills a stage as soon as the MMAs reading it
        # have completed, so copy latency is hidden behind all S stages
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
        # MMA issuer (thread 0)
        self.emit("if (tid == 0) {")
        self.indent += 1
        self.emit("for (tila::i64 i = 0; i < cl_n; ++i) {")
        self.indent += 1
        self.emit(f"const int st = (int)(i % {S});")
        self.emit(f"tila::mbar_wait({full('st')}, (tila::u32)((i / {S}) & 1), tila_err, __LINE__, &tila_dead);")
        self.emit("tila::tc_fence_after();")
        # adjacent MN-major B tiles form one operand of N = fx * 128
        merged = pb.inner == 1 and b_bytes == pb.nbox * pb.box_bytes
        K = pa.shape[1]
        for i in range(fy):
            a_val = self._smem_val(D.f16, pa.shape, self._smem_op(pa, f"{ring} + st * {stage} + {i * a_bytes}"))
            targets = [(0, fx)] if merged else [(j, 1) for j in range(fx)]
            for j0, nb in targets:
                b_val = self._smem_val(D.f16, (pb.shape[0], 128 * nb),
                                       self._smem_op(pb, f"{ring} + st * {stage} + {fy * a_bytes + j0 * b_bytes}"))
                for kk in range(K // 16):
                    da, a_mn = self._operand_desc(a_val, "A", kk)
                    db, b_mn = self._operand_desc(b_val, "B", kk)
                    idesc = f"tila::idesc_f16_f32(128, {128 * nb}, {a_mn}, {b_mn})"
                    self.emit(f"tila::mma_f16_ss(tila_tmem + {cols[(i, j0)]}, {da}, {db}, {idesc}, 1u);")
        self.emit(f"tila::mma_commit({empty('st')});")
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
        # epilogues, one program at a time (uniform branches: `live` depends on
        # blockIdx).  TMA stores rotate through staging slots in the freed
        # ring; a program that does not run commits the same number of (empty)
        # bulk groups, so that group k always belongs to store k.
        self._store_ring = {"base": ring, "bytes": S * stage, "size": None, "next": 0}
        for (i, j) in inst:
            self.env = dict(envs[(i, j)])
            self._pid_expr = {ay: f"pid_{ay}_{i}", ax: f"pid_{ax}_{j}"}
            self.env[d.acc] = Val("tmem", D.f32, (128, N), tmem_col=str(cols[(i, j)]))
            self.emit(f"if (live_{ay}_{i} && live_{ax}_{j}) {{")
            self.indent += 1
            self.conv_cache = {}
            before = self._store_ring["next"]
            self.stmts(suffix)
            used = self._store_ring["next"] - before
            self.indent -= 1
            if used:
                self.emit("} else if (tid == 0) {")
                self.emit("  " + " ".join(["tila::bulk_commit();"] * used))
            self.emit("}")
        if self._store_ring["next"]:
            self.emit("if (tid == 0) tila::bulk_wait_read();   // staging reads done before exit")
        self._store_ring = None
        self._pid_expr = {}

    # -- balanced split of the K loops over persistent CTAs (stream-K) ------------

    def _streamk_ok(self, prefix, d, ay, ax):
        """The persistent form (opt-in: TILA_B200_STREAMK=1) needs a
        zero-initialised accumulator (every piece starts it with a
        non-accumulating MMA) and the two fused axes 0 and 1.  It is off by
        default: at 4096^3 it measured 132 us against 108 us for one CTA per
        tile (each piece drains the operand ring and runs its epilogue
        before the next starts, about three times per CTA, which costs more
        than the even split recovers from the partial last wave)."""
        import os
        if os.environ.get("TILA_B200_STREAMK", "0") != "1" or {ay, ax} != {0, 1}:
            return False
        init = [st for st in prefix if isinstance(st, T_.TAssign) and st.name == d.acc]
        return bool(init) and isinstance(init[-1].value, T_.TZeros)

    def _emit_fused_streamk(self, prefix, loop, suffix, cl, d, ay, ax, pa, pb, N):
        """The 2 x 2 contraction as a persistent kernel over units (tile, K
        step), where a tile is one CTA's 2 x 2 block of programs.  The host
        launches P CTAs along x (axis 2 of the program grid stays on z); CTA
        b takes units [total b / P, total (b + 1) / P).  With P = #SMs and
        more tiles than SMs every CTA runs the same number of K steps (the
        last wave of whole tiles otherwise leaves SMs idle), and each range
        is at least one tile long, so a CTA's pieces are: the high-K part of
        a tile (its first piece), whole tiles, the low-K part of a tile (its
        last piece).  The high-K part is computed first by CTA b + 1, which
        parks its accumulators in the workspace slot of CTA b + 1 and
        releases that slot's flag; CTA b, which reaches the tile's low-K part
        at the end of its range, waits for the flag, adds the parked values
        and runs the program's own epilogue, then clears the flag for the
        next launch.  Sums over K are split in two at most, so results agree
        with the unsplit kernel within the accumulation's rounding; with
        P = #tiles (not more tiles than SMs) there is no split at all."""
        from .emitter import Val
        fy = fx = FUSE
        self.fuse = {ay: fy, ax: fx}
        self.persistent = True
        self.uses_mma = True
        self.uses_tmem = True
        inst = [(i, j) for i in range(fy) for j in range(fx)]
        base_env = dict(self.env)
        start = self.value(loop.start) if loop.start is not None else Val("scalar", D.i64, expr="0", const=0)
        end = self.value(loop.end)
        stepv = int(self.value(loop.step).const)
        a_bytes = (pa.nbox * pa.box_bytes + 1023) // 1024 * 1024
        b_bytes = (pb.nbox * pb.box_bytes + 1023) // 1024 * 1024
        stage = fy * a_bytes + fx * b_bytes
        tx = fy * pa.bytes + fx * pb.bytes
        S = max(2, min(6, (200 * 1024) // stage))
        ring = self.smem.alloc(S * stage, 1024)
        bars = self.smem.alloc(8 * (2 * S + 1), 8)
        full = lambda e: f"reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * ({e}))"
        empty = lambda e: f"reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * ({S} + ({e})))"
        accbar = f"reinterpret_cast<tila::u64*>(tila_smem + {bars + 16 * S})"
        cols = {(i, j): self.tmem_alloc_cols(N) for (i, j) in inst}
        lay = TmemRows((128, N), self.T)
        if lay.groups != 1:
            self.fail("the persistent contraction needs one thread per accumulator row")
        e = self.emit
        e(f"{{ // persistent {fy}x{fx}-program tiles, K loops split evenly over the CTAs: "
          f"{S}-stage TMA ring, tcgen05.mma into TMEM")
        self.indent += 1
        e(f"const tila::i64 cl_start = (tila::i64)({start.expr});")
        e(f"const tila::i64 cl_end = (tila::i64)({end.expr});")
        e(f"const tila::i64 cl_n = cl_end > cl_start ? (cl_end - cl_start + {stepv - 1}) / {stepv} : 0;")
        e("const tila::i64 sk_kn = cl_n > 0 ? cl_n : 1;   // units per tile (one epilogue-only unit when K is empty)")
        e(f"const tila::i64 sk_n0 = (launch_0 + {FUSE - 1}) / {FUSE}, sk_n1 = (launch_1 + {FUSE - 1}) / {FUSE};")
        e("const tila::i64 sk_total = sk_n0 * sk_n1 * sk_kn;")
        e("const tila::i64 sk_u0 = sk_total * (tila::i64)blockIdx.x / gridDim.x;")
        e("const tila::i64 sk_u1 = sk_total * ((tila::i64)blockIdx.x + 1) / gridDim.x;")
        e("const tila::i64 sk_slot = (tila::i64)blockIdx.z * gridDim.x + blockIdx.x;")
        e("if (tid == 0) {")
        e(f"  for (int i = 0; i < {2 * S + 1}; ++i) tila::mbar_init(reinterpret_cast<tila::u64*>(tila_smem + {bars} + 8 * i), 1);")
        e("  tila::mbar_fence_init();")
        e("}")
        e("tila::tc_fence_before();")
        e("__syncthreads();")
        e("tila::tc_fence_after();")
        e("tila::u32 sk_ph = 0;")
        e("for (tila::i64 sk_p = sk_u0; sk_p < sk_u1; ) {")
        self.indent += 1
        e("const tila::i64 sk_t = sk_p / sk_kn, sk_ka = sk_p - sk_t * sk_kn;")
        e("const tila::i64 sk_end = (sk_t + 1) * sk_kn < sk_u1 ? (sk_t + 1) * sk_kn : sk_u1;")
        e("const tila::i64 sk_kb = sk_end - sk_t * sk_kn;")
        e("const tila::i32 sk_c0 = (tila::i32)(sk_t % sk_n0), sk_c1 = (tila::i32)(sk_t / sk_n0);")
        e("const bool sk_park = sk_ka > 0;                 // the high-K part of a split tile")
        e("const bool sk_fin = sk_ka == 0 && sk_kb < sk_kn;   // the low-K part: finishes the tile")
        for ax_ in (0, 1):
            for k in range(FUSE):
                e(f"const tila::i32 pid_{ax_}_{k} = (tila::i32)(sk_c{ax_} * {FUSE} + {k} + pid_off_{ax_});")
                e(f"const bool live_{ax_}_{k} = (tila::i32)(sk_c{ax_} * {FUSE} + {k}) < launch_{ax_};")
        envs = {}
        for (i, j) in inst:
            self.env = dict(base_env)
            self._pid_expr = {ay: f"pid_{ay}_{i}", ax: f"pid_{ax}_{j}"}
            for st in prefix:
                self.s_TAssign(st)
            envs[(i, j)] = dict(self.env)
        self._pid_expr = {}
        self.env = dict(envs[(0, 0)])

        def issue(jexpr, st):
            e("{")
            self.indent += 1
            lv = self.fresh(f"s_{loop.var}")
            e(f"const tila::i32 {lv} = (tila::i32)(cl_start + ({jexpr}) * {stepv});")
            e(f"tila::mbar_arrive_expect_tx({full(st)}, {tx}u);")
            for role, plan, nm, count, offset in (("A", pa, d.a_name, fy, 0), ("B", pb, d.b_name, fx, fy * a_bytes)):
                for k in range(count):
                    self.env = dict(envs[(k, 0)] if role == "A" else envs[(0, k)])
                    self.env[loop.var] = Val("scalar", D.i32, expr=lv)
                    for s2 in cl.functional:
                        self.s_TAssign(s2)
                    coords = [self.value(c) for c in cl.loads[nm].coords]
                    size = a_bytes if role == "A" else b_bytes
                    self._emit_tma(plan, self._tma_coords(plan, coords),
                                   f"{ring} + ({st}) * {stage} + {offset + k * size}", full(st))
            self.indent -= 1
            e("}")

        # producer (thread 32): the piece's units; a ring stage is reused once
        # the MMAs of the unit S before have completed
        e("if (tid == 32 && cl_n > 0) {")
        self.indent += 1
        e("for (tila::i64 u = sk_p; u < sk_end; ++u) {")
        self.indent += 1
        e("const tila::i64 q = u - sk_u0;")
        e(f"const int sj = (int)(q % {S});")
        e(f"if (q >= {S}) tila::mbar_wait({empty('sj')}, (tila::u32)(((q / {S}) - 1) & 1), tila_err, __LINE__, &tila_dead);")
        issue("u - sk_t * sk_kn", "sj")
        self.indent -= 1
        e("}")
        self.indent -= 1
        e("}")
        # MMA issuer (thread 0): the first MMA into each accumulator of a
        # piece does not accumulate (no zero fill of TMEM needed)
        e("if (tid == 0) {")
        self.indent += 1
        e("if (cl_n > 0) {")
        self.indent += 1
        e("for (tila::i64 u = sk_p; u < sk_end; ++u) {")
        self.indent += 1
        e("const tila::i64 q = u - sk_u0;")
        e(f"const int st = (int)(q % {S});")
        e(f"tila::mbar_wait({full('st')}, (tila::u32)((q / {S}) & 1), tila_err, __LINE__, &tila_dead);")
        e("tila::tc_fence_after();")
        e("const bool sk_first = u == sk_p;")
        merged = pb.inner == 1 and b_bytes == pb.nbox * pb.box_bytes
        K = pa.shape[1]
        for i in range(fy):
            a_val = self._smem_val(D.f16, pa.shape, self._smem_op(pa, f"{ring} + st * {stage} + {i * a_bytes}"))
            targets = [(0, fx)] if merged else [(j, 1) for j in range(fx)]
            for j0, nb in targets:
                b_val = self._smem_val(D.f16, (pb.shape[0], 128 * nb),
                                       self._smem_op(pb, f"{ring} + st * {stage} + {fy * a_bytes + j0 * b_bytes}"))
                for kk in range(K // 16):
                    da, a_mn = self._operand_desc(a_val, "A", kk)
                    db, b_mn = self._operand_desc(b_val, "B", kk)
                    idesc = f"tila::idesc_f16_f32(128, {128 * nb}, {a_mn}, {b_mn})"
                    accf = "sk_first ? 0u : 1u" if kk == 0 else "1u"
                    e(f"tila::mma_f16_ss(tila_tmem + {cols[(i, j0)]}, {da}, {db}, {idesc}, {accf});")
        e(f"tila::mma_commit({empty('st')});")
        self.indent -= 1
        e("}")
        self.indent -= 1
        e("}")
        e(f"tila::mma_commit({accbar});")
        self.indent -= 1
        e("}")
        e(f"tila::mbar_wait({accbar}, sk_ph, tila_err, __LINE__, &tila_dead);")
        e("sk_ph ^= 1u;")
        e("tila::tc_fence_after();")
        e("if (sk_fin) {   // the next CTA parked this tile's high-K part")
        e("  if (tid == 0) tila::flag_wait(tila_sk_flags + sk_slot + 1, 1u, tila_err, __LINE__, &tila_dead);")
        e("  __syncthreads();")
        e("}")
        # epilogues, one program at a time; TMA stores stage through the ring
        # (every unit of the piece has been consumed by a completed MMA)
        self._store_ring = {"base": ring, "bytes": S * stage, "size": None, "next": 0}
        for idx, (i, j) in enumerate(inst):
            a = self.fresh("acc")
            e(f"float {a}[{N}];")
            e("if (cl_n > 0) {")
            e(f"  tila::tmem_load_row<{N}>(tila_tmem + {cols[(i, j)]} + ((tid & 96u) << 16), {a});")
            e("} else {")
            e("  #pragma unroll")
            e(f"  for (int c = 0; c < {N}; ++c) {a}[c] = 0.0f;")
            e("}")
            wsx = f"(tila_sk_ws + ((sk_slot{{}}) * {len(inst)} + {idx}) * {128 * N} + (tid & 127))"
            e("if (sk_park) {")
            e("  #pragma unroll")
            e(f"  for (int c = 0; c < {N}; ++c) {wsx.format('')}[c * 128] = {a}[c];")
            e("} else {")
            self.indent += 1
            e("if (sk_fin) {")
            e("  #pragma unroll")
            # L2 reads: the values come from another SM
            e(f"  for (int c = 0; c < {N}; ++c) {a}[c] += __ldcg({wsx.format(' + 1')} + c * 128);")
            e("}")
            self.env = dict(envs[(i, j)])
            self._pid_expr = {ay: f"pid_{ay}_{i}", ax: f"pid_{ax}_{j}"}
            self.env[d.acc] = Val("reg", D.f32, (128, N), name=a, layout=lay)
            e(f"if (live_{ay}_{i} && live_{ax}_{j}) {{")
            self.indent += 1
            self.conv_cache = {}
            before = self._store_ring["next"]
            self.stmts(suffix)
            used = self._store_ring["next"] - before
            self.indent -= 1
            if used:
                e("} else if (tid == 0) {")
                e("  " + " ".join(["tila::bulk_commit();"] * used))
            e("}")
            self.indent -= 1
            e("}")
        used_any = self._store_ring["next"] > 0
        self._store_ring = None
        self._pid_expr = {}
        e("if (sk_park) {   // publish the parked accumulators")
        e("  __threadfence();")
        e("  __syncthreads();")
        e("  if (tid == 0) tila::flag_release(tila_sk_flags + sk_slot, 1u);")
        e("}")
        e("if (sk_fin) {   // the parked values are consumed: clear the flag for the next launch")
        e("  __syncthreads();")
        e("  if (tid == 0) tila_sk_flags[sk_slot + 1] = 0u;")
        e("}")
        if used_any:
            e("if (tid == 0) tila::bulk_wait_read();   // staging reads done before the ring is refilled")
        e("tila::tc_fence_before();")
        e("__syncthreads();   // accumulators and staging free for the next piece")
        e("tila::tc_fence_after();")
        e("sk_p = sk_end;")
        self.indent -= 1
        e("}")
        self.indent -= 1
        e("}")
        self._free_smem.append((ring, S * stage))

    def _smem_op(self, plan, base):
        from .mma import SmemOperand
        return SmemOperand(plan, base)
