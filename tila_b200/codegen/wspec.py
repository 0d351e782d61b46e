"""Warp-specialised lowering of the online-softmax attention loop.

Applies to the asynchronous accumulator loops that already run two programs
per CTA (one per warpgroup, see ``AsyncLoopMixin._pingpong_ok``) when the
loops have exactly the flash-attention shape: one synchronous dot
``S = dot(Q, K)`` whose A operand is a one-shot TMA tile loaded before the
loop and whose B operand is an in-loop TMA tile, and one accumulating dot
``acc = dot(cast[f16](P), V, acc=acc)`` with V an in-loop TMA tile.  The
kernel may have one such loop or a chain of them in which every loop starts
where the previous one ends (examples/fused_attention.py:104-126, the
CAUSAL=0 loop; 62-103, the CAUSAL=1 loops below and on the diagonal); in
every program the chain then walks one contiguous range of K/V tiles from a
start that both programs of a CTA share, so the shorter program's tiles are
a prefix of the longer one's.

The CTA then has three roles instead of two programs that each issue their own
copies and MMAs:

* warpgroups 0 and 1 run programs ``2 * blockIdx.x + w`` as before, but only
  the CUDA-core part of each iteration: wait for S in tensor memory, compute
  the softmax update, rescale the accumulator in place, store P (f16) into
  tensor memory and arrive on the program's "P ready" barrier;
* a copy thread (first thread of the third warpgroup) loads both programs'
  Q tiles once and streams K and V through a two-stage ring shared by the
  two programs (each tile crosses L2 once per CTA instead of once per
  program), as many tiles as the longer program needs;
* an MMA thread (first thread of the next warp) issues every
  ``tcgen05.mma``: per iteration, for each program that still runs, P@V of
  iteration j, then S of iteration j + 1, so the tensor pipe holds the other
  program's work while one program is in its softmax.  Each program's
  iterations are counted from its own program id (``tila_nw``); a run-time
  check of the chain's contiguity records ``kErrSchedule`` if it fails;
* the two softmax warpgroups are not serialised by a hand-off: both run
  concurrently; ``setmaxnreg`` moves registers from the producer warpgroup
  to them (``ws_budget``).

Barriers (all waits bounded, see ``tila::mbar_wait``): per program the S
barrier (``tila_mma_bar``, committed by the producer after S), the
accumulator barrier (committed after P@V) and the "P ready" barrier (128
consumer arrivals); per ring stage K/V "full" (TMA transaction count) and
"empty" (committed after the MMAs that read the stage).  ``tcgen05.mma``
operations of one thread execute in issue order, so S(j + 1), issued after
P@V(j), overwrites the tensor-memory columns that P@V(j) reads only after
that MMA consumed them, and a consumer that has waited for S(j + 1) knows that
P@V(j) is complete.

When the programs' trip counts grow (or shrink) with program_id(0), the CTAs
are renumbered so that the heaviest start first within groups of CTA_GROUP
positions along the other grid axes (``cta_order_prelude``).

The producer's code is built from the same TMA plans, descriptors and
coordinate expressions as the consumer's would be; a coordinate that depends
on anything but the program ids, kernel parameters and the loop variable, or
K/V coordinates that depend on program_id(0), make the kernel fall back to
the two-program lowering.
"""

from __future__ import annotations

import dataclasses
import math
import re

from .._reference import tila

T_ = tila.tir
D = tila.dtypes

RING = 2                   # stages of the K and V rings


def ws_budget(T):
    """(threads, registers per thread at launch, producer, consumer registers)
    of the warp-specialised kernel whose programs have T = 128 threads.

    The CTA is two programs of T threads plus the producer warpgroup.
    ``__launch_bounds__(threads, 1)`` gives every thread 65536 / threads
    registers at launch, rounded down to a multiple of 8; that times the
    thread count is the pool the warpgroups trade in (setmaxnreg).  The
    producer gives back all but its share, the consumers take theirs, and the
    shares add up to at most the pool, so reg_alloc never waits for
    registers that do not exist.  The host refuses to launch the kernel
    unless ptxas allocated exactly the launch count.  (Programs requested
    with 8 warps get this 4-warp form too: with two 256-thread softmax
    warpgroups the registers left per thread made the kernel spill.)"""
    assert T == 128
    threads = 2 * T + 128
    launch = (65536 // threads) // 8 * 8
    producer, consumer = 64, 216
    assert 128 * producer + 2 * T * consumer <= threads * launch
    assert producer <= launch <= consumer and producer % 8 == 0 and consumer % 8 == 0
    return threads, launch, producer, consumer


_IDENT = re.compile(r"[A-Za-z_][A-Za-z0-9_]*")
_ALLOWED = {"pid_0", "pid_1", "pid_2", "tila_pit", "int", "long", "unsigned", "float", "double",
            "true", "false", "LL", "ULL", "u", "ull"}


def _multiple_of(em, node, depth=0):
    """A positive integer that provably divides the value of TIR expression
    ``node`` in every program (1 when nothing is known; 0 stands for the
    value 0, which every integer divides)."""
    if depth > 24 or node is None:
        return 1
    if isinstance(node, T_.TLit) and isinstance(node.value, int) and not isinstance(node.value, bool):
        return abs(node.value)
    if isinstance(node, T_.TName):
        c = em.consts.get(node.name)
        if isinstance(c, int) and not isinstance(c, bool):
            return abs(c)
        d = em.pdefs.resolve(node)
        return 1 if d is node else _multiple_of(em, d, depth + 1)
    if isinstance(node, T_.TCast):
        return _multiple_of(em, node.operand, depth + 1)
    if isinstance(node, T_.TBin):
        a, b = _multiple_of(em, node.left, depth + 1), _multiple_of(em, node.right, depth + 1)
        if node.op == "*":
            return a * b
        if node.op in ("+", "-"):
            return math.gcd(a, b)
    return 1


def _eval_at_pid0(em, node, pid0, depth=0):
    """Value of integer TIR expression ``node`` with program_id(0) = pid0,
    when it is built from that id, Consts and literals only (else None)."""
    if depth > 24 or node is None:
        return None
    if isinstance(node, T_.TPid):
        return pid0 if node.axis == 0 else None
    if isinstance(node, T_.TLit) and isinstance(node.value, int) and not isinstance(node.value, bool):
        return node.value
    if isinstance(node, T_.TName):
        c = em.consts.get(node.name)
        if isinstance(c, int) and not isinstance(c, bool):
            return c
        d = em.pdefs.resolve(node)
        return None if d is node else _eval_at_pid0(em, d, pid0, depth + 1)
    if isinstance(node, T_.TCast):
        return _eval_at_pid0(em, node.operand, pid0, depth + 1)
    if isinstance(node, T_.TBin) and node.op in ("+", "-", "*"):
        a = _eval_at_pid0(em, node.left, pid0, depth + 1)
        b = _eval_at_pid0(em, node.right, pid0, depth + 1)
        if a is None or b is None:
            return None
        return a + b if node.op == "+" else a - b if node.op == "-" else a * b
    return None


# heads (grid axes 1 and 2) per group of the heavy-first CTA order
CTA_GROUP = 8


def cta_order_prelude(heavy_last):
    """Kernel prologue that renumbers the CTAs of a grid whose programs' work
    grows (``heavy_last``) or shrinks along axis 0: CTAs are dispatched in
    linear order, and the renumbering hands out, for every group of
    CTA_GROUP positions along axes 1 and 2, the heaviest axis-0 position
    first.  The long CTAs then start early (no tail of long CTAs on a few
    SMs) while the CTAs running at one time share a few groups' tiles in
    L2.  A bijection of the grid; programs compute what they computed."""
    bx = "tila_X - 1u - tila_q" if heavy_last else "tila_q"
    return f"""  // CTA order: heaviest axis-0 position first within groups of {CTA_GROUP} positions along axes 1-2
  const unsigned tila_X = gridDim.x, tila_YZ = gridDim.y * gridDim.z;
  const unsigned tila_lin = blockIdx.x + tila_X * (blockIdx.y + gridDim.y * blockIdx.z);
  const unsigned tila_full = tila_YZ / {CTA_GROUP}u * {CTA_GROUP}u;
  const bool tila_in_full = tila_lin < tila_full * tila_X;
  const unsigned tila_gs = tila_in_full ? {CTA_GROUP}u : tila_YZ - tila_full;
  const unsigned tila_base = tila_in_full ? tila_lin / ({CTA_GROUP}u * tila_X) * {CTA_GROUP}u : tila_full;
  const unsigned tila_r = tila_in_full ? tila_lin % ({CTA_GROUP}u * tila_X) : tila_lin - tila_full * tila_X;
  const unsigned tila_q = tila_r / tila_gs, tila_h = tila_base + tila_r % tila_gs;
  const unsigned tila_bx = {bx}, tila_by = tila_h % gridDim.y, tila_bz = tila_h / gridDim.y;
"""


def _plan_key(plan):
    """A TMA plan without its TIR coordinate nodes (compared by value)."""
    return tuple((f.name, getattr(plan, f.name)) for f in dataclasses.fields(plan)
                 if f.name not in ("coords", "coord_nodes"))


def _portable(expr: str) -> bool:
    """``expr`` reads only program ids, kernel parameters, the producer's loop
    variable, literals and tila:: helpers (so it means the same in the
    producer warp as in a consumer)."""
    stripped = re.sub(r"tila::[A-Za-z0-9_:<>]+", " ", expr)
    stripped = re.sub(r"\b(0x[0-9a-fA-F]+|\d+)[uUlL]*\b", " ", stripped)
    for ident in _IDENT.findall(stripped):
        if ident in _ALLOWED or ident.startswith(("p_", "nprog_", "pid_off_")):
            continue
        return False
    return True


class WarpSpecMixin:
    """Mixed into :class:`tila_b200.codegen.emitter.KernelEmitter`."""

    # -- first pass: is the loop of the warp-specialised shape? ------------------

    def ws_detect(self, s, start, end, stepv, al, ctx):
        """First pass: record the loops of the warp-specialised shape.

        A kernel qualifies when its asynchronous accumulator loops form one
        chain of flash-attention-shaped loops (module doc) over the same
        one-shot Q tile: each loop starts where the previous one ends, with
        the same step, so that for every program the loops walk one
        contiguous range of K/V tiles from a start that is the same for both
        programs of a CTA (examples/fused_attention.py: one loop with
        CAUSAL=0, the below-diagonal loop and the diagonal loop with
        CAUSAL=1).  The two programs may run different numbers of
        iterations; the producer serves the longer one."""
        q = self._ws_loop_shape(s, start, al)
        if getattr(self, "_ws_bad", False):
            return
        if q is None:
            self._ws_bad, self._ws_found = True, None
            return
        loop = dict(start=start.expr, end=end.expr, step=int(stepv),
                    even=all(n is None or self._pid0_free(n) for n in (s.start, s.end)))
        found = self._ws_found
        if found is None:
            if s.start is not None and not self._pid0_free(s.start):
                self._ws_bad = True
                return
            self._ws_found = {"q": q, "loops": [loop]}
            self._ws_last_loop = s
            return
        prev, prev_node = found["loops"][-1], self._ws_last_loop
        whole = _multiple_of(self, prev_node.start) if prev_node.start is not None else 0
        whole = math.gcd(whole, _multiple_of(self, prev_node.end))
        if (q != found["q"] or loop["step"] != prev["step"] or loop["start"] != prev["end"]
                or whole % loop["step"]):
            self._ws_bad, self._ws_found = True, None
            return
        found["loops"].append(loop)
        self._ws_last_loop = s

    def _ws_loop_shape(self, s, start, al):
        """The name of the one-shot Q tile when loop ``s`` has the
        flash-attention shape, else None."""
        from .pipeline import _walk
        if self.T not in (128, 256) or not self._pingpong_ok(s, start, al, any_T=True):
            return None
        if al.cast_loads or len(al.loads) != 2 or len(al.accs) != 1:
            return None
        (acc_name, acc_dot), = al.accs.items()
        if not (isinstance(acc_dot.a, T_.TCast) and isinstance(acc_dot.a.operand, T_.TName)
                and acc_dot.a.operand.name not in al.loads):
            return None
        syncs = []
        for st in s.body:
            _walk(st.value, lambda n: syncs.append(n) if isinstance(n, T_.TDot) and n.acc is None else None)
        if len(syncs) != 1:
            return None
        sd = syncs[0]
        if not (isinstance(sd.a, T_.TName) and isinstance(sd.b, T_.TName) and sd.b.name in al.loads
                and sd.b.name != acc_dot.b.name):
            return None
        q = self.env.get(sd.a.name)
        op = getattr(q, "smem", None)
        if q is None or q.kind != "smem" or op is None or op.bar is None or not op.nbytes:
            return None
        _, (M, N), _ = self.vt_info(sd.vt)
        if M != 128 or self.vt_info(acc_dot.vt)[1][0] != 128:
            return None
        return sd.a.name

    def ws_ready(self):
        """The recorded chain may run warp-specialised: Q is read by the
        chain's dots only."""
        f = self._ws_found
        if f is None or getattr(self, "_ws_bad", False):
            return None
        if len(self.uses.get(f["q"], [])) != len(f["loops"]):
            return None
        # programs whose trip counts grow or shrink with program_id(0): the
        # CTAs are renumbered heaviest-first (see cta_order_prelude)
        f["heavy_last"] = None
        if not all(loop["even"] for loop in f["loops"]):
            last = self._ws_last_loop
            n0, n1 = _eval_at_pid0(self, last.end, 0), _eval_at_pid0(self, last.end, 1)
            if n0 is not None and n1 is not None and n0 != n1:
                f["heavy_last"] = n1 > n0
        return f

    # -- second pass: the consumer side --------------------------------------------

    def ws_oneshot(self, x, assigned_name, plan, coords):
        """The Q tile: shared memory and a barrier in the program's region; the
        producer copies it, the consumers never touch it."""
        size = plan.nbox * max(plan.outer_extent, 128) * 128
        off = self.smem.alloc(size, 1024)
        bar_off = self.smem.alloc(8, 8)
        coords_if = self._tma_coords(plan, coords)
        if not all(_portable(c) for c in coords_if):
            self.fail("warp-specialised loop: the Q copy depends on program-local values")
        self._ws["q_load"] = dict(plan=plan, coords=coords_if, off=off, bar_off=bar_off, size=size)
        self.tensor_map_param(plan)        # a kernel parameter of the producer's copies
        from .mma import SmemOperand
        dt, shape, _ = self.vt_info(x.vt)
        v = self._smem_val(dt, shape, SmemOperand(plan, str(off), None, "0u", None, nbytes=size))
        return v

    def ws_loop_setup(self, s, start, end, stepv, al):
        from .emitter import Val
        from .layouts import TmemRows
        from .mma import AsyncCtx, SmemOperand
        from .pipeline import _walk
        ws = self._ws
        chain = ws.get("loops") or [dict(start=start.expr, end=end.expr, step=int(stepv))]
        k = ws.get("loops_seen", 0)
        if ("q_load" not in ws or k >= len(chain) or chain[k]["start"] != start.expr
                or chain[k]["end"] != end.expr or chain[k]["step"] != int(stepv)):
            self.fail("warp-specialised loop: unexpected loop structure")
        ws["loops"] = chain
        ws["loops_seen"] = k + 1
        self.uses_mma = True
        self.uses_tmem = True
        ctx = AsyncCtx(al, s.var, stepv, f"(tila::i64)({end.expr})", {}, {})
        ctx.body = s.body
        ctx.cast_loads = set()
        ctx.p_early_after = self._early_p_points(s.body, al)
        ctx.p_early = False
        ctx.pingpong = False
        ctx.turns = None
        ctx.ws = True
        (acc_name, acc_dot), = al.accs.items()
        syncs = []
        for st in s.body:
            _walk(st.value, lambda n: syncs.append(n) if isinstance(n, T_.TDot) and n.acc is None else None)
        sd = syncs[0]
        if sd.a.name != ws["q"]:
            self.fail("warp-specialised loop: unexpected synchronous dot")
        k_name, v_name = sd.b.name, acc_dot.b.name
        for name, ld in al.loads.items():
            ctx.loads[name] = dict(plan=self.tma_plan(ld), node=ld, base=None, bar=None,
                                   phase=None, flag=None)
        if k > 0:
            return self._ws_loop_continue(s, ctx, acc_name, acc_dot, k_name, v_name)
        _, (M, N), _ = self.vt_info(acc_dot.vt)
        col = self.tmem_alloc_cols(N)
        self._loop_acc_cols.add((str(col), N))
        bar_off = self.smem.alloc(8, 8)
        ctx.accs[acc_name] = dict(col=col, N=N, bar_off=bar_off,
                                  bar=f"reinterpret_cast<tila::u64*>(tila_smem + {bar_off})",
                                  phase=self._tma_state_var(f"tila_ph_{bar_off}"),
                                  pend=self._tma_state_var(f"tila_p_{bar_off}"),
                                  releases=[], dot=acc_dot)
        p_full = self.smem.alloc(8, 8)
        ctx.p_full_off = p_full
        K_pv = self.vt_info(acc_dot.a.vt)[1][1]
        self.tmem_scratch_need = max(self.tmem_scratch_need, K_pv // 2)
        # the accumulator's initial value into tensor memory
        pre = self.env[acc_name]
        lay = TmemRows((128, N), self.T)
        if pre.kind == "tmem":
            pre = self.tmem_to_reg(pre)
        if pre.dt.name != "f32":
            pre = self.coerce(pre, D.f32)
        if pre.kind == "scalar":
            pre = self.materialize_elementwise(D.f32, (128, N), [pre], lambda e: e[0], layout=lay)
        pre = self.materialize(pre, lay)
        goff = f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else ""
        self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {col}{goff} + ((tid & 96u) << 16), {pre.name});")
        self.emit(f"// warp-specialised loop over {s.var}: S from the producer warp, P handed back "
                  f"through tensor memory, {acc_name} accumulated in tensor memory")
        a = ctx.accs[acc_name]
        self.emit(f"{a['phase']} = 0u; {a['pend']} = 0u;")
        self.env[acc_name] = Val("tmem", D.f32, (128, N), tmem_col=str(col))
        # producer templates: TMA copies of K and V for loop value tila_pit
        copies = self._ws_kv_copies(ctx, k_name, v_name)
        for loop in chain:
            if not (_portable(loop["start"]) and _portable(loop["end"])):
                self.fail("warp-specialised loop: loop bounds depend on program-local values")
        # MMA templates (@QB@, @KB@, @VB@: byte offsets in the CTA's shared memory)
        q = ws["q_load"]
        qv = self._smem_val(D.f16, q["plan"].shape, SmemOperand(q["plan"], "@QB@"))
        kv = self._smem_val(D.f16, copies[k_name]["plan"].shape, SmemOperand(copies[k_name]["plan"], "@KB@"))
        vv = self._smem_val(D.f16, copies[v_name]["plan"].shape, SmemOperand(copies[v_name]["plan"], "@VB@"))
        _, (Ms, Ns), _ = self.vt_info(sd.vt)
        Ks = q["plan"].shape[1] if q["plan"].inner == 1 else q["plan"].shape[0]
        Npad = max(16, Ns)
        self.tmem_scratch_need = max(self.tmem_scratch_need, Npad)
        s_mma = []
        a_mn = self._operand_desc(qv, "A", 0)[1]
        b_mn = self._operand_desc(kv, "B", 0)[1]
        for kk in range(Ks // 16):
            da, _ = self._operand_desc(qv, "A", kk)
            db, _ = self._operand_desc(kv, "B", kk)
            s_mma.append(f"tila::mma_f16_ss(@TM@ + @SCOL@, {da}, {db}, "
                         f"tila::idesc_f16_f32(128, {Npad}, {a_mn}, {b_mn}), {'1u' if kk else '0u'});")
        pv_mma = []
        vb_mn = self._operand_desc(vv, "B", 0)[1]
        for kk in range(K_pv // 16):
            db, _ = self._operand_desc(vv, "B", kk)
            pv_mma.append(f"tila::mma_f16_ts(@TM@ + {col}, @TM@ + @SCOL@ + {kk * 8}, {db}, "
                          f"tila::idesc_f16_f32(128, {N}, 0, {vb_mn}), 1u);")
        ws.update(k=copies[k_name], v=copies[v_name], s_mma=s_mma, pv_mma=pv_mma,
                  step=stepv, acc_bar=bar_off, p_full=p_full, acc_col=col,
                  acc_entry=ctx.accs[acc_name], acc_name=acc_name)
        self._wg_candidate = True
        self.actx = ctx
        return ctx

    def _ws_kv_copies(self, ctx, k_name, v_name):
        """TMA plans and coordinates of the loop's K and V copies for loop
        value ``tila_pit`` (the producer's); they must read nothing but the
        program ids, kernel parameters and the loop value, and not depend on
        program_id(0): both programs of the CTA share the stream."""
        saved_env, saved_lines, saved_indent = dict(self.env), self.lines, self.indent
        self.lines, self.indent = [], 0
        try:
            self._functional_prefix(ctx, "tila_pit")
            copies = {}
            for name in (k_name, v_name):
                x = ctx.loads[name]
                coords = [self.value(c) for c in x["node"].coords]
                copies[name] = dict(plan=x["plan"], coords=self._tma_coords(x["plan"], coords))
                self.tensor_map_param(x["plan"])
            stray = [ln for ln in self.lines if ln.strip()]
        finally:
            self.env, self.lines, self.indent = saved_env, saved_lines, saved_indent
        if stray or not all(_portable(c) and not re.search(r"\bpid_0\b", c)
                            for cp in copies.values() for c in cp["coords"]):
            self.fail("warp-specialised loop: K/V copies depend on program-local values")
        return copies

    def _ws_loop_continue(self, s, ctx, acc_name, acc_dot, k_name, v_name):
        """A later loop of the chain: the accumulator, its barriers and phase
        variables and the producer's templates carry over from the first loop
        (its iterations continue the same stream of K/V tiles and MMAs)."""
        from .emitter import Val
        ws = self._ws
        if acc_name != ws["acc_name"] or self.vt_info(acc_dot.vt)[1][1] != ws["acc_entry"]["N"]:
            self.fail("warp-specialised loop: the loops accumulate into different tiles")
        copies = self._ws_kv_copies(ctx, k_name, v_name)
        for cur, first in ((copies[k_name], ws["k"]), (copies[v_name], ws["v"])):
            if cur["coords"] != first["coords"] or _plan_key(cur["plan"]) != _plan_key(first["plan"]):
                self.fail("warp-specialised loop: the loops copy different K/V tiles")
        pre = self.env.get(acc_name)
        if pre is None or pre.kind != "tmem" or str(pre.tmem_col) != str(ws["acc_col"]):
            self.fail("warp-specialised loop: the accumulator left tensor memory between the loops")
        ctx.accs[acc_name] = dict(ws["acc_entry"], dot=acc_dot)
        ctx.p_full_off = ws["p_full"]
        self.emit(f"// warp-specialised loop over {s.var} (continues the previous loop's stream)")
        self.env[acc_name] = Val("tmem", D.f32, (128, ws["acc_entry"]["N"]), tmem_col=str(ws["acc_col"]))
        self.actx = ctx
        return ctx

    def ws_sync_dot(self, x):
        """S = dot(Q, K) of the warp-specialised loop: the producer issued it
        and commits it to tila_mma_bar; read it from tensor memory."""
        from .emitter import Val
        dt, (M, N), _ = self.vt_info(x.vt)
        if dt.name != "f32" or not (isinstance(x.a, T_.TName) and x.a.name == self._ws["q"]):
            self.fail("warp-specialised loop: unexpected synchronous dot")
        self.uses_mma = True
        self.uses_tmem = True
        self.tmem_scratch_need = max(self.tmem_scratch_need, max(16, N))
        self.emit("tila::mbar_wait(tila_mma_bar, tila_mma_phase, tila_err, __LINE__, &tila_dead);")
        self.emit("tila_mma_phase ^= 1u;")
        self.emit("tila::tc_fence_after();")
        reg = self.tmem_to_reg(Val("tmem", D.f32, (M, N), tmem_col="tila_tmem_scratch_col"))
        self.emit("tila::tc_fence_before();")
        return reg

    def ws_acc_dot(self, x, name):
        """acc = dot(cast[f16](P), V, acc=acc): store P into tensor memory and
        hand it to the producer, which issues P@V and commits it to the
        accumulator barrier."""
        from .emitter import Val
        from .layouts import TmemRows
        ctx = self.actx
        a = ctx.accs[name]
        N = a["N"]
        self.wait_all_accs(release=False)
        acc = self.env[name]
        if acc.kind != "tmem":
            lay = TmemRows((128, N), self.T)
            accv = acc if acc.dt.name == "f32" else self.coerce(acc, D.f32)
            accv = self.materialize(accv, lay) if not (accv.kind == "reg" and accv.layout == lay) else accv
            goff = f" + (tid >> 7) * {lay.cpg}" if lay.groups > 1 else ""
            self.emit(f"tila::tmem_store_row<{lay.nreg}>(tila_tmem + {a['col']}{goff} + ((tid & 96u) << 16), {accv.name});")
        if ctx.p_early:
            ctx.p_early = False
        else:
            pv = self.value(x.a.operand)
            if pv.kind == "smem":
                self.fail("warp-specialised loop: P must be a register tile")
            self._store_p(pv, ctx)
        self.emit("tila::tmem_wait_st();")
        self.emit("tila::tc_fence_before();")
        self.emit(f"tila::mbar_arrive(reinterpret_cast<tila::u64*>(tila_smem + {ctx.p_full_off}));")
        self.emit(f"{a['pend']} = 1u;")
        v = Val("tmem", D.f32, (128, N), tmem_col=str(a["col"]))
        v.pending = name
        return v

    def ws_finish(self, ctx):
        """After the last loop of the chain: the Q tile is dead (its last
        reader, S of the last iteration, completed before the final P@V); its
        shared memory can stage the epilogue's stores."""
        ws = self._ws
        if ws["loops_seen"] < len(ws["loops"]):
            return
        q = ws["q_load"]
        self._free_smem.append((q["off"], q["size"]))

    # -- assembly ------------------------------------------------------------------

    def ws_producer(self, per_prog, ring_off, bars_off, scratch_col):
        """Code of the two producer threads: (copy thread 256, MMA thread 288)."""
        ws = self._ws
        kp, vp = ws["k"], ws["v"]
        kbytes = kp["plan"].nbox * max(kp["plan"].outer_extent, 128) * 128
        vbytes = vp["plan"].nbox * max(vp["plan"].outer_extent, 128) * 128
        kring = [ring_off + i * kbytes for i in range(RING)]
        vring = [ring_off + RING * kbytes + i * vbytes for i in range(RING)]
        bar = lambda i: f"reinterpret_cast<tila::u64*>(tila_smem_all + {bars_off + 8 * i})"
        k_full = [bar(i) for i in range(RING)]
        k_empty = [bar(RING + i) for i in range(RING)]
        v_full = [bar(2 * RING + i) for i in range(RING)]
        v_empty = [bar(3 * RING + i) for i in range(RING)]
        region = lambda w, off: f"reinterpret_cast<tila::u64*>(tila_smem_all + {w * per_prog + off})"
        q = ws["q_load"]
        L = []
        e = L.append

        def tma(plan, coords, dst, barx, ind="      "):
            for b in range(plan.nbox):
                cs = list(coords)
                if b:
                    cs[0] = f"({cs[0]} + {plan.box_elems * b})"
                tm = self.tensor_map_param(plan)
                e(f"{ind}tila::tma_load_{plan.rank}d(tila_smem_all + {dst} + {b * plan.box_bytes}, &{tm}, {barx}, {', '.join(cs)});")

        def wait(barx, parity):
            e(f"      if (!tila::mbar_wait({barx}, {parity}, tila_err, __LINE__, &tila_dead)) goto tila_producer_end;")

        def mmas(lines, w, qb=None, kb=None, vb=None):
            for ln in lines:
                ln = ln.replace("@TM@", f"(tila_tmem_base + {w} * {self.tmem_cols})").replace("@SCOL@", str(scratch_col))
                if qb is not None:
                    ln = ln.replace("@QB@", str(qb))
                if kb is not None:
                    ln = ln.replace("@KB@", kb)
                if vb is not None:
                    ln = ln.replace("@VB@", vb)
                e("      " + ln)

        step = ws["step"]
        # per program w: its iterations over the chain of loops (bounds
        # evaluated with its own program id), which must walk one contiguous
        # range from the first loop's start (that start is the same for both
        # programs, so the shorter program's tiles are a prefix of the other's)
        head = ["    const bool tila_live_w[2] = {(tila::i32)(blockIdx.x * 2) < launch_0, "
                "(tila::i32)(blockIdx.x * 2 + 1) < launch_0};",
                f"    const tila::i64 tila_lo = (tila::i64)({ws['loops'][0]['start']});",
                "    tila::i64 tila_nw[2] = {0, 0};",
                "    bool tila_chain_ok = true;"]
        for w in range(2):
            head.append(f"    if (tila_live_w[{w}]) {{")
            head.append(f"      const tila::i32 pid_0 = (tila::i32)(blockIdx.x * 2 + {w} + pid_off_0); (void)pid_0;")
            head.append("      tila::i64 pos_ = tila_lo;")
            for loop in ws["loops"]:
                head.append(f"      {{ const tila::i64 s_ = (tila::i64)({loop['start']}), e_ = (tila::i64)({loop['end']});")
                head.append(f"        const tila::i64 t_ = e_ > s_ ? (e_ - s_ + {step - 1}) / {step} : 0;")
                head.append(f"        if (t_ > 0 && s_ != pos_) tila_chain_ok = false;")
                head.append(f"        tila_nw[{w}] += t_; if (t_ > 0) pos_ = s_ + t_ * {step}; }}")
            head.append("    }")
        head.append("    if (!tila_chain_ok) tila_nw[0] = tila_nw[1] = 0;")
        head.append("    const tila::i64 tila_n = tila_nw[0] > tila_nw[1] ? tila_nw[0] : tila_nw[1];")

        # -- copy thread (threadIdx.x == 256): Q once, then K and V of every
        #    iteration into stage j & 1 as soon as the MMAs that read the
        #    stage's previous tile are done (empty barrier of that use)
        e("    // copies: both programs' Q tiles, then K and V through the two-stage ring")
        L.extend(head)
        for w in range(2):
            # (a program with no iterations never waits for its Q tile, so
            # none is copied: its epilogue reuses that shared memory)
            e(f"    if (tila_nw[{w}] > 0) {{")
            e(f"      const tila::i32 pid_0 = (tila::i32)(blockIdx.x * 2 + {w} + pid_off_0);")
            e(f"      tila::mbar_arrive_expect_tx({region(w, q['bar_off'])}, {q['plan'].bytes}u);")
            tma(q["plan"], q["coords"], w * per_prog + q["off"], region(w, q["bar_off"]))
            e("    }")
        e("    for (tila::i64 j = 0; j < tila_n; ++j) {")
        e("      const tila::u32 up = (tila::u32)(((j >> 1) - 1) & 1);   // parity of the stage's previous use")
        e(f"      const tila::i32 tila_pit = (tila::i32)(tila_lo + j * {step});")
        e("      (void)tila_pit;")
        for name, cp, full, empty, base in (("K", kp, k_full, k_empty, kring), ("V", vp, v_full, v_empty, vring)):
            for st in range(RING):
                e(f"      if ((j & 1) == {st}) {{  // {name} of iteration j into stage {st}")
                e(f"        if (j >= 2 && !tila::mbar_wait({empty[st]}, up, tila_err, __LINE__, &tila_dead)) goto tila_copy_end;")
                e(f"        tila::mbar_arrive_expect_tx({full[st]}, {cp['plan'].bytes}u);")
                tma(cp["plan"], cp["coords"], base[st], full[st], "        ")
                e("      }")
        e("    }")
        e("  tila_copy_end: ;")
        copy_lines = list(L)
        L.clear()

        # -- MMA thread: per iteration j and program w (while j < its trip
        #    count) P@V(j), then S(j+1) into the columns P@V(j) has just read
        e("    // MMAs: S = Q K^T and O += P V of both programs, in issue order per program")
        e("    const tila::u32 tila_sb4 = tila::smem_u32(tila_smem_all) >> 4;")
        L.extend(head)
        e("    if (!tila_chain_ok) { tila::report_error(tila_err, tila::kErrSchedule, __LINE__); tila_dead = 1; }")
        e("    if (tila_n > 0) {")
        for w in range(2):
            e(f"      if (tila_nw[{w}] > 0) {{")
            e(f"        if (!tila::mbar_wait({region(w, q['bar_off'])}, 0u, tila_err, __LINE__, &tila_dead)) goto tila_mma_end;")
            e("      }")
        e(f"      if (!tila::mbar_wait({k_full[0]}, 0u, tila_err, __LINE__, &tila_dead)) goto tila_mma_end;")
        e("      tila::tc_fence_after();")
        for w in range(2):
            e(f"      if (tila_nw[{w}] > 0) {{")
            mmas(ws["s_mma"], w, qb=w * per_prog + q["off"], kb=str(kring[0]))
            e(f"        tila::mma_commit({region(w, 0)});")
            e("      }")
        e(f"      tila::mma_commit({k_empty[0]});")
        e("    }")
        e("    for (tila::i64 j = 0; j < tila_n; ++j) {")
        e("      const int st = (int)(j & 1), nx = (int)((j + 1) & 1);")
        e("      const tila::u32 par = (tila::u32)((j >> 1) & 1), npar = (tila::u32)(((j + 1) >> 1) & 1);")
        e("      const bool more = j + 1 < tila_n;")
        e(f"      if (!tila::mbar_wait(st ? {v_full[1]} : {v_full[0]}, par, tila_err, __LINE__, &tila_dead)) goto tila_mma_end;")
        e(f"      if (more && !tila::mbar_wait(nx ? {k_full[1]} : {k_full[0]}, npar, tila_err, __LINE__, &tila_dead)) goto tila_mma_end;")
        e(f"      const tila::u32 vb = st ? {vring[1]}u : {vring[0]}u;")
        e(f"      const tila::u32 kb = nx ? {kring[1]}u : {kring[0]}u;")
        for w in range(2):
            e(f"      if (j < tila_nw[{w}]) {{")
            e(f"        if (!tila::mbar_wait({region(w, ws['p_full'])}, (tila::u32)(j & 1), tila_err, __LINE__, &tila_dead)) goto tila_mma_end;")
            e("        tila::tc_fence_after();")
            mmas(ws["pv_mma"], w, vb="vb")
            e(f"        tila::mma_commit({region(w, ws['acc_bar'])});")
            e(f"        if (j + 1 < tila_nw[{w}]) {{")
            mmas(ws["s_mma"], w, qb=w * per_prog + q["off"], kb="kb")
            e(f"          tila::mma_commit({region(w, 0)});")
            e("        }")
            e("      }")
        e("      // stage frees: K of iteration j + 1 once the S(j + 1) that read it are done, V of j once the P@V(j) are")
        e(f"      if (more) tila::mma_commit(nx ? {k_empty[1]} : {k_empty[0]});")
        e(f"      tila::mma_commit(st ? {v_empty[1]} : {v_empty[0]});")
        e("    }")
        e("  tila_mma_end: ;")
        nbars = 4 * RING
        return (copy_lines, list(L)), nbars, kbytes * RING + vbytes * RING
