"""Benchmark of the B200 Tila backend on the five benchmarked workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--only]
                    [--impl reference]

One JSON line on rank 0.  The headline workload (default: row softmax,
f32 [8192, 1000], the second configuration) gives ``metric``/``value``; every
other workload is measured in the same run under ``workloads`` unless
``--only`` is given.

Per workload:
* ``value``   device time of K steps (CUDA graph of K kernel launches, inputs
  resident in HBM, rotating input sets whose total footprint exceeds L2), max
  over ranks; whole-job units / time.
* ``e2e``     the same metric through the public API: ``kernel[grid](...)``
  on CUDA tensors with the inputs copied from pinned host memory and the
  output copied back inside the timed region (Tila's host-side contract and
  proof checks included, as for every Tila launch).
* ``roofline``  achieved / measured peak (MEASURED_PEAKS.json) of the
  dominant kernel.
* ``cpu_baseline``  Tila's NumPy reference interpreter on a bounded sample of
  the workload, spread over every host core by worker processes (rank 0,
  N = 1).

Multi-GPU (torchrun, one process per GPU): weak scaling.  The job is N copies
of the configuration along its program axis (rows, output tiles or
batch*heads); each rank launches its share of the global program grid with
``tila_b200.program_range`` and the output shards are gathered to rank 0
with NCCL (timed separately as ``gather_ms``).

``--impl reference`` times the reference itself - Tila's NumPy interpreter,
its only CPU execution path - on the same workloads and prints the same line
with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import atexit
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * (1 << 20)
ORDER = ["softmax", "add", "matmul", "unfused_attention", "fused_attention", "fused_attention_causal"]


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def _traffic_table():
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ---------------------------------------------------------------------------
# clocks sampling
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.index = self._gpu_id(device)
        self.proc = None
        self.file = None

    @staticmethod
    def _gpu_id(device):
        import torch
        try:
            p = torch.cuda.get_device_properties(device)
            return f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        except Exception:
            return str(device.index)

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# workloads: setup of N-way weak-scaled problems and their steps
# ---------------------------------------------------------------------------

class Case:
    """One workload instance on this rank: device buffers (several sets, so
    that consecutive steps read memory that is not L2-resident), the launches
    of one step, and the metadata for the JSON line."""

    def __init__(self, key, world, rank, device, strong=False):
        import torch
        import tila_b200
        from tila_b200 import workloads as W
        self.key, self.world, self.rank, self.device = key, world, rank, device
        # weak scaling: the job is `world` copies of the configuration along
        # its program axis; strong scaling: one configuration split `world` ways
        self.mult = 1 if strong else world
        self.W, self.ti, self.torch = W, tila_b200.tila, torch
        self.tila_b200 = tila_b200
        getattr(self, f"_setup_{key}")()

    # helpers
    def _dev(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a)).to(self.device)

    def _sets(self, bytes_per_set):
        return max(1, min(16, -(-2 * L2_BYTES // max(1, bytes_per_set))))

    def _shard(self, total):
        from tila_b200.multigpu import shard_range
        return shard_range(total, self.world, self.rank)

    # -- add --
    def _setup_add(self):
        W, torch = self.W, self.torch
        n1 = 1 << 20
        n = n1 * self.mult
        x, y = W.add_inputs(n, seed=0)
        self.host_inputs = [x, y]
        nset = self._sets(3 * 4 * n1)
        self.sets = [(self._dev(x), self._dev(y), torch.empty(n, device=self.device)) for _ in range(nset)]
        grid = (n // 1024,)
        self.axis, self.grid_axis_total = 0, grid[0]
        self.rows_per_program = 1024
        self.launches = [lambda s: W.add_kernel[grid](s[0], s[1], s[2], BLOCK=1024)]
        self.kernels = [W.add_kernel]
        self.out_index = 2
        self.units_per_rank = W.add_bytes(n1)
        self.dominant = 0
        self.dominant_units = W.add_bytes(n1)
        self.metric_unit = ("HBM GB/s", "GB/s", 1e9)
        self.dtype = "f32"
        self.config = {"workload": "add", "N": n1, "BLOCK": 1024, "dtype": "f32"}
        self.e2e_call = lambda xs: (grid, [xs[0], xs[1]], lambda: torch.empty(n, device=self.device),
                                    lambda args, out: W.add_kernel[grid](args[0], args[1], out, BLOCK=1024))

    # -- softmax --
    def _setup_softmax(self):
        W, torch = self.W, self.torch
        m1, ncol = 8192, 1000
        m = m1 * self.mult
        x = W.softmax_inputs(m, ncol, seed=0)
        self.host_inputs = [x]
        nset = self._sets(2 * 4 * m1 * ncol)
        self.sets = [(self._dev(x), torch.empty((m, ncol), device=self.device)) for _ in range(nset)]
        grid = (m,)
        self.axis, self.grid_axis_total = 0, m
        self.rows_per_program = 1
        self.launches = [lambda s: W.softmax_kernel[grid](s[0], s[1], BN=1024)]
        self.kernels = [W.softmax_kernel]
        self.out_index = 1
        self.units_per_rank = W.softmax_bytes(m1, ncol)
        self.dominant = 0
        self.dominant_units = self.units_per_rank
        self.metric_unit = ("HBM GB/s", "GB/s", 1e9)
        self.dtype = "f32"
        self.config = {"workload": "softmax", "M": m1, "N": ncol, "BN": 1024, "dtype": "f32"}
        self.e2e_call = lambda xs: (grid, [xs[0]], lambda: torch.empty((m, ncol), device=self.device),
                                    lambda args, out: W.softmax_kernel[grid](args[0], out, BN=1024))

    # -- matmul --
    def _setup_matmul(self):
        W, torch = self.W, self.torch
        m1 = 4096
        m = m1 * self.mult
        a, b = W.matmul_inputs(m, 4096, 4096, seed=0)
        self.host_inputs = [a, b]
        self.e2e_whole_inputs = {1}       # every rank's programs read all of B
        nset = self._sets(2 * 4096 * 4096 * 2 + 4 * 4096 * 4096)
        self.sets = [(self._dev(a), self._dev(b), torch.empty((m, 4096), device=self.device))
                     for _ in range(nset)]
        grid = (m // 128, 4096 // 128)
        self.axis, self.grid_axis_total = 0, grid[0]
        self.rows_per_program = 128
        self.launches = [lambda s: W.matmul_kernel[grid](s[0], s[1], s[2], BM=128, BN=128, BK=64)]
        self.kernels = [W.matmul_kernel]
        self.out_index = 2
        self.units_per_rank = W.matmul_flops()
        self.dominant = 0
        self.dominant_units = self.units_per_rank
        self.metric_unit = ("f16 TFLOPS", "TFLOP/s", 1e12)
        self.dtype = "f16 in, f32 accumulate"
        self.config = {"workload": "matmul", "M": 4096, "N": 4096, "K": 4096, "BM": 128,
                       "BN": 128, "BK": 64}
        self.e2e_call = lambda xs: (grid, [xs[0], xs[1]],
                                    lambda: torch.empty((m, 4096), device=self.device),
                                    lambda args, out: W.matmul_kernel[grid](args[0], args[1], out,
                                                                           BM=128, BN=128, BK=64))

    # -- unfused attention --
    def _setup_unfused_attention(self):
        W, torch = self.W, self.torch
        bh1, l, d = 128, 1024, 64
        bh = bh1 * self.mult
        q, k, v = W.attention_inputs(bh, l, d, seed=0)
        self.host_inputs = [q, k, v]
        qg, kg, vg = self._dev(q), self._dev(k), self._dev(v)
        s = torch.empty((bh, l, l), device=self.device)
        p = torch.empty_like(s)
        o = torch.empty((bh, l, d), device=self.device)
        self.sets = [(qg, kg, vg, s, p, o)]
        g1, g2, g3 = (l // 128, l // 128, bh), (bh * l,), (l // 128, bh)
        # shard axes: scores by heads (axis 2), softmax by rows (axis 0), pv by heads (axis 1)
        self.multi_shard = [(2, bh), (0, bh * l), (1, bh)]
        self.grid_axis_total, self.rows_per_program = bh, 1     # the output O: one head per program
        self.launches = [
            lambda st: W.attention_scores[g1](st[0], st[1], st[3], 0.125, BM=128, BN=128, BD=64),
            lambda st: W.softmax_kernel[g2](st[3].view(bh * l, l), st[4].view(bh * l, l), BN=1024),
            lambda st: W.attention_pv[g3](st[4], st[2], st[5], BM=128, BN=128, BD=64),
        ]
        self.kernels = [W.attention_scores, W.softmax_kernel, W.attention_pv]
        self.out_index = 5
        self.units_per_rank = W.unfused_flops(bh1, l, d)
        self.bytes_per_rank = W.unfused_bytes(bh1, l, d)
        # algorithmic bytes of each launch: scores (Q, K read, S written),
        # softmax (S read, P written), P @ V (P, V read, O written)
        self.kernel_units = [2 * bh1 * l * d * 2 + bh1 * l * l * 4, 2 * 4 * bh1 * l * l,
                             bh1 * l * l * 4 + bh1 * l * d * 2 + bh1 * l * d * 4]
        self.dominant = 1
        self.dominant_units = self.kernel_units[1]
        self.metric_unit = ("f16 TFLOPS", "TFLOP/s", 1e12)
        self.dtype = "f16 in, f32 accumulate"
        self.config = {"workload": "unfused_attention", "batch": 8, "heads": 16, "seq": l,
                       "head_dim": d, "launches": 3}

        def e2e_launches(args, out):
            # S and P are per-call intermediates (stream-ordered allocations)
            s_ = torch.empty((bh, l, l), device=self.device)
            p_ = torch.empty_like(s_)
            steps = [lambda: W.attention_scores[g1](args[0], args[1], s_, 0.125, BM=128, BN=128, BD=64),
                     lambda: W.softmax_kernel[g2](s_.view(bh * l, l), p_.view(bh * l, l), BN=1024),
                     lambda: W.attention_pv[g3](p_, args[2], out, BM=128, BN=128, BD=64)]
            for (ax, lo, hi), fn in zip(self._ranges(), steps):
                with self.tila_b200.program_range(ax, lo, hi):
                    fn()
        self.e2e_call = lambda xs: (g1, xs, lambda: torch.empty((bh, l, d), device=self.device),
                                    e2e_launches)

    # -- fused attention --
    def _setup_fused_attention(self):
        W, torch = self.W, self.torch
        bh1, l, d = 128, 4096, 128
        bh = bh1 * self.mult
        q, k, v = W.attention_inputs(bh, l, d, seed=0)
        self.host_inputs = [q, k, v]
        self.sets = [(self._dev(q), self._dev(k), self._dev(v),
                      torch.empty((bh, l, d), device=self.device))]
        grid = (l // 128, bh)
        self.axis, self.grid_axis_total = 1, bh
        self.rows_per_program = 1
        scale = d ** -0.5
        self.launches = [lambda s: W.fused_attention_kernel[grid](s[0], s[1], s[2], s[3], scale,
                                                           CAUSAL=0, BM=128, BN=128, BD=128)]
        self.kernels = [W.fused_attention_kernel]
        self.out_index = 3
        self.units_per_rank = W.fused_flops(bh1, l, d)
        self.dominant = 0
        self.dominant_units = self.units_per_rank
        self.metric_unit = ("f16 TFLOPS", "TFLOP/s", 1e12)
        self.dtype = "f16 in, f32 accumulate"
        self.config = {"workload": "fused_attention", "batch": 4, "heads": 32, "seq": l,
                       "head_dim": d, "BM": 128, "BN": 128, "causal": False, "num_warps": 4}
        self.e2e_call = lambda xs: (grid, xs, lambda: torch.empty((bh, l, d), device=self.device),
                                    lambda args, out: W.fused_attention_kernel[grid](*args, out, scale,
                                                                              CAUSAL=0, BM=128, BN=128, BD=128))

    # -- causal fused attention (the CAUSAL=1 kernel of the same example) --
    def _setup_fused_attention_causal(self):
        W, torch = self.W, self.torch
        bh1, l, d = 128, 4096, 128
        bh = bh1 * self.mult
        q, k, v = W.attention_inputs(bh, l, d, seed=0)
        self.host_inputs = [q, k, v]
        self.sets = [(self._dev(q), self._dev(k), self._dev(v),
                      torch.empty((bh, l, d), device=self.device))]
        grid = (l // 128, bh)
        self.axis, self.grid_axis_total = 1, bh
        self.rows_per_program = 1
        scale = d ** -0.5
        # 4 warps per program: the warp-specialised form, two programs per CTA
        # whose two loops (below the diagonal, then the diagonal tile) walk
        # one stream of K/V tiles of per-program length
        causal = W.fused_attention_kernel[grid].with_options(num_warps=4)
        self.launches = [lambda s: causal(s[0], s[1], s[2], s[3], scale, CAUSAL=1, BM=128, BN=128, BD=128)]
        self.kernels = [W.fused_attention_kernel]
        self.out_index = 3
        self.units_per_rank = W.causal_flops(bh1, l, d)
        self.dominant = 0
        self.dominant_units = self.units_per_rank
        self.metric_unit = ("f16 TFLOPS", "TFLOP/s", 1e12)
        self.dtype = "f16 in, f32 accumulate"
        self.config = {"workload": "fused_attention_causal", "batch": 4, "heads": 32, "seq": l,
                       "head_dim": d, "BM": 128, "BN": 128, "causal": True, "num_warps": 4,
                       "flop_count": "half of the non-causal 4*BH*L^2*D"}
        self.e2e_call = lambda xs: (grid, xs, lambda: torch.empty((bh, l, d), device=self.device),
                                    lambda args, out: causal(*args, out, scale, CAUSAL=1,
                                                             BM=128, BN=128, BD=128))

    # -- launching ---------------------------------------------------------

    def _ranges(self):
        if getattr(self, "multi_shard", None):
            return [(ax, *self._shard(total)) for ax, total in self.multi_shard]
        return [(self.axis, *self._shard(self.grid_axis_total))] * len(self.launches)

    def gather_rows(self, out):
        """Leading rows of ``out`` each rank's programs write (the program
        split of the output's launch, times the rows one program writes)."""
        from tila_b200.multigpu import shard_rows
        return shard_rows(self.grid_axis_total, self.rows_per_program, out.shape[0], self.world)

    def prepare(self):
        """Launch every step once through the public API (compiling and
        checking it), and keep the prepared launches for replay."""
        from tila_b200.backend import last_launch
        self.records = []
        ranges = self._ranges()
        for s in self.sets:
            recs = []
            for i, fn in enumerate(self.launches):
                ax, lo, hi = ranges[i]
                with self.tila_b200.program_range(ax, lo, hi):
                    fn(s)
                recs.append(last_launch(self.kernels[i]))
            self.records.append(recs)
        self.torch.cuda.synchronize(self.device)

    def step(self, i):
        for r in self.records[i % len(self.records)]:
            r.launch()


def run_ours(args, world, rank, device, keys):
    import torch
    import torch.distributed as dist
    peaks = _peaks()
    traffic = _traffic_table()
    results = {}
    for key in keys:
        case = Case(key, world, rank, device)
        case.prepare()
        K, Wm = args.steps, args.warmup
        for i in range(Wm):
            case.step(i)
        torch.cuda.synchronize(device)
        # capture the K timed steps in one CUDA graph (no host gaps between launches)
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            case.step(0)
        torch.cuda.synchronize(device)
        with torch.cuda.graph(graph, stream=stream):
            for i in range(K):
                case.step(i)
        torch.cuda.synchronize(device)
        graph.replay()              # one untimed replay
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(device) as clocks:
            # keep the GPU busy around the timed replay so that the clock
            # samples (every 100 ms) see the same load as the timed steps
            cur = torch.cuda.current_stream(device)
            t_end = time.perf_counter() + 0.3
            while time.perf_counter() < t_end:
                graph.replay()
                torch.cuda.synchronize(device)
            # a short device-side spin ahead of the start event keeps the GPU
            # busy while the host submits the graph, so the events bracket the
            # K steps themselves, not the host's graph-launch latency
            torch.cuda._sleep(200_000)
            start.record(cur)
            graph.replay()
            end.record(cur)
            torch.cuda.synchronize(device)
            t_end = time.perf_counter() + 0.2
            while time.perf_counter() < t_end:
                graph.replay()
                torch.cuda.synchronize(device)
        ms_local = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms_local], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_total = float(t.item())
        else:
            ms_total = ms_local
        ms_step = ms_total / K
        name, unit, scale = case.metric_unit
        value = case.units_per_rank * world / (ms_step * 1e-3) / scale
        # multi-launch steps: each kernel in its own graph of K launches,
        # timed with events on the launching stream; the dominant kernel is
        # the one that takes longest
        dom_ms = ms_step
        per_kernel = []
        if len(case.launches) > 1:
            for j in range(len(case.launches)):
                g2 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g2, stream=stream):
                    for i in range(K):
                        case.records[i % len(case.records)][j].launch()
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    g2.replay()
                    e0.record(stream)
                    g2.replay()
                    e1.record(stream)
                torch.cuda.synchronize(device)
                per_kernel.append(e0.elapsed_time(e1) / K)
                del g2
            case.dominant = max(range(len(per_kernel)), key=lambda j: per_kernel[j])
            case.dominant_units = case.kernel_units[case.dominant]
            dom_ms = per_kernel[case.dominant]
        dom_kernel = case.records[0][case.dominant].kernel_name
        if W_ROOF.get(key, "hbm") == "hbm":
            achieved = case.dominant_units / (dom_ms * 1e-3) / 1e9
            peak, runit = peaks["hbm_gbs"], "GB/s"
        else:
            achieved = case.dominant_units / (dom_ms * 1e-3) / 1e12
            peak, runit = peaks["bf16_tflops"], "TFLOP/s"
        tr = traffic.get(f"{dom_kernel}@{key}") or traffic.get(dom_kernel)
        roof = {"bound": W_ROOF.get(key, "hbm"), "kernel": dom_kernel, "achieved": round(achieved, 2),
                "peak": peak, "unit": runit, "frac": round(achieved / peak, 4),
                "traffic": tr.get("bytes_per_launch") if tr else None,
                "algorithmic": case.dominant_units, "peak_source": peaks["source"]}
        if runit == "TFLOP/s" and peaks.get("bf16_tflops_sustained"):
            # the timed steps follow 0.3 s of load (clocks at the power cap):
            # the sustained GEMM figure is reported beside the burst one
            sus = peaks["bf16_tflops_sustained"]
            roof.update(peak_kind="burst", peak_sustained=sus, frac_sustained=round(achieved / sus, 4))
        # NCCL gather of the output shards to rank 0 (timed separately)
        gather_ms = None
        if world > 1:
            out = case.sets[0][case.out_index]
            gather_ms = _gather(out, case, world, rank, device)
        # every timed launch wrote its device errors (bounded-wait timeouts)
        # into the error block; a run with one is not a measurement
        errors = case.tila_b200.read_device_errors(device)
        if errors:
            from tila_b200.backend import describe_error
            raise RuntimeError(f"{key}: a timed launch recorded a device error: {describe_error(errors)}")
        entry = {"metric": name, "value": round(value, 3), "unit": unit, "ms_per_step": round(ms_step, 5),
                 "steps": K, "gpu_launches": K * len(case.launches), "device_errors": 0,
                 "roofline": roof, "config": case.config, "clocks": clocks.summary(),
                 "dtype": case.dtype}
        if key == "unfused_attention":
            entry["hbm_gbs"] = round(case.bytes_per_rank * world / (ms_step * 1e-3) / 1e9, 2)
        if per_kernel:
            entry["kernels"] = {case.records[0][j].kernel_name: {
                "ms": round(per_kernel[j], 5),
                "gbs": round(case.kernel_units[j] / (per_kernel[j] * 1e-3) / 1e9, 1)}
                for j in range(len(per_kernel))}
        if gather_ms is not None:
            entry["gather_ms"] = round(gather_ms, 4)
        del graph
        if case.e2e_call is not None and not args.no_e2e:
            entry["e2e"] = _e2e(case, args, world, rank, device)
        if rank == 0 and world == 1 and not args.no_cpu:
            entry["cpu_baseline"] = cpu_reference(key, keys, steps=1)
        if gather_ms is not None:
            # the same steps followed by the gather (weak scaling, the gather
            # measured above; device times added)
            entry["with_gather"] = {
                "value": round(case.units_per_rank * world / ((ms_step + gather_ms) * 1e-3) / scale, 3),
                "ms_per_step": round(ms_step + gather_ms, 5)}
        results[key] = entry
        del case
        torch.cuda.empty_cache()
        if world > 1:
            entry["strong"] = _strong(key, args, world, rank, device)
            torch.cuda.empty_cache()
    return results


def _strong(key, args, world, rank, device):
    """Strong scaling: the configuration itself (not N copies) split N ways.
    Each timed step is this rank's share of the launches followed by the NCCL
    all-gather (C ABI) that leaves the whole output on every rank; device
    time of K steps with CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    from tila_b200.multigpu import gather_leading
    case = Case(key, world, rank, device, strong=True)
    case.prepare()
    comm = _communicator(world, rank, device)

    def step(i):
        case.step(i)
        out = case.sets[i % len(case.sets)][case.out_index]
        gather_leading(out, world, rank, rows=case.gather_rows(out), comm=comm)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)
    dist.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(i)
    e1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    name, unit, scale = case.metric_unit
    res = {"value": round(case.units_per_rank / (ms * 1e-3) / scale, 3), "unit": unit,
           "ms_per_step": round(ms, 5), "steps": args.steps, "gather_included": True,
           "split": f"{case.grid_axis_total} programs of axis {case.axis if not getattr(case, 'multi_shard', None) else 'per launch'} over {world} ranks"}
    del case
    return res


W_ROOF = {"add": "hbm", "softmax": "hbm", "matmul": "tensor", "unfused_attention": "hbm",
          "fused_attention": "tensor", "fused_attention_causal": "tensor"}


_COMM = {}


def _communicator(world, rank, device):
    """The C-ABI NCCL communicator (tila_mg_*) of this run, created once."""
    from tila_b200.multigpu import Communicator
    if "comm" not in _COMM:
        _COMM["comm"] = Communicator(world, rank, device)
    return _COMM["comm"]


def _gather(out, case, world, rank, device):
    """NCCL all-gather (through the library's C ABI) of the output rows each
    rank computed, timed on the device, max over ranks."""
    import torch
    import torch.distributed as dist
    from tila_b200.multigpu import gather_leading
    comm = _communicator(world, rank, device)
    rows = case.gather_rows(out)
    gather_leading(out, world, rank, rows=rows, comm=comm)     # first call sets up NCCL's buffers
    dist.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gather_leading(out, world, rank, rows=rows, comm=comm)
    e1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _e2e(case, args, world, rank, device):
    """Public-API time: every step copies its inputs host-to-device from pinned
    memory, launches ``kernel[grid](...)`` (Tila's contract checks included)
    and reads its output back.  Consecutive steps are pipelined over two
    buffer sets on three streams (copy-in, compute, copy-out), the way a
    serving loop overlaps PCIe traffic in both directions with kernels."""
    import torch
    import torch.distributed as dist
    grid, inputs, make_out, call = case.e2e_call(case.host_inputs)
    pinned = [torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in inputs]
    dev_in = [[torch.empty(p.shape, dtype=p.dtype, device=device) for p in pinned] for _ in range(2)]
    outs = [make_out(), make_out()]
    host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    ax, lo, hi = case._ranges()[0]
    # this rank's leading rows: the output rows its programs write, which are
    # also the input rows they read (inputs every program reads whole, such
    # as matmul's B, travel whole); each rank moves only its own share
    r0, r1 = case.gather_rows(outs[0])[rank]
    whole = getattr(case, "e2e_whole_inputs", set())
    in_rows = [slice(None) if i in whole else slice(r0, r1) for i in range(len(pinned))]
    # enough steps that the pipeline's fill (the first copy-in) and drain (the
    # last copy-out), both inside the timed region, weigh little
    steps = max(8, min(4 * args.steps, 48))
    s_in, s_comp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    ev = lambda: torch.cuda.Event()
    in_ready = [ev(), ev()]      # inputs of set b copied
    in_free = [ev(), ev()]       # the kernel reading set b finished
    out_ready = [ev(), ev()]     # output of set b written
    out_free = [ev(), ev()]      # output of set b copied back
    for b in range(2):
        for e, st in ((in_free[b], s_comp), (out_free[b], s_out)):
            e.record(st)

    # each set's copy views (destination, source), sliced once
    in_copies = [[(d[rows], p[rows]) for p, d, rows in zip(pinned, dev_in[b], in_rows)] for b in range(2)]
    out_copies = [(host_out[b][r0:r1], outs[b][r0:r1]) for b in range(2)]

    def step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[b])
            for d, p in in_copies[b]:
                d.copy_(p, non_blocking=True)
            in_ready[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_ready[b])
            s_comp.wait_event(out_free[b])
            with case.tila_b200.program_range(ax, lo, hi):
                call(dev_in[b], outs[b])
            in_free[b].record(s_comp)
            out_ready[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(out_ready[b])
            out_copies[b][0].copy_(out_copies[b][1], non_blocking=True)
            out_free[b].record(s_out)

    for i in range(2):
        step(i)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    # device time from the first copy-in to the last copy-out, max over ranks
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    t_host = time.perf_counter()
    for i in range(steps):
        step(i)
    t_host = time.perf_counter() - t_host
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_comp)
    e1.record(s_out)
    torch.cuda.synchronize(device)
    dt = e0.elapsed_time(e1) * 1e-3 / steps
    if world > 1:
        t = torch.tensor([dt], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    name, unit, scale = case.metric_unit
    h2d = sum(p[rows].numel() * p.element_size() for p, rows in zip(pinned, in_rows)) * world
    d2h = host_out[0][r0:r1].numel() * host_out[0].element_size() * world
    return {"value": round(case.units_per_rank * world / dt / scale, 3), "unit": unit,
            "ms_per_step": round(dt * 1e3, 3), "steps": steps,
            # host time to issue one step (the kernel[grid] call, the copies
            # and the stream events); a step cannot take less on the device
            # once the host is the slower side
            "host_ms_per_step": round(t_host * 1e3 / steps, 3),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "pipelining": "two buffer sets, copy-in / compute / copy-out streams"
                          + ("; each rank copies its own rows, bytes summed over ranks" if world > 1 else "")}


# ---------------------------------------------------------------------------
# CPU: Tila's NumPy reference interpreter on every host core
# ---------------------------------------------------------------------------
#
# The interpreter runs one program after another in one Python thread, so it
# uses the host's cores through processes: a spawned pool of one worker per
# core (one BLAS thread each), every worker holding the seeded inputs of each
# workload's per-step sample and running a contiguous share of the sample's
# program axis through ``kernel[grid](numpy arrays)`` - the reference's own
# launch path, contract checks included.  A step is one pass over the whole
# sample; its rate is the sample's work over the step's wall time.

# per workload: (length of the sample's program axis, what the sample is)
_REF_SAMPLE = {
    "add": (1024, "full workload (N=1048576, 1024 programs of 1024)"),
    "softmax": (8192, "full workload (8192 rows of 1000, BN=1024)"),
    "matmul": (16, "16 of the 32 rows of 128x128 output tiles (C 2048x4096, full K=4096)"),
    "unfused_attention": (16, "16 of the 128 batch*heads (L=1024, D=64)"),
    "fused_attention": (16, "16 of the 128 batch*heads (L=4096, D=128)"),
    "fused_attention_causal": (16, "16 of the 128 batch*heads (L=4096, D=128, causal)"),
}
_REF_DATA = {}
_REF_POOL = []


def _ref_units(key):
    from tila_b200 import workloads as W
    n = _REF_SAMPLE[key][0]
    return {"add": (W.add_bytes(n * 1024), "GB/s", 1e9),
            "softmax": (W.softmax_bytes(n, 1000), "GB/s", 1e9),
            "matmul": (W.matmul_flops(n * 128, 4096, 4096), "TFLOP/s", 1e12),
            "unfused_attention": (W.unfused_flops(n, 1024, 64), "TFLOP/s", 1e12),
            "fused_attention": (W.fused_flops(n, 4096, 128), "TFLOP/s", 1e12),
            "fused_attention_causal": (W.causal_flops(n, 4096, 128), "TFLOP/s", 1e12)}[key]


def _ref_init(keys):
    """Pool worker start: the seeded inputs of the samples of ``keys`` (the
    same generators and seeds as the GPU arm), then one launch of each kernel on
    one entry of the program axis, so that Tila's per-process first-call
    work (decoration, TIR) stays out of the timed steps.  A failure is kept
    and raised by every task (a raising initializer would make the pool
    restart the worker for ever)."""
    def zeros(shape):
        z = np.empty(shape, np.float32)
        z.fill(0.0)             # every page mapped now, not in a timed pass
        return z

    try:
        from tila_b200 import workloads as W
        if "add" in keys:
            x, y = W.add_inputs(1024 * 1024)
            _REF_DATA["add"] = (x, y, zeros(x.shape))
        if "softmax" in keys:
            x = W.softmax_inputs(8192, 1000)
            _REF_DATA["softmax"] = (x, zeros(x.shape))
        if "matmul" in keys:
            a, b = W.matmul_inputs(16 * 128, 4096, 4096)
            _REF_DATA["matmul"] = (a, b, zeros((16 * 128, 4096)))
        if "unfused_attention" in keys:
            q, k, v = W.attention_inputs(16, 1024, 64)
            _REF_DATA["unfused_attention"] = (q, k, v, zeros((16, 1024, 1024)), zeros((16, 1024, 1024)),
                                              zeros((16, 1024, 64)))
        if {"fused_attention", "fused_attention_causal"} & set(keys):
            q, k, v = W.attention_inputs(16, 4096, 128)
            _REF_DATA["fused_attention"] = _REF_DATA["fused_attention_causal"] = \
                (q, k, v, zeros((16, 4096, 128)))
        for key in keys:
            _ref_run(key, 0, 1)
    except Exception as exc:        # noqa: BLE001 - reported by _ref_run
        _REF_DATA["error"] = f"{type(exc).__name__}: {exc}"


def _ref_run(key, lo, hi):
    """Pool worker: run the interpreter on entries [lo, hi) of the sample's
    program axis (each a contiguous slice of the inputs, launched with the
    grid that slice calls for).  Returns the seconds taken."""
    from tila_b200 import workloads as W
    if "error" in _REF_DATA:
        raise RuntimeError("reference worker setup failed: " + _REF_DATA["error"])
    d = _REF_DATA[key]
    h = hi - lo
    t0 = time.perf_counter()
    if key == "add":
        x, y, o = (t[lo * 1024:hi * 1024] for t in d)
        W.add_kernel[(h,)](x, y, o, BLOCK=1024)
    elif key == "softmax":
        x, o = (t[lo:hi] for t in d)
        W.softmax_kernel[(h,)](x, o, BN=1024)
    elif key == "matmul":
        a, b, c = d
        W.matmul_kernel[(h, 32)](a[lo * 128:hi * 128], b, c[lo * 128:hi * 128], BM=128, BN=128, BK=64)
    elif key == "unfused_attention":
        q, k, v, s, p, o = (t[lo:hi] for t in d)
        W.attention_scores[(8, 8, h)](q, k, s, 0.125, BM=128, BN=128, BD=64)
        W.softmax_kernel[(h * 1024,)](s.reshape(h * 1024, 1024), p.reshape(h * 1024, 1024), BN=1024)
        W.attention_pv[(8, h)](p, v, o, BM=128, BN=128, BD=64)
    else:
        q, k, v, o = (t[lo:hi] for t in d)
        W.fused_attention_kernel[(32, h)](q, k, v, o, 128 ** -0.5,
                                          CAUSAL=int(key == "fused_attention_causal"), BM=128, BN=128, BD=128)
    return time.perf_counter() - t0


# A worker holds Tila, NumPy and torch (about 0.55 GB) plus the samples' inputs
# (about 0.4 GB); past this many workers the host memory they take grows
# faster than the interpreter's rate.
_REF_MAX_WORKERS = 32


def _ref_workers():
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    return max(1, min(cores, _REF_MAX_WORKERS))


def _ref_pool(keys):
    """The worker pool for the workloads ``keys`` (spawned, never forked: the
    parent may hold a CUDA context), started once; the workers inherit one
    BLAS thread each and Tila's race analysis switched off, which the
    parent's own environment does not keep."""
    if not _REF_POOL:
        import multiprocessing as mp
        env = {"OMP_NUM_THREADS": "1", "OPENBLAS_NUM_THREADS": "1", "MKL_NUM_THREADS": "1",
               "TILA_RACE": "off"}
        saved = {k: os.environ.get(k) for k in env}
        os.environ.update(env)
        try:
            n = _ref_workers()
            _REF_POOL.append((mp.get_context("spawn").Pool(n, initializer=_ref_init,
                                                            initargs=(tuple(keys),)), n))
            atexit.register(_ref_close)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
    return _REF_POOL[0]


def _ref_shards(length, parts):
    """Contiguous, nearly equal ranges [lo, hi) covering range(length)."""
    cuts = [length * i // parts for i in range(parts + 1)]
    return [(lo, hi) for lo, hi in zip(cuts, cuts[1:]) if hi > lo]


def _ref_close():
    """Stop the workers before the interpreter shuts down (a pool collected
    during shutdown fails in its finaliser)."""
    while _REF_POOL:
        pool, _ = _REF_POOL.pop()
        pool.terminate()
        pool.join()


def cpu_reference(key, keys, steps=1, min_seconds=1.0):
    """Tila's interpreter on all host cores: one untimed pass over the
    sample, then timed passes, at least ``steps`` of them and at least
    ``min_seconds`` in all (short samples get several passes); the median
    pass gives the rate in the workload's unit.  ``keys``: every workload
    of this run (the pool, started by the first call, prepares them all)."""
    pool, n = _ref_pool(keys)
    length, desc = _REF_SAMPLE[key]
    shards = [(key, lo, hi) for lo, hi in _ref_shards(length, n)]
    pool.starmap(_ref_run, shards, chunksize=1)
    times = []
    while len(times) < max(1, steps) or (sum(times) < min_seconds and len(times) < 100):
        t0 = time.perf_counter()
        pool.starmap(_ref_run, shards, chunksize=1)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    units, unit, scale = _ref_units(key)
    return {"value": units / dt / scale, "unit": unit, "cores": len(shards), "kind": "reference",
            "sample": f"Tila NumPy interpreter, {desc}, split over {len(shards)} worker processes "
                      f"(one BLAS thread each) on {len(shards)} of {os.cpu_count()} host cores; "
                      f"median of {len(times)} pass(es) of {dt:.3f} s"}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="softmax", choices=ORDER)
    ap.add_argument("--only", action="store_true", help="measure the headline workload only")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = _dist_env()
    keys = [args.workload] + ([] if args.only else [k for k in ORDER if k != args.workload])

    if args.impl == "reference":
        if rank != 0:
            return
        out = {}
        for key in keys:
            base = cpu_reference(key, keys, steps=min(args.steps, 3))
            v = base["value"]
            out[key] = {"value": v, "unit": base["unit"], "cpu_baseline": base,
                        "e2e": {"value": v, "unit": base["unit"], "h2d_bytes_per_step": 0,
                                "d2h_bytes_per_step": 0}}
        head = out[keys[0]]
        line = {"impl": "reference", "metric": _metric_name(keys[0]), "value": head["value"],
                "unit": head["unit"], "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": _dtype(keys[0]), "data": "synthetic (seeded)",
                "config": _config(keys[0]), "cpu_baseline": head["cpu_baseline"],
                "e2e": head["e2e"], "workloads": {k: v for k, v in out.items() if k != keys[0]}}
        print(json.dumps(line))
        return

    import torch
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    import tila_b200  # noqa: F401
    try:
        res = run_ours(args, world, rank, device, keys)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
    if rank == 0:
        head = res[keys[0]]
        line = {"metric": head["metric"], "value": head["value"], "unit": head["unit"],
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": head["dtype"],
                "data": "synthetic (seeded NumPy inputs of the configured shapes)",
                "config": dict(head["config"], parallelism=f"grid-partitioned x{world}",
                               l2="inputs rotated across buffer sets larger than L2"),
                "roofline": head["roofline"], "clocks": head["clocks"],
                "gpu_launches": head["gpu_launches"]}
        for k in ("e2e", "cpu_baseline", "gather_ms", "with_gather", "strong", "hbm_gbs",
                  "device_errors"):
            if k in head:
                line[k] = head[k]
        line["workloads"] = {k: v for k, v in res.items() if k != keys[0]}
        print(json.dumps(line))
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        if "comm" in _COMM:
            _COMM.pop("comm").close()
        dist.destroy_process_group()


def _metric_name(key):
    return "HBM GB/s" if W_ROOF[key] == "hbm" and key != "unfused_attention" else "f16 TFLOPS"


def _dtype(key):
    return "f32" if key in ("add", "softmax") else "f16 in, f32 accumulate"


def _config(key):
    return {"add": {"workload": "add", "N": 1 << 20, "BLOCK": 1024},
            "softmax": {"workload": "softmax", "M": 8192, "N": 1000, "BN": 1024},
            "matmul": {"workload": "matmul", "M": 4096, "N": 4096, "K": 4096},
            "unfused_attention": {"workload": "unfused_attention", "batch": 8, "heads": 16,
                                  "seq": 1024, "head_dim": 64},
            "fused_attention": {"workload": "fused_attention", "batch": 4, "heads": 32,
                                "seq": 4096, "head_dim": 128}}[key]


if __name__ == "__main__":
    main()
