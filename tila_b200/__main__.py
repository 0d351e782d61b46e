"""``python -m tila_b200 build`` - the B200 counterpart of ``tila build``.

Writes, for every ``@ti.jit`` kernel of a Tila source file, the CUDA C++
this backend generates (``<kernel>.cu``), its TIR (``<kernel>.tir.txt``,
as ``tila build`` writes it, cli.py:163-173), a source map from generated
lines to Tila source lines (``<kernel>.map.json``) and, with ``--cubin``, the
sm_100a cubin NVRTC produces.  Bindings are not known at build time, so the
code assumes contiguous buffers whose base addresses are 16-byte aligned
(launches specialise on the actual bindings).

    python -m tila_b200 build examples/add_kernel.py -o build/ [--const NAME=V] [--cubin]
"""

from __future__ import annotations

import argparse
import json
import os
import sys


def _default_facts(tk):
    """Binding facts for build-time code: contiguous, 16-byte aligned buffers
    whose row strides are multiples of 16 bytes - the bindings the
    benchmarked kernels receive, so f16/f32 buffers of rank 2 and more get
    the TMA/tcgen05 plans that such a launch gets (backend.binding_facts)."""
    from .codegen.emitter import BufferInfo
    out = {}
    for p in list(tk.buffers) + list(tk.ptr_params):
        dt = p.vtype.elem
        rank = len(getattr(p.vtype, "dims", ()) or ()) or 1
        is_ptr = p in tk.ptr_params
        out[p.name] = BufferInfo(name=p.name, dtype=dt, rank=rank, unit_last=True,
                                 stride_div=(16,) * (rank - 1) + (1,), base_align=16,
                                 writable=p.vtype.access is not None and
                                 getattr(p.vtype.access, "name", "") != "READ_ONLY",
                                 is_ptr=is_ptr,
                                 tma_ok=(not is_ptr and rank >= 2 and dt is not None
                                         and dt.name in ("f16", "f32")))
    return out


def build(path, out_dir, const_args=(), cubin=False, num_warps=4):
    from ._reference import tila
    from tila import cli as tila_cli
    from .codegen.emitter import KernelEmitter
    from . import native
    mod = tila_cli._load(path)
    kerns = tila_cli._jit_functions(mod)
    if not kerns:
        print(f"{path}: no @ti.jit kernels found")
        return 1
    os.makedirs(out_dir, exist_ok=True)
    for name, k in kerns.items():
        consts = tila_cli._consts(list(const_args), k.tk.consts)
        _, tir = k.materialize(consts)
        full = dict(consts)
        for c in k.tk.consts:
            if c.name not in full and getattr(c, "default", None) is not None:
                full[c.name] = c.default
        spec = KernelEmitter(k.tk, full, _default_facts(k.tk), num_warps=num_warps,
                             source_map=True).generate()
        smap = {}
        for i, line in enumerate(spec.source.splitlines(), start=1):
            s = line.strip()
            if s.startswith("// @tila-line "):
                smap[i] = int(s.split()[-1])
        with open(os.path.join(out_dir, f"{name}.cu"), "w", encoding="utf-8") as f:
            f.write(spec.source)
        with open(os.path.join(out_dir, f"{name}.tir.txt"), "w", encoding="utf-8") as f:
            f.write(tir)
        with open(os.path.join(out_dir, f"{name}.map.json"), "w", encoding="utf-8") as f:
            json.dump({"kernel": spec.name, "threads": spec.threads, "smem_bytes": spec.smem_bytes,
                       "tmem_cols": spec.tmem_cols, "source": os.path.abspath(path),
                       "cuda_line_to_tila_line": smap}, f, indent=1)
        wrote = [f"{name}.cu", f"{name}.tir.txt", f"{name}.map.json"]
        if cubin:
            data = native.compile_spec(spec)
            with open(os.path.join(out_dir, f"{name}.cubin"), "wb") as f:
                f.write(data)
            wrote.append(f"{name}.cubin")
        print(f"{name}: wrote {out_dir}/" + ", ".join(wrote))
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m tila_b200")
    ap.add_argument("command", choices=["build"])
    ap.add_argument("path")
    ap.add_argument("-o", "--out", default="build")
    ap.add_argument("--const", action="append", metavar="NAME=V", default=[])
    ap.add_argument("--cubin", action="store_true", help="also compile the sm_100a cubin (NVRTC)")
    ap.add_argument("--num-warps", type=int, default=4)
    args = ap.parse_args(argv)
    from ._reference import tila
    try:
        return build(args.path, args.out, args.const, args.cubin, args.num_warps)
    except tila.errors.TilaError as e:
        print(e.render(), file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())
