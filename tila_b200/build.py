"""Builds the native part of the backend.

* ``libtila_b200.so``: the C-ABI launcher (csrc/launcher.cpp), linked
  against NVRTC; libcuda is opened at run time.
* a compile check of the tile library for sm_100a with nvcc;
* optionally, the cubins of the five benchmarked workloads (NVRTC works without
  a GPU), so that a fresh GPU machine does not spend its first launches
  compiling.

Run as ``python -m tila_b200.build [--warm]``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def build_library(verbose=False) -> Path:
    """nvcc build of the C-ABI library: the launcher (host C++) and the
    no-allocation entry point (a .cu with a device array, sm_100a)."""
    out = PKG / "libtila_b200.so"
    srcs = [PKG / "csrc" / "launcher.cpp", PKG / "csrc" / "noalloc.cu", PKG / "csrc" / "mg.cpp"]
    hdr = ROOT / "include" / "tila_b200.h"
    if out.exists() and out.stat().st_mtime > max([p.stat().st_mtime for p in srcs] + [hdr.stat().st_mtime]):
        return out
    cmd = [str(CUDA / "bin" / "nvcc"), "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", f"-I{CUDA / 'include'}",
           *[str(p) for p in srcs], f"-L{CUDA / 'lib64'}", "-lnvrtc", "-ldl",
           "-Xlinker", f"-rpath,{CUDA / 'lib64'}", "-o", str(out) + ".tmp"]
    subprocess.run(cmd, check=True, capture_output=not verbose)
    os.replace(str(out) + ".tmp", out)
    return out


def check_tile_library():
    """nvcc compile of every tile header for sm_100a (catches PTX errors)."""
    with tempfile.TemporaryDirectory() as d:
        cu = Path(d) / "tile_check.cu"
        cu.write_text('#include "tila_tile.cuh"\n'
                      'extern "C" __global__ void tila_tile_check(float* x) {\n'
                      '  x[threadIdx.x] = tila::max_nan(x[0], tila::round_f16(x[1]));\n}\n')
        cmd = [str(CUDA / "bin" / "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a",
               "-lineinfo", "-O3", "-fmad=false", f"-I{PKG / 'csrc' / 'tile'}", "-c", str(cu),
               "-o", str(Path(d) / "tile_check.o")]
        subprocess.run(cmd, check=True, capture_output=True)


REFERENCE_TREE = "tila_reference_tree"


def ensure_reference_install(src=None):
    """Install Tila (the package this backend plugs into) into
    ``baseline/_ref`` from a read-only Tila source tree ``src`` (a checkout
    with ``pyproject.toml``; default: ``$TILA_REFERENCE_SRC``) when it is
    missing, and copy the tree's ``examples/``, ``tests/`` and ``tools/``
    beside the package (``baseline/_ref/tila_reference_tree``).  The example
    kernels are what the benchmark and the parity tests launch unchanged, and
    the GPU suites under ``tests/`` (which replay failures with
    ``tools/replay_backend.py``) are run against this backend; none of them is
    part of the installed wheel.  Returns the install directory, or None when neither
    an install nor a source tree is available."""
    target = ROOT / "baseline" / "_ref"
    tree = target / REFERENCE_TREE
    have_pkg = (target / "tila" / "__init__.py").exists()
    parts = ("examples", "tests", "tools")
    have_tree = all((tree / part).is_dir() for part in parts)
    if have_pkg and have_tree:
        return target
    src = src or os.environ.get("TILA_REFERENCE_SRC")
    if not src or not (Path(src) / "pyproject.toml").exists():
        return target if have_pkg else None
    src = Path(src)
    if not have_pkg:
        with tempfile.TemporaryDirectory() as d:
            tmp = Path(d) / "tila_src"
            shutil.copytree(src, tmp, ignore=shutil.ignore_patterns(".git"))
            subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                            "--no-deps", "--target", str(target), str(tmp)],
                           check=True, capture_output=True)
    if not have_tree:
        staging = target / (REFERENCE_TREE + ".tmp")
        shutil.rmtree(staging, ignore_errors=True)
        for part in parts:
            shutil.copytree(src / part, staging / part,
                            ignore=shutil.ignore_patterns("__pycache__", "*.pyc", ".pytest_cache"))
        shutil.rmtree(tree, ignore_errors=True)
        os.replace(staging, tree)
    return target


def warm_cubins():
    """Generate and compile the five workloads' kernels into the cubin cache."""
    import torch
    from . import workloads as W
    from .backend import binding_facts
    from .codegen.emitter import KernelEmitter
    from . import native
    f16, f32 = torch.float16, torch.float32
    cases = [
        (W.add_kernel, dict(x=torch.zeros(1 << 20), y=torch.zeros(1 << 20), out=torch.zeros(1 << 20)),
         dict(BLOCK=1024)),
        (W.softmax_kernel, dict(x=torch.zeros(8, 1000), o=torch.zeros(8, 1000)), dict(BN=1024)),
        (W.matmul_kernel, dict(a=torch.zeros(256, 256, dtype=f16), b=torch.zeros(256, 256, dtype=f16),
                              c=torch.zeros(256, 256)), dict(BM=128, BN=128, BK=64)),
        (W.attention_scores, dict(q=torch.zeros(2, 256, 64, dtype=f16), k=torch.zeros(2, 256, 64, dtype=f16),
                                  s=torch.zeros(2, 256, 256)), dict(BM=128, BN=128, BD=64)),
        (W.attention_pv, dict(p=torch.zeros(2, 256, 256), v=torch.zeros(2, 256, 64, dtype=f16),
                              o=torch.zeros(2, 256, 64)), dict(BM=128, BN=128, BD=64)),
        (W.fused_attention_kernel, dict(q=torch.zeros(2, 256, 128, dtype=f16), k=torch.zeros(2, 256, 128, dtype=f16),
                                 v=torch.zeros(2, 256, 128, dtype=f16), o=torch.zeros(2, 256, 128)),
         dict(CAUSAL=0, BM=128, BN=128, BD=128)),
    ]
    names = []
    for jf, tensors, consts in cases:
        facts = binding_facts(jf.tk, tensors)
        spec = KernelEmitter(jf.tk, consts, facts, num_warps=4).generate()
        native.compile_spec(spec)
        names.append(spec.name)
    return names


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    build_library(verbose=True)
    check_tile_library()
    if "--warm" in argv:
        print("compiled:", ", ".join(warm_cubins()))


if __name__ == "__main__":
    main()
