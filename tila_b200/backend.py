"""Execution of checked Tila kernels on B200 (the replacement of the Triton
branch of ``_Launcher._execute``, runtime.py:1062-1108).

Per launch: derive the binding facts that specialise code generation
(dtypes, unit last-dim strides, stride and base-address divisibility), look
up or build the kernel (TIR -> CUDA C++ -> NVRTC cubin -> CUlibrary), check
its resources against the device (backend.preflight, backend.py:61-88), and
launch it on the current PyTorch stream through the C ABI.  Compile and load
failures raise ``TILA-TARGET-010`` with a replayable artifact, resource
overflows ``TILA-TARGET-011``, unsupported TIR ``TILA-TARGET-009``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from contextlib import contextmanager
from dataclasses import dataclass, asdict

import importlib

from ._reference import tila
from . import native

_tila_backend = importlib.import_module("tila.backend")
from .codegen.emitter import BufferInfo, CodegenError, KernelEmitter

TilaError = tila.errors.TilaError
Loc = tila.errors.Loc
_runtime = tila.runtime

SCALAR_CTYPES = {
    "bool": ctypes.c_uint8, "i8": ctypes.c_int8, "i16": ctypes.c_int16, "i32": ctypes.c_int32,
    "i64": ctypes.c_int64, "u8": ctypes.c_uint8, "u16": ctypes.c_uint16, "u32": ctypes.c_uint32,
    "u64": ctypes.c_uint64, "f32": ctypes.c_float, "f64": ctypes.c_double,
}

# ---------------------------------------------------------------------------
# launch sharding (multi-GPU): a thread-local program-range restriction
# ---------------------------------------------------------------------------

_shard = threading.local()


@contextmanager
def program_range(axis: int, start: int, stop: int):
    """Restrict B200 launches inside the block to programs with
    ``start <= program_id(axis) < stop``.  Launch contracts and proofs still
    run on the full grid, and ``program_id``/``num_programs`` keep their
    global values, so each shard computes exactly its programs' outputs."""
    prev = getattr(_shard, "value", None)
    _shard.value = (int(axis), int(start), int(stop))
    try:
        yield
    finally:
        _shard.value = prev


def current_program_range():
    return getattr(_shard, "value", None)


# ---------------------------------------------------------------------------
# device errors
# ---------------------------------------------------------------------------
#
# Every generated kernel takes a 16-byte error block (include/tila_b200.h,
# TILA_ERROR_BLOCK_BYTES): the first device error of a launch - a bounded
# wait that timed out, a failed tensor-memory allocation, a false ti.assume in
# a debug build - is recorded there with its Tila source line, and the thread
# that records it also stores it into a page-locked host word whose device
# address the block carries.  The host reads that word without synchronising:
# every launch on the device first checks it and raises TILA-TARGET-005 for an
# error an earlier launch recorded, so a kernel that stopped early is never
# taken for a result by the next step.  ``check_device_errors`` does the same
# check on demand; ``read_device_errors`` synchronises and reads the block.

ERROR_CODES = {
    1: "a bounded wait on an mbarrier timed out (a TMA copy, tensor-core commit or "
       "partner warpgroup never arrived); the program stopped early and its outputs are incomplete",
    2: "tensor memory allocation failed",
    3: "a ti.assume predicate was false (TILA_DEBUG=1 build)",
    4: "the loops of a warp-specialised kernel did not cover one contiguous range of iterations "
       "at run time (a loop ended before it started); the kernel's outputs are incomplete",
}


class _ErrorBlock:
    def __init__(self, device):
        import torch
        self.device = device
        self.block = torch.zeros(native.ERROR_BLOCK_BYTES // 4, dtype=torch.int32, device=device)
        with torch.cuda.device(device):
            self.host, addr = native.host_word_alloc()
        self.block.view(torch.int64)[1] = addr
        self.word = ctypes.c_uint32.from_address(self.host)

    def pending(self) -> int:
        return self.word.value

    def clear(self):
        """Stream-ordered reset of the block's error word and of the host word."""
        self.word.value = 0
        self.block[0].zero_()


_err_blocks = {}


def _error_block(device) -> _ErrorBlock:
    b = _err_blocks.get(device.index)
    if b is None:
        b = _err_blocks[device.index] = _ErrorBlock(device)
    return b


def _error_word(device):
    """The error block tensor passed to every launch on ``device``."""
    return _error_block(device).block


def describe_error(word: int) -> str:
    code, line = word >> 24, word & 0xFFFFFF
    what = ERROR_CODES.get(code, f"device error code {code}")
    return f"{what} (Tila source line {line})"


def check_device_errors(device=None) -> None:
    """Raise ``TILA-TARGET-005`` if a kernel launched on ``device`` has
    recorded a device error that no one has read yet.  Does not synchronise:
    it sees errors of kernels that have reached them."""
    import torch
    idx = torch.cuda.current_device() if device is None else torch.device(device).index
    b = _err_blocks.get(idx)
    if b is None:
        return
    word = b.pending()
    if word:
        b.clear()
        _reset_streamk_flags(torch.device("cuda", idx))
        raise TilaError("TILA-TARGET-005", "a kernel launched earlier on this device failed",
                        Loc(word & 0xFFFFFF),
                        details=[f"device: cuda:{idx}", f"error: {describe_error(word)}"],
                        fixes=["the outputs of that launch are incomplete: launch it again"])


def read_device_errors(device=None, reset=True) -> int:
    """Synchronise and return the first in-kernel error recorded on ``device``
    (0 = none; high byte = code, low 24 bits = Tila source line; see
    ``ERROR_CODES``).  ``reset`` clears it."""
    import torch
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    b = _err_blocks.get(device.index)
    if b is None:
        return 0
    val = int(b.block[0].item()) & 0xFFFFFFFF
    if reset and (val or b.pending()):
        b.clear()
        _reset_streamk_flags(device)
    return val


# ---------------------------------------------------------------------------
# compiled kernels
# ---------------------------------------------------------------------------

@dataclass
class Compiled:
    spec: object
    library: object
    kernel: object
    attrs: dict = None


def _pow2_div(v, cap):
    v = abs(int(v))
    if v == 0:
        return cap
    d = 1
    while v % (d * 2) == 0 and d < cap:
        d *= 2
    return d


def binding_facts(tk, tensors) -> dict:
    """Launch facts that specialise the generated code (a coarse, value-free
    projection of runtime._binding_signature, runtime.py:1221-1231)."""
    out = {}
    for p in list(tk.buffers) + list(tk.ptr_params):
        t = tensors[p.name]
        dt = _runtime._tensor_info(t)[0]
        strides = tuple(int(s) for s in t.stride())
        is_ptr = p in tk.ptr_params
        access = p.vtype.access
        writable = access is not tila.types.READ_ONLY
        base_align = _pow2_div(t.data_ptr(), 256) if t.data_ptr() else 256
        esize = t.element_size()
        tma_ok = (dt is not None and dt.name in ("f16", "f32") and len(strides) >= 2 and strides[-1] == 1
                  and base_align >= 16 and all((s * esize) % 16 == 0 and s > 0 for s in strides[:-1])
                  and all(0 < n < (1 << 31) for n in t.shape) and not is_ptr)
        out[p.name] = BufferInfo(
            name=p.name, dtype=dt, rank=len(strides),
            unit_last=bool(strides) and strides[-1] == 1,
            stride_div=tuple(_pow2_div(s, 16) for s in strides),
            base_align=base_align, writable=writable, is_ptr=is_ptr, tma_ok=tma_ok)
    return out


def _cache_for(jf):
    """The kernel cache of ``jf``: the reference's per-function dict
    (``JITFunction._kern_cache``, runtime.py:147), so that its size means
    what it means on the Triton path (one entry per compiled variant)."""
    cache = getattr(jf, "_kern_cache", None)
    if cache is None:
        cache = jf._kern_cache = {}
    return cache


def _debug():
    return os.environ.get("TILA_DEBUG", "") == "1"


def tir_fingerprint(tk) -> str:
    """Hash of the typed TIR as it is now.  The reference keys its cache on
    the generated source (runtime.py:684-696), so a kernel whose TIR was
    edited after decoration compiles again; this key does the same without
    generating code first."""
    import hashlib
    return hashlib.sha256(repr(tk.body).encode()).hexdigest()


def compile_kernel(jf, consts, facts, num_warps, context=None) -> Compiled:
    """The compiled kernel for a specialisation, from ``jf._kern_cache`` or
    built.  The key follows the reference's semantic key
    (``_triton_cache_key``, runtime.py:684-696): intrinsic registry revision,
    function, typed Consts, debug mode, warps, Python source and TIR
    fingerprints, binding facts, constant payloads; and the backend's own
    code-generation switches (TILA_B200_*)."""
    tk = jf.tk
    key = ("b200", tila.intrinsics.INTRINSIC_REGISTRY_SEMANTIC_REVISION, id(jf),
           tuple((k, "Bool" if type(v) is bool else "Int", v) for k, v in sorted(consts.items())),
           _debug(), num_warps, jf.source_fingerprint, tir_fingerprint(tk),
           tuple(f.key() for f in facts.values()), tila.tir.constant_signature(tk.body),
           tuple(sorted((k, v) for k, v in os.environ.items() if k.startswith("TILA_B200_"))))
    cache = _cache_for(jf)
    hit = cache.get(key)
    if hit is not None:
        return hit
    try:
        spec = KernelEmitter(tk, consts, facts, num_warps=num_warps, debug=_debug()).generate()
    except CodegenError as exc:
        raise TilaError("TILA-TARGET-009", f"B200 backend cannot lower this kernel: {exc}",
                        Loc(exc.line),
                        fixes=["restructure the kernel, or run it on CPU arrays (interpreter)"]) from exc
    try:
        try:
            cubin = native.compile_spec(spec)
        except native.NativeError as exc:
            # a kernel whose loop bodies do not fit the register file once
            # specialised for interior tiles is compiled with one body per loop
            if "Register allocation failed" not in (exc.log or ""):
                raise
            spec = KernelEmitter(tk, consts, facts, num_warps=num_warps, debug=_debug(),
                                 versioning=False).generate()
            cubin = native.compile_spec(spec)
        lib = native.Library(cubin)
        kern = lib.kernel(spec.name)
    except native.NativeError as exc:
        raise _failure(exc, "compile" if exc.status == native.TILA_ERR_COMPILE else "load",
                       spec.source, context or {}) from exc
    entry = Compiled(spec, lib, kern)
    cache[key] = entry
    return entry


def _failure(exc, phase, source, context, resource=None):
    """A TILA-TARGET-010/011 error with the reference's replayable artifact
    (backend.failure, backend.py:30-58)."""
    if resource is not None:
        class _Res(Exception):
            pass
        r = _Res(str(exc))
        r.name, r.required, r.limit = resource
        return _tila_backend.failure(r, phase="resources", source=source, source_map={},
                                    context=context, resource=True)
    return _tila_backend.failure(exc, phase=phase, source=source, source_map={}, context=context)


def preflight(entry: Compiled, context) -> dict:
    """Resource check before the first launch on a device (backend.py:61-88)."""
    attrs = entry.kernel.attributes()
    spec = entry.spec
    limit = attrs["max_dynamic_smem_bytes"]
    if spec.smem_bytes > limit:
        raise _failure(RuntimeError("shared memory"), "resources", spec.source, context,
                       resource=("shared memory", spec.smem_bytes, limit))
    if spec.threads > attrs["max_threads_per_block"]:
        raise _failure(RuntimeError("threads"), "resources", spec.source, context,
                       resource=("threads", spec.threads, attrs["max_threads_per_block"]))
    if spec.launch_regs and attrs["registers_per_thread"] != spec.launch_regs:
        # the kernel's warpgroups trade registers (setmaxnreg) within a pool of
        # threads x launch registers; any other count could leave a warpgroup
        # waiting for registers that do not exist, so it is never launched
        raise _failure(RuntimeError("registers"), "resources", spec.source, context,
                       resource=("registers per thread at launch", spec.launch_regs,
                                 attrs["registers_per_thread"]))
    return {"shared_bytes": spec.smem_bytes + attrs["static_smem_bytes"],
            "shared_limit_bytes": limit + attrs["static_smem_bytes"],
            "threads": spec.threads, "max_threads": attrs["max_threads_per_block"],
            "registers_per_thread": attrs["registers_per_thread"],
            "spill_count": attrs["local_bytes_per_thread"],
            "tmem_columns": spec.tmem_cols,
            "performance_only": ["registers_per_thread", "spill_count"]}


_tmap_cache = {}


def _tensor_map(t, info):
    """TMA descriptor of tensor ``t`` for a generated kernel's box (innermost
    dimension first; SWIZZLE_128B; out-of-bounds elements read as zero)."""
    shape, strides = tuple(t.shape), tuple(t.stride())
    key = (t.data_ptr(), shape, strides, tuple(info["box"]), info["swizzle"], info["dtype"])
    tm = _tmap_cache.get(key)
    if tm is None:
        es = t.element_size()
        dims = list(reversed(shape))
        sb = [strides[i] * es for i in reversed(range(len(shape) - 1))]
        tm = native.encode_tensor_map(info["dtype"], t.data_ptr(), dims, sb, info["box"],
                                      info["swizzle"])
        if len(_tmap_cache) > 4096:
            _tmap_cache.clear()
        _tmap_cache[key] = tm
    return tm


def pack_args(entry: Compiled, tk, tensors, scalar_vals, grid, pid_off, err_word, launch_grid, extra=None):
    args = []
    for kind, name, ct in entry.spec.params:
        if kind in ("buffer", "ptr"):
            args.append(ctypes.c_uint64(tensors[name].data_ptr()))
        elif kind == "scalar":
            p = next(s for s in tk.scalars if s.name == name)
            v = scalar_vals[name]
            dn = p.dtype.name
            if dn in ("f16", "bf16"):
                import numpy as np
                if dn == "f16":
                    bits = int(np.asarray(v, dtype=np.float16).view(np.uint16))
                else:
                    import ml_dtypes
                    bits = int(np.asarray(v, dtype=np.float32).astype(ml_dtypes.bfloat16).view(np.uint16))
                args.append(ctypes.c_uint16(bits))
            else:
                args.append(SCALAR_CTYPES[dn](v))
        elif kind == "nprog":
            args.append(ctypes.c_int32(grid[name]))
        elif kind == "pid_off":
            args.append(ctypes.c_int32(pid_off[name]))
        elif kind == "launch":
            args.append(ctypes.c_int32(launch_grid[name]))
        elif kind == "err":
            args.append(ctypes.c_uint64(err_word.data_ptr()))
        elif kind in ("skws", "skflags"):
            args.append(ctypes.c_uint64(extra[kind].data_ptr()))
        elif kind == "tensormap":
            args.append(_tensor_map(tensors[ct["buffer"]], ct))
        else:
            raise AssertionError(kind)
    return args


def execute(launcher, tensors, scalar_vals, stride_vals, consts, grid, entry=None):
    """Compile (cached) and launch a checked kernel on the tensors' device.
    ``entry``: the compiled kernel of an earlier launch whose binding
    signature, Consts, options and TIR are those of this one (plugin.py's
    repeated-signature path), used without recomputing the cache key."""
    import torch
    jf, tk = launcher.jf, launcher.jf.tk
    # what the launch needs besides the tensors; a repeated launch with the
    # same binding signature replays it (plugin.py, repeated-signature path)
    launcher._b200_last_exec = (dict(tensors), scalar_vals, stride_vals, consts, grid)
    device = next(iter(tensors.values())).device

    def context():
        target = getattr(launcher, "target", None)
        return {"kernel": tk.name, "tila_source": jf.tila_source,
                "source_file": jf.fn.__code__.co_filename,
                "source_start_line": jf.source_start_line, "consts": consts,
                "scalars": scalar_vals, "grid": grid, "num_warps": launcher.num_warps,
                "debug": _debug(), "backend": "b200",
                "target": asdict(target) if target is not None else None}
    check_device_errors(device)
    with torch.cuda.device(device):
        if entry is None or entry.attrs is None or entry.attrs.get("_device") != device.index:
            ctx = context()
            entry = compile_kernel(jf, consts, binding_facts(tk, tensors), launcher.num_warps, ctx)
            if entry.attrs is None or entry.attrs.get("_device") != device.index:
                entry.attrs = preflight(entry, ctx)
                entry.attrs["_device"] = device.index
        jf.last_backend_resources = {k: v for k, v in entry.attrs.items() if k != "_device"}
        g = tuple(grid) + (1,) * (3 - len(grid))
        launch_grid, pid_off = list(g), [0, 0, 0]
        shard = current_program_range()
        if shard is not None:
            ax, lo, hi = shard
            lo, hi = max(0, lo), min(g[ax], hi)
            if hi <= lo:
                return
            launch_grid[ax] = hi - lo
            pid_off[ax] = lo
        err = _error_word(device)
        stream = torch.cuda.current_stream(device).cuda_stream
        cuda_grid = list(launch_grid)
        for ax, f in entry.spec.fuse.items():        # CTAs that run blocks of programs
            cuda_grid[ax] = -(-cuda_grid[ax] // f)
        extra = None
        if entry.spec.persistent:
            cuda_grid, extra = _streamk_geometry(cuda_grid, device, stream)
        args = pack_args(entry, tk, tensors, scalar_vals, g, pid_off, err, launch_grid, extra)
        record = LaunchRecord(entry, tuple(cuda_grid), args, device,
                              dict(tensors, **(extra or {})))
        jf._b200_last_launch = record
        try:
            record.launch(stream)
        except native.NativeError as exc:
            if exc.status == native.TILA_ERR_RESOURCES:
                raise _failure(exc, "resources", entry.spec.source, context(),
                               resource=("launch", entry.spec.smem_bytes, exc.log)) from exc
            raise _failure(exc, "launch", entry.spec.source, context()) from exc
        if entry.spec.assume_lines:
            # debug build: a false ti.assume stopped its program and left its
            # line in the error word (the interpreter asserts there too)
            word = read_device_errors(device, reset=False)
            if word >> 24 == 3:
                read_device_errors(device)
                raise AssertionError(f"device_assert failed: ti.assume at line {word & 0xFFFFFF} "
                                     f"of {tk.name} (TILA_DEBUG=1)")


# Stream-K contraction kernels (codegen/fused.py): the persistent CTAs' workspace
# slots (one per CTA: 4 programs x 128 x 128 f32 partial accumulators) and the
# flags that hand a tile's parked high-K part to the CTA that finishes it.  One
# set per device and stream, so that launches on different streams never share
# them; launches on one stream are ordered.  Every flag a launch sets is
# cleared by the same launch.
_SK_SLOT_BYTES = 4 * 128 * 128 * 4
_SK_MAX_BYTES = 256 << 20
_sk_buffers = {}


def _streamk_geometry(cuda_grid, device, stream):
    """Grid of a stream-K launch: as many CTAs as SMs when there are more
    tiles than SMs (the K loops are then split evenly over them), one CTA per
    tile otherwise; axis 2 stays on z.  Returns (grid, workspace args)."""
    import torch
    tiles = cuda_grid[0] * cuda_grid[1]
    sms = _sm_count(device)
    split = tiles > sms and cuda_grid[2] == 1 and cuda_grid[2] * sms * _SK_SLOT_BYTES <= _SK_MAX_BYTES
    nct = sms if split else tiles
    key = (device.index, int(stream))
    bufs = _sk_buffers.get(key)
    slots = cuda_grid[2] * nct if split else 1
    if bufs is None or bufs["skflags"].numel() < slots:
        bufs = {"skws": torch.empty(slots * _SK_SLOT_BYTES // 4, dtype=torch.float32, device=device),
                "skflags": torch.zeros(slots, dtype=torch.int32, device=device)}
        _sk_buffers[key] = bufs
    return [nct, 1, cuda_grid[2]], bufs


_sm_counts = {}


def _sm_count(device):
    import torch
    n = _sm_counts.get(device.index)
    if n is None:
        n = _sm_counts[device.index] = torch.cuda.get_device_properties(device).multi_processor_count
    return n


def _reset_streamk_flags(device):
    """After a device error a launch may have stopped between parking a tile
    and clearing its flag: clear every flag of the device."""
    for (dev, _), bufs in _sk_buffers.items():
        if dev == device.index:
            bufs["skflags"].zero_()


def launch_flags() -> int:
    """Launch flags of generated kernels.  Every generated kernel waits for
    the previous grid in its stream before touching global memory, so it is
    launched to overlap that grid's tail (TILA_B200_OVERLAP=0 turns it off)."""
    if os.environ.get("TILA_B200_OVERLAP", "1") == "0":
        return 0
    return native.LAUNCH_OVERLAP_PREVIOUS


class LaunchRecord:
    """One prepared launch (kernel, geometry, packed arguments).  Re-issuing it
    skips Tila's host-side contract checks, so benchmarks can time the kernel
    alone; the tensors it points at must stay alive and unchanged in shape."""

    def __init__(self, entry, grid, args, device, tensors=None):
        self.entry, self.grid, self.args, self.device = entry, grid, args, device
        # the packed arguments are raw device addresses: hold the tensors so
        # that a replay never touches memory returned to the allocator
        self.tensors = dict(tensors or {})

    def launch(self, stream=None):
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(self.device).cuda_stream
        self.entry.kernel.launch(self.grid, (self.entry.spec.threads, 1, 1), self.args,
                                 smem_bytes=self.entry.spec.smem_bytes, stream=stream,
                                 flags=launch_flags())

    @property
    def kernel_name(self):
        return self.entry.spec.name


def last_launch(jf) -> LaunchRecord:
    """The most recent B200 launch of ``jf`` (see :class:`LaunchRecord`)."""
    rec = getattr(jf, "_b200_last_launch", None)
    if rec is None:
        raise RuntimeError(f"{jf.__name__} has not been launched on the B200 backend")
    return rec


def generated_source(jf, consts, tensors, num_warps=4) -> str:
    """CUDA C++ the backend generates for a binding (inspection / CLI)."""
    facts = binding_facts(jf.tk, tensors)
    return KernelEmitter(jf.tk, consts, facts, num_warps=num_warps).generate().source
