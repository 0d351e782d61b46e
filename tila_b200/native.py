"""ctypes binding of ``libtila_b200.so`` (C ABI in ``include/tila_b200.h``).

This module is the only place that calls into the native launcher.  It
provides: NVRTC compilation of generated CUDA C++ into sm_100a cubins (with an
on-disk cubin cache), library loading, kernel lookup, resource queries,
launching, and TMA tensor-map encoding.

The library must exist: the B200 backend has no fallback path, so a missing
or unloadable library raises instead of silently running something else.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import threading
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "libtila_b200.so"
TILE_INCLUDE_DIR = PACKAGE_DIR / "csrc" / "tile"
CACHE_DIR = Path(os.environ.get("TILA_B200_CACHE", PACKAGE_DIR / "_cubin_cache"))

TILA_OK = 0
TILA_ERR_DRIVER_MISSING = -1
TILA_ERR_DRIVER = -2
TILA_ERR_COMPILE = -3
TILA_ERR_LOAD = -4
TILA_ERR_RESOURCES = -5
TILA_ERR_ARGUMENT = -6
TILA_ERR_NO_CONTEXT = -7

#: Symbols that include/tila_b200.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "tila_nvrtc_compile", "tila_nvrtc_version", "tila_free_buffer", "tila_init",
    "tila_library_load", "tila_library_unload", "tila_kernel_get",
    "tila_kernel_attrs_get", "tila_launch", "tila_encode_tensor_map",
    "tila_device_info", "tila_status_string", "tila_launch_noalloc",
    "tila_mg_unique_id", "tila_mg_comm_init", "tila_mg_gather", "tila_mg_comm_destroy",
    "tila_host_word_alloc", "tila_host_word_free", "tila_noalloc_read_error",
)

#: Size of the error block every generated kernel takes (include/tila_b200.h).
ERROR_BLOCK_BYTES = 16

#: Capacity of the static scratch behind tila_launch_noalloc (include/tila_b200.h).
NOALLOC_SCRATCH_BYTES = 256


class NativeError(RuntimeError):
    """A failing call of the native launcher: ``status`` is the C status code."""

    def __init__(self, status: int, message: str, log: str = ""):
        super().__init__(message + (f"\n{log}" if log else ""))
        self.status = status
        self.log = log


class LaunchConfig(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_uint32 * 3), ("block", ctypes.c_uint32 * 3),
                ("cluster", ctypes.c_uint32 * 3), ("smem_bytes", ctypes.c_uint32),
                ("stream", ctypes.c_uint64), ("flags", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


# tila_launch_config.flags
LAUNCH_OVERLAP_PREVIOUS = 1


class KernelAttrs(ctypes.Structure):
    _fields_ = [("registers_per_thread", ctypes.c_int32),
                ("static_smem_bytes", ctypes.c_int32),
                ("local_bytes_per_thread", ctypes.c_int32),
                ("max_threads_per_block", ctypes.c_int32),
                ("max_dynamic_smem_bytes", ctypes.c_int32),
                ("binary_version", ctypes.c_int32)]


class TensorMap(ctypes.Structure):
    """128-byte CUtensorMap storage (64-byte alignment is enforced at encode)."""
    _fields_ = [("opaque", ctypes.c_uint64 * 16)]


_lib = None
_lib_lock = threading.Lock()


def library() -> ctypes.CDLL:
    """Load ``libtila_b200.so`` (raises if it is missing: no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not LIBRARY_PATH.exists():
            raise NativeError(TILA_ERR_LOAD, f"{LIBRARY_PATH.name} is not built; "
                              "run __graft_entry__.build() or `python -m tila_b200.build`")
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        c_char_p, c_size_t, c_int, c_void_p = (ctypes.c_char_p, ctypes.c_size_t,
                                               ctypes.c_int, ctypes.c_void_p)
        lib.tila_nvrtc_compile.argtypes = [c_char_p, c_char_p, ctypes.POINTER(c_char_p), c_int,
                                           ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t),
                                           c_char_p, c_size_t]
        lib.tila_nvrtc_version.argtypes = [ctypes.POINTER(c_int)]
        lib.tila_free_buffer.argtypes = [c_void_p]
        lib.tila_free_buffer.restype = None
        lib.tila_init.argtypes = [c_char_p, c_size_t]
        lib.tila_library_load.argtypes = [c_void_p, c_size_t, ctypes.POINTER(c_void_p),
                                          c_char_p, c_size_t]
        lib.tila_library_unload.argtypes = [c_void_p]
        lib.tila_kernel_get.argtypes = [c_void_p, c_char_p, ctypes.POINTER(c_void_p),
                                        c_char_p, c_size_t]
        lib.tila_kernel_attrs_get.argtypes = [c_void_p, ctypes.POINTER(KernelAttrs),
                                              c_char_p, c_size_t]
        lib.tila_launch.argtypes = [c_void_p, ctypes.POINTER(LaunchConfig),
                                    ctypes.POINTER(c_void_p), c_char_p, c_size_t]
        lib.tila_encode_tensor_map.argtypes = [c_void_p, c_int, c_int, ctypes.c_uint64,
                                               ctypes.POINTER(ctypes.c_uint64),
                                               ctypes.POINTER(ctypes.c_uint64),
                                               ctypes.POINTER(ctypes.c_uint32), c_int,
                                               c_char_p, c_size_t]
        lib.tila_device_info.argtypes = [ctypes.POINTER(c_int)] * 4 + [c_char_p, c_size_t]
        lib.tila_launch_noalloc.argtypes = [c_void_p, ctypes.POINTER(LaunchConfig),
                                            ctypes.POINTER(c_void_p), c_int, ctypes.c_uint32,
                                            c_char_p, c_size_t]
        lib.tila_host_word_alloc.argtypes = [ctypes.POINTER(c_void_p), ctypes.POINTER(ctypes.c_uint64),
                                             c_char_p, c_size_t]
        lib.tila_host_word_free.argtypes = [c_void_p]
        lib.tila_noalloc_read_error.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint64,
                                                c_int, c_char_p, c_size_t]
        lib.tila_status_string.argtypes = [c_int]
        lib.tila_status_string.restype = c_char_p
        lib.tila_mg_unique_id.argtypes = [c_void_p, c_char_p, c_size_t]
        lib.tila_mg_comm_init.argtypes = [c_void_p, c_int, c_int, ctypes.POINTER(c_void_p),
                                          c_char_p, c_size_t]
        lib.tila_mg_gather.argtypes = [c_void_p, c_void_p, c_void_p, c_size_t, ctypes.c_uint64,
                                       c_char_p, c_size_t]
        lib.tila_mg_comm_destroy.argtypes = [c_void_p]
        _lib = lib
        return lib


def _check(status: int, what: str, log=None):
    if status != TILA_OK:
        text = log.value.decode(errors="replace") if log is not None else ""
        msg = library().tila_status_string(status).decode()
        raise NativeError(status, f"{what}: {msg}", text)


def nvrtc_version() -> int:
    v = ctypes.c_int()
    _check(library().tila_nvrtc_version(ctypes.byref(v)), "nvrtcVersion")
    return v.value


def default_options(extra=(), fp_contract=False) -> list[str]:
    """NVRTC options of every generated kernel.

    ``--fmad=false`` keeps each f32 add and multiply separately rounded, which
    is what NumPy (the interpreter's arithmetic) does; divisions and square
    roots stay IEEE (no fast-math).  ``fp_contract`` (tensor-core kernels,
    compared within a tolerance) lets a*b+c contract into one FMA.
    """
    fmad = "--fmad=true" if fp_contract else "--fmad=false"
    return ["-arch=sm_100a", "--std=c++17", fmad, "-default-device",
            "-lineinfo", f"-I{TILE_INCLUDE_DIR}", "-DNDEBUG", *extra]


def compile_spec(spec) -> bytes:
    """Compile a generated kernel (``codegen.emitter.KernelSpec``)."""
    return compile_cubin(spec.source, spec.name,
                         default_options(fp_contract=getattr(spec, "fp_contract", False)))


def _tile_headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(TILE_INCLUDE_DIR.glob("*.cuh")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


_compile_lock = threading.Lock()


def compile_cubin(source: str, name: str, options=None) -> bytes:
    """Compile generated CUDA C++ to an sm_100a cubin, through the disk cache.

    The cache key covers the source, the options, the NVRTC version and the
    tile-library headers.  Raises :class:`NativeError` (status
    ``TILA_ERR_COMPILE``) with the NVRTC log on failure.
    """
    opts = default_options() if options is None else list(options)
    key = hashlib.sha256("\0".join([source, *opts, str(nvrtc_version()),
                                    _tile_headers_digest()]).encode()).hexdigest()
    path = CACHE_DIR / f"{key}.cubin"
    if path.exists():
        return path.read_bytes()
    lib = library()
    arr = (ctypes.c_char_p * len(opts))(*[o.encode() for o in opts])
    out = ctypes.c_void_p()
    size = ctypes.c_size_t()
    log = ctypes.create_string_buffer(1 << 16)
    with _compile_lock:
        status = lib.tila_nvrtc_compile(source.encode(), f"{name}.cu".encode(), arr, len(opts),
                                        ctypes.byref(out), ctypes.byref(size), log, len(log))
    _check(status, f"NVRTC compile of {name}", log)
    try:
        data = ctypes.string_at(out.value, size.value)
    finally:
        lib.tila_free_buffer(out)
    try:
        CACHE_DIR.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        tmp.write_bytes(data)
        os.replace(tmp, path)
    except OSError:
        pass
    return data


def init() -> None:
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_init(log, len(log)), "CUDA driver initialisation", log)


class Library:
    """A loaded cubin (CUlibrary); kernels are looked up by name."""

    def __init__(self, cubin: bytes):
        init()
        self._cubin = ctypes.create_string_buffer(cubin, len(cubin))
        handle = ctypes.c_void_p()
        log = ctypes.create_string_buffer(4096)
        _check(library().tila_library_load(self._cubin, len(cubin), ctypes.byref(handle),
                                           log, len(log)), "cubin load", log)
        self.handle = handle
        self._kernels = {}

    def kernel(self, name: str) -> "Kernel":
        k = self._kernels.get(name)
        if k is None:
            handle = ctypes.c_void_p()
            log = ctypes.create_string_buffer(1024)
            _check(library().tila_kernel_get(self.handle, name.encode(), ctypes.byref(handle),
                                             log, len(log)), f"kernel lookup {name}", log)
            k = self._kernels[name] = Kernel(self, handle, name)
        return k


class Kernel:
    def __init__(self, lib: Library, handle: ctypes.c_void_p, name: str):
        self.library = lib
        self.handle = handle
        self.name = name

    def attributes(self) -> dict:
        a = KernelAttrs()
        log = ctypes.create_string_buffer(1024)
        _check(library().tila_kernel_attrs_get(self.handle, ctypes.byref(a), log, len(log)),
               f"attributes of {self.name}", log)
        return {f: getattr(a, f) for f, _ in KernelAttrs._fields_}

    def launch(self, grid, block, args, smem_bytes=0, stream=0, cluster=(1, 1, 1), flags=0):
        """Launch with ``args``: a sequence of ctypes objects, one per parameter.
        ``flags``: LAUNCH_* bits (LAUNCH_OVERLAP_PREVIOUS only for kernels that
        wait on the previous grid before touching global memory)."""
        cfg = LaunchConfig()
        for i in range(3):
            cfg.grid[i] = grid[i]
            cfg.block[i] = block[i]
            cfg.cluster[i] = cluster[i]
        cfg.smem_bytes = smem_bytes
        cfg.stream = stream
        cfg.flags = flags
        ptrs = (ctypes.c_void_p * max(1, len(args)))(
            *[ctypes.addressof(a) for a in args])
        log = ctypes.create_string_buffer(1024)
        _check(library().tila_launch(self.handle, ctypes.byref(cfg), ptrs, log, len(log)),
               f"launch of {self.name}", log)

    def launch_noalloc(self, grid, block, args, scratch_arg, scratch_bytes, smem_bytes=0,
                       stream=0, flags=0):
        """Launch through tila_launch_noalloc: argument ``scratch_arg`` (the
        kernel's scratch pointer) is replaced by the library's static device
        scratch, so this call allocates no device memory.  Returns the C status."""
        cfg = LaunchConfig()
        for i in range(3):
            cfg.grid[i] = grid[i]
            cfg.block[i] = block[i]
            cfg.cluster[i] = 1
        cfg.smem_bytes = smem_bytes
        cfg.stream = stream
        cfg.flags = flags
        ptrs = (ctypes.c_void_p * max(1, len(args)))(
            *[ctypes.addressof(a) for a in args])
        log = ctypes.create_string_buffer(1024)
        status = library().tila_launch_noalloc(self.handle, ctypes.byref(cfg), ptrs, scratch_arg,
                                               scratch_bytes, log, len(log))
        self.last_log = log.value.decode(errors="replace")
        return status


# CUtensorMapDataType / CUtensorMapSwizzle numbering (cuda.h).
TMA_DTYPE = {"u8": 0, "u16": 1, "u32": 2, "i32": 3, "u64": 4, "i64": 5, "f16": 6,
             "f32": 7, "f64": 8, "bf16": 9}
TMA_SWIZZLE = {0: 0, 32: 1, 64: 2, 128: 3}


def encode_tensor_map(dtype: str, address: int, dims, strides_bytes, box, swizzle_bytes=128):
    """Encode a tiled TMA descriptor; dims/box innermost first, strides for dims 1.."""
    tm = _aligned_tensor_map()
    rank = len(dims)
    d = (ctypes.c_uint64 * rank)(*dims)
    s = (ctypes.c_uint64 * max(1, rank - 1))(*strides_bytes) if rank > 1 else None
    b = (ctypes.c_uint32 * rank)(*box)
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_encode_tensor_map(ctypes.addressof(tm), TMA_DTYPE[dtype], rank, address,
                                            d, s, b, TMA_SWIZZLE[swizzle_bytes], log, len(log)),
           "tensor map encode", log)
    return tm


def _aligned_tensor_map() -> TensorMap:
    raw = ctypes.create_string_buffer(128 + 64)
    offset = (-ctypes.addressof(raw)) % 64
    tm = TensorMap.from_buffer(raw, offset)
    tm._keepalive = raw
    return tm


def noalloc_read_error(stream=0, reset=True) -> int:
    """The error word the last tila_launch_noalloc launch on the current
    device recorded in the library's static scratch (synchronises ``stream``)."""
    word = ctypes.c_uint32()
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_noalloc_read_error(ctypes.byref(word), stream, int(bool(reset)), log,
                                             len(log)), "read of the no-allocation error word", log)
    return word.value


def host_word_alloc():
    """(host address, device address) of a zeroed page-locked 64-byte buffer
    that kernels can write (needs a current CUDA context)."""
    host, dev = ctypes.c_void_p(), ctypes.c_uint64()
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_host_word_alloc(ctypes.byref(host), ctypes.byref(dev), log, len(log)),
           "page-locked host word", log)
    return host.value, dev.value


def host_word_free(host: int) -> None:
    _check(library().tila_host_word_free(ctypes.c_void_p(host)), "free of a page-locked host word")


def device_info() -> dict:
    vals = [ctypes.c_int() for _ in range(4)]
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_device_info(*[ctypes.byref(v) for v in vals], log, len(log)),
           "device info", log)
    return dict(zip(("sm_count", "max_smem_optin", "cc_major", "cc_minor"),
                    (v.value for v in vals)))


# -- multi-GPU gather (tila_mg_*): NCCL behind the C ABI ----------------------

MG_UNIQUE_ID_BYTES = 128


def mg_unique_id() -> bytes:
    """A fresh communicator id (created by rank 0, shared with the others)."""
    buf = ctypes.create_string_buffer(MG_UNIQUE_ID_BYTES)
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_mg_unique_id(buf, log, len(log)), "communicator id", log)
    return buf.raw


def mg_comm_init(uid: bytes, nranks: int, rank: int) -> int:
    """Join communicator ``uid`` on the current device; returns the handle."""
    if len(uid) != MG_UNIQUE_ID_BYTES:
        raise ValueError("communicator id must have 128 bytes")
    buf = ctypes.create_string_buffer(uid, MG_UNIQUE_ID_BYTES)
    handle = ctypes.c_void_p()
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_mg_comm_init(buf, nranks, rank, ctypes.byref(handle), log, len(log)),
           "communicator init", log)
    return handle.value


def mg_gather(comm: int, send_ptr: int, recv_ptr: int, bytes_per_rank: int, stream: int) -> None:
    """recv[r * bytes_per_rank:(r + 1) * bytes_per_rank] = rank r's send, for every rank."""
    log = ctypes.create_string_buffer(1024)
    _check(library().tila_mg_gather(ctypes.c_void_p(comm), ctypes.c_void_p(send_ptr), ctypes.c_void_p(recv_ptr),
                                    bytes_per_rank, stream, log, len(log)), "gather", log)


def mg_comm_destroy(comm: int) -> None:
    _check(library().tila_mg_comm_destroy(ctypes.c_void_p(comm)), "communicator destroy")
