"""The C-ABI library: it loads without a GPU, exports every symbol the
header declares, and its NVRTC half compiles generated CUDA for sm_100a."""

import ctypes
import re
from pathlib import Path

import pytest

from tila_b200 import native

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "tila_b200.h").read_text()
    return sorted(set(re.findall(r"\b(tila_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = native.library()
    declared = header_symbols()
    assert declared, "no functions found in include/tila_b200.h"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert set(declared) == set(native.EXPORTED_SYMBOLS)


def test_status_strings():
    lib = native.library()
    assert lib.tila_status_string(0) == b"ok"
    assert b"NVRTC" in lib.tila_status_string(native.TILA_ERR_COMPILE)


def test_nvrtc_compiles_sm100a_cubin():
    src = '#include "tila_tile.cuh"\nextern "C" __global__ void k(float* x) { x[threadIdx.x] = tila::round_f16(x[0]); }\n'
    cubin = native.compile_cubin(src, "probe")
    assert cubin[:4] == b"\x7fELF"


def test_nvrtc_error_is_reported_with_log():
    with pytest.raises(native.NativeError) as exc:
        native.compile_cubin('extern "C" __global__ void k() { this is not C++; }\n', "bad")
    assert exc.value.status == native.TILA_ERR_COMPILE
    assert "error" in exc.value.log.lower()


def test_driver_entry_points_fail_cleanly_without_gpu():
    lib = native.library()
    buf = ctypes.create_string_buffer(256)
    status = lib.tila_init(buf, len(buf))
    if status == native.TILA_OK:
        pytest.skip("a CUDA driver is present on this machine")
    assert status in (native.TILA_ERR_DRIVER_MISSING, native.TILA_ERR_DRIVER)
    assert buf.value


def test_argument_validation():
    lib = native.library()
    assert lib.tila_launch(None, None, None, None, 0) == native.TILA_ERR_ARGUMENT
    assert lib.tila_library_load(None, 0, None, None, 0) == native.TILA_ERR_ARGUMENT


def test_gather_entry_points_validate_arguments():
    """The multi-GPU gather rejects bad arguments before touching NCCL."""
    lib = native.library()
    log = ctypes.create_string_buffer(256)
    handle = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(native.MG_UNIQUE_ID_BYTES)
    assert lib.tila_mg_comm_init(uid, 2, 5, ctypes.byref(handle), log, len(log)) == -6
    assert lib.tila_mg_comm_init(uid, 0, 0, ctypes.byref(handle), log, len(log)) == -6
    assert lib.tila_mg_gather(None, None, None, 16, 0, log, len(log)) == -6
    assert lib.tila_mg_comm_destroy(None) == -6
    with pytest.raises(ValueError):
        native.mg_comm_init(b"short", 1, 0)
