"""C++ spellings and literal encodings of Tila dtypes in generated kernels.

Register representation: f16 and bf16 tile elements live in f32 registers
holding a value that is exactly representable in the narrow type; every
arithmetic result is rounded back (``tila::round_f16``), which reproduces
NumPy's float16 / ml_dtypes bfloat16 arithmetic (computed in float32, then
rounded; interp.py:218-235).  Memory keeps the narrow 16-bit encoding.
"""

from __future__ import annotations

import struct

import numpy as np

from .._reference import tila

D = tila.dtypes

CTYPE = {
    "bool": "bool", "i8": "tila::i8", "i16": "tila::i16", "i32": "tila::i32",
    "i64": "tila::i64", "u8": "tila::u8", "u16": "tila::u16", "u32": "tila::u32",
    "u64": "tila::u64", "f16": "float", "bf16": "float", "f32": "float", "f64": "double",
}
MEMTYPE = dict(CTYPE, f16="tila::u16", bf16="tila::u16", bool="tila::u8")
SIZE = {"bool": 1, "i8": 1, "i16": 2, "i32": 4, "i64": 8, "u8": 1, "u16": 2, "u32": 4,
        "u64": 8, "f16": 2, "bf16": 2, "f32": 4, "f64": 8}


def name(dt) -> str:
    return dt.name


def ctype(dt) -> str:
    return CTYPE[dt.name]


def memtype(dt) -> str:
    return MEMTYPE[dt.name]


def size(dt) -> int:
    return SIZE[dt.name]


def is_float(dt) -> bool:
    return dt.name in ("f16", "bf16", "f32", "f64")


def is_int(dt) -> bool:
    return dt.name in ("i8", "i16", "i32", "i64", "u8", "u16", "u32", "u64")


def is_signed(dt) -> bool:
    return dt.name in ("i8", "i16", "i32", "i64")


def int_min(dt) -> int:
    return -(1 << (int(dt.name[1:]) - 1)) if is_signed(dt) else 0


def load_conv(dt, expr: str) -> str:
    """Memory encoding -> register value."""
    if dt.name == "f16":
        return f"tila::h2f({expr})"
    if dt.name == "bf16":
        return f"tila::bf2f({expr})"
    if dt.name == "bool":
        return f"(({expr}) != 0)"
    return expr


def store_conv(dt, expr: str) -> str:
    """Register value -> memory encoding (exact: the value is representable)."""
    if dt.name == "f16":
        return f"tila::f2h({expr})"
    if dt.name == "bf16":
        return f"tila::f2bf({expr})"
    if dt.name == "bool":
        return f"((tila::u8)(({expr}) ? 1 : 0))"
    return expr


def round_to(dt, expr: str) -> str:
    """Round an f32 (or f64) computation to the register value of dt."""
    if dt.name == "f16":
        return f"tila::round_f16({expr})"
    if dt.name == "bf16":
        return f"tila::round_bf16({expr})"
    return expr


def float_literal(dt, value) -> str:
    """Exact C++ spelling of a float literal rounded the way NumPy rounds it."""
    n = dt.name
    if n == "f64":
        bits = struct.unpack("<Q", struct.pack("<d", float(value)))[0]
        return f"__longlong_as_double(0x{bits:016x}LL)"
    if n == "f32":
        v = np.float32(value)
    elif n == "f16":
        v = np.float32(np.float16(value))
    elif n == "bf16":
        v = np.float32(_bf16(value))
    else:
        raise ValueError(n)
    bits = int(np.asarray(v, dtype=np.float32).view(np.uint32))
    return f"__uint_as_float(0x{bits:08x}u)"


def _bf16(value):
    import ml_dtypes
    return np.asarray(value, dtype=np.float64).astype(np.float32).astype(ml_dtypes.bfloat16)


def int_literal(dt, value: int) -> str:
    bits = int(dt.name[1:])
    v = int(value) % (1 << bits)
    if is_signed(dt) and v >= 1 << (bits - 1):
        v -= 1 << bits
    if dt.name in ("i64",):
        return f"((tila::i64){v}LL)" if v != -(1 << 63) else "((tila::i64)(-9223372036854775807LL - 1))"
    if dt.name == "u64":
        return f"((tila::u64){v}ULL)"
    if dt.name == "i32" and v == -(1 << 31):
        return "((tila::i32)(-2147483647 - 1))"
    return f"(({CTYPE[dt.name]}){v})"


def literal(dt, value) -> str:
    if dt.name == "bool":
        return "true" if value else "false"
    if is_float(dt):
        return float_literal(dt, value)
    return int_literal(dt, int(value))


def constant_bits(dt, bits: int) -> str:
    """TConstant payload (exact bit pattern) as a register value."""
    n = dt.name
    if n == "f64":
        return f"__longlong_as_double(0x{bits:016x}LL)"
    if n == "f32":
        return f"__uint_as_float(0x{bits:08x}u)"
    if n == "f16":
        return f"tila::h2f((tila::u16)0x{bits:04x})"
    if n == "bf16":
        return f"tila::bf2f((tila::u16)0x{bits:04x})"
    raise ValueError(n)


def convert(src, dst, expr: str) -> str:
    """Value conversion with NumPy astype semantics (interp.py:236-251)."""
    s, d = src.name, dst.name
    if s == d:
        return expr
    if d == "bool":
        return f"(({expr}) != 0)"
    if is_float(dst):
        if s == "bool":
            return round_to(dst, f"(({CTYPE[d]})(({expr}) ? 1 : 0))")
        if d == "f64":
            return f"((double)({expr}))"
        if d in ("f16", "bf16"):
            if s == "f64":
                return f"tila::h2f(tila::d2h({expr}))" if d == "f16" else f"tila::bf2f(tila::d2bf({expr}))"
            if is_int(src):
                # integer -> narrow float with a single rounding
                return (f"tila::h2f(tila::d2h((double)({expr})))" if d == "f16"
                        else f"tila::bf2f(tila::d2bf((double)({expr})))")
            return round_to(dst, f"((float)({expr}))")
        # f32
        if s == "f64" or is_int(src):
            return f"((float)({expr}))"
        return f"((float)({expr}))"
    # integer destination
    if is_float(src):
        return f"(({CTYPE[d]})(({CTYPE[d]})({'trunc' if s == 'f64' else 'truncf'}({expr}))))"
    if s == "bool":
        return f"(({CTYPE[d]})(({expr}) ? 1 : 0))"
    return f"(({CTYPE[d]})({expr}))"
