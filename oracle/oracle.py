"""numpy front end of the CPU oracle (test infrastructure only).

Wraps oracle/liboracle_bnbq.so (the C restatement in bnbq_oracle.c) and
restates ``create_dynamic_map`` (reference kernels/quantize.py:53-88) in
numpy. Only the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline use this module; the product never imports it.

bfloat16 arrays are carried as uint16 bit patterns (numpy has no bf16).
Element-type codes: F32 = 0, F16 = 1, BF16 = 2 (as include/bnbq.h).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

F32, F16, BF16 = 0, 1, 2
HERE = Path(__file__).resolve().parent

NF4_TABLE = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], np.float32)
NF4_THRESHOLDS = np.array([
    0xbf591cd9, 0xbf1c5270, 0xbeeb8480, 0xbeadea76, 0xbe703cec,
    0xbe0d38bc, 0xbd3a7871, 0x3d22faff, 0x3df64863, 0x3e5067e0,
    0x3e9582d4, 0x3ec753f9, 0x3f006d03, 0x3f248daf, 0x3f5c89d9], np.uint32).view(np.float32)

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = HERE / "liboracle_bnbq.so"
        if not path.exists():
            from . import build as _b  # type: ignore
            _b.build()
        _lib = C.CDLL(str(path))
        _declare(_lib)
    return _lib


def _declare(L: C.CDLL) -> None:
    p, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float
    sig = {
        "or_num_threads": ([], i32), "or_set_threads": ([i32], None),
        "or_code_nf4": ([f32], C.c_uint8), "or_code_8bit": ([p, f32], C.c_uint8),
        "or_q8_thresholds": ([p, p], i32),
        "or_absmax": ([i32, p, i64, i32, p], None),
        "or_rcp_ieee_ftz": ([p, p, i64], None),
        "or_quantize_nf4": ([i32, p, i64, i32, p, p, p, p], None),
        "or_quantize_8bit": ([i32, p, i64, i32, p, p, p, p, p, p], None),
        "or_dequantize": ([i32, i32, p, p, p, i64, i32, p, p], None),
        "or_nested_absmax": ([p, p, p, f32, i64, i32, i64, p], None),
        "or_mean": ([p, i64, p], None),
        "or_gemv_f64": ([i32, p, i32, i32, p, i64, i32, p, p, p], None),
        "or_gemv_ref": ([i32, p, i32, i32, p, i64, i32, p, p], None),
        "or_nf4_bucket_tables": ([p, p], i32), "or_check_nf4_buckets": ([i64], i64),
        "or_q8_fine_tables": ([p, p, p, p], i32), "or_check_q8_buckets": ([p, i64, p], i64),
        "or_codes_nf4": ([p, i64, p], None), "or_codes_8bit": ([p, p, i64, p], None),
        "or_codes_8bit_count": ([p, p, i64, p], None), "or_mul_ftz": ([p, p, i64, p], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def num_threads() -> int:
    return int(lib().or_num_threads())


# ----------------------------------------------------------- conversions

def f32_to_bf16(x) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bits (canonical NaN 0x7fff)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_to_f32(b) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def elem_dtype(code: int):
    return {F32: np.float32, F16: np.float16, BF16: np.uint16}[code]


def to_f32(x, code: int) -> np.ndarray:
    return bf16_to_f32(x) if code == BF16 else np.asarray(x).astype(np.float32)


# ------------------------------------------------------------ code choice

def codes_nf4(s) -> np.ndarray:
    s = _c(s, np.float32)
    out = np.empty(s.size, np.uint8)
    lib().or_codes_nf4(_p(s), s.size, _p(out))
    return out


def codes_8bit(code, s) -> np.ndarray:
    code, s = _c(code, np.float32), _c(s, np.float32)
    out = np.empty(s.size, np.uint8)
    lib().or_codes_8bit(_p(code), _p(s), s.size, _p(out))
    return out


def q8_thresholds(code):
    code = _c(code, np.float32)
    T = np.empty(255, np.float32)
    ok = lib().or_q8_thresholds(_p(code), _p(T))
    return T if ok else None


def codes_8bit_count(T, s) -> np.ndarray:
    T, s = _c(T, np.float32), _c(s, np.float32)
    out = np.empty(s.size, np.uint8)
    lib().or_codes_8bit_count(_p(T), _p(s), s.size, _p(out))
    return out


def mul_ftz(a, b) -> np.ndarray:
    a, b = np.broadcast_arrays(_c(a, np.float32), _c(b, np.float32))
    a, b = _c(a, np.float32), _c(b, np.float32)
    out = np.empty(a.size, np.float32)
    lib().or_mul_ftz(_p(a), _p(b), a.size, _p(out))
    return out


# ---------------------------------------------------------------- kernels

def absmax(x, dtype: int, blocksize: int) -> np.ndarray:
    x = _c(x, elem_dtype(dtype))
    out = np.empty(-(-x.size // blocksize), np.float32)
    lib().or_absmax(dtype, _p(x), x.size, blocksize, _p(out))
    return out


def quantize_nf4(x, dtype: int, blocksize: int, rcp=None, want_ambiguous=False):
    """(q, absmax[, ambiguous]) as the reference's quantize_nf4. ``rcp``:
    per-block reciprocals taken from the device; without it, elements whose
    code depends on the exact rcp.approx value are flagged ambiguous."""
    x = _c(x, elem_dtype(dtype))
    n = x.size
    q = np.zeros(-(-n // 2), np.uint8)
    am = np.empty(-(-n // blocksize), np.float32)
    amb = np.zeros(n, np.uint8) if want_ambiguous else None
    r = None if rcp is None else _c(rcp, np.float32)
    lib().or_quantize_nf4(dtype, _p(x), n, blocksize, _p(r), _p(q), _p(am), _p(amb))
    return (q, am, amb.astype(bool)) if want_ambiguous else (q, am)


def quantize_8bit(x, dtype: int, blocksize: int, code, offset=None, rcp=None, want_ambiguous=False):
    x = _c(x, elem_dtype(dtype))
    n = x.size
    code = _c(code, np.float32)
    q = np.zeros(n, np.uint8)
    am = np.empty(-(-n // blocksize), np.float32)
    amb = np.zeros(n, np.uint8) if want_ambiguous else None
    off = None if offset is None else np.array([offset], np.float32)
    r = None if rcp is None else _c(rcp, np.float32)
    lib().or_quantize_8bit(dtype, _p(x), n, blocksize, _p(code), _p(off), _p(r), _p(q), _p(am), _p(amb))
    return (q, am, amb.astype(bool)) if want_ambiguous else (q, am)


def dequantize_nf4(q, absmax_, n: int, blocksize: int, dtype: int) -> np.ndarray:
    q, a = _c(q, np.uint8), _c(absmax_, np.float32)
    out = np.empty(n, elem_dtype(dtype))
    lib().or_dequantize(1, dtype, _p(q), _p(a), None, n, blocksize, None, _p(out))
    return out


def dequantize_8bit(q, absmax_, code, blocksize: int, dtype: int, offset=None) -> np.ndarray:
    q, a, code = _c(q, np.uint8), _c(absmax_, np.float32), _c(code, np.float32)
    out = np.empty(q.size, elem_dtype(dtype))
    off = None if offset is None else np.array([offset], np.float32)
    lib().or_dequantize(0, dtype, _p(q), _p(a), _p(code), q.size, blocksize, _p(off), _p(out))
    return out


def nested_absmax(absmax_q, absmax2, code2, offset: float, blocksize2: int, block0: int = 0):
    aq, a2, c2 = _c(absmax_q, np.uint8), _c(absmax2, np.float32), _c(code2, np.float32)
    out = np.empty(aq.size, np.float32)
    lib().or_nested_absmax(_p(aq), _p(a2), _p(c2), float(np.float32(offset)), aq.size,
                           blocksize2, block0, _p(out))
    return out


def mean_f32(a) -> np.float32:
    a = _c(a, np.float32)
    out = np.empty(1, np.float32)
    lib().or_mean(_p(a), a.size, _p(out))
    return out[0]


def gemv_f64(x, dtype: int, w, n_rows: int, blocksize: int, absmax_f32):
    """(y, sum|x*w|) in float64 against the float32 dequantized weight."""
    x, w, a = _c(x, elem_dtype(dtype)), _c(w, np.uint8), _c(absmax_f32, np.float32)
    m, k = x.shape
    y = np.empty((m, n_rows), np.float64)
    ya = np.empty((m, n_rows), np.float64)
    lib().or_gemv_f64(dtype, _p(x), m, k, _p(w), n_rows, blocksize, _p(a), _p(y), _p(ya))
    return y, ya


def gemv_ref(x, dtype: int, w, n_rows: int, blocksize: int, absmax_f32):
    """The reference GEMV's own float32 numerics (chunked), output in dtype."""
    x, w, a = _c(x, elem_dtype(dtype)), _c(w, np.uint8), _c(absmax_f32, np.float32)
    m, k = x.shape
    y = np.empty((m, n_rows), elem_dtype(dtype))
    lib().or_gemv_ref(dtype, _p(x), m, k, _p(w), n_rows, blocksize, _p(a), _p(y))
    return y


# ------------------------------------------------- kernel-algorithm checks

def check_nf4_buckets(stride: int = 1) -> int:
    return int(lib().or_check_nf4_buckets(stride))


def nf4_bucket_tables():
    thr = np.empty(64, np.float32)
    base = np.empty(64, np.int32)
    if lib().or_nf4_bucket_tables(_p(thr), _p(base)) != 0:
        raise AssertionError("two NF4 thresholds share a bucket")
    return thr, base


def check_q8_buckets(code, stride: int = 1):
    """(mismatches, mb) of the 8-bit kernel's bucket-table code choice against
    the literal search; mismatches -1 when the table formulation does not
    apply to this codebook (the kernel then runs the literal search)."""
    code = _c(code, np.float32)
    mb = C.c_int(0)
    bad = lib().or_check_q8_buckets(_p(code), stride, C.byref(mb))
    return int(bad), int(mb.value)


# ----------------------------------------------------- create_dynamic_map

def create_dynamic_map(signed: bool = True, max_exponent_bits: int = 7, total_bits: int = 8) -> np.ndarray:
    """The 256-entry dynamic codebook (reference kernels/quantize.py:53-88):
    per exponent level, the float32 midpoints of a float32 linspace(0.1, 1)
    scaled by a power of ten, mirrored when signed, plus 0 and 1, zero-filled
    to 256 and sorted."""
    data: list[float] = []
    non_sign_bits = total_bits - 1
    additional_items = 2 ** (non_sign_bits - max_exponent_bits) - 1
    i = 0
    for i in range(max_exponent_bits):
        items = 2 ** (i + non_sign_bits - max_exponent_bits) + 1 if signed \
            else 2 ** (i + non_sign_bits - max_exponent_bits + 1) + 1
        bounds = np.linspace(0.1, 1, int(items), dtype=np.float32)
        means = (bounds[:-1] + bounds[1:]) / 2.0
        scale = 10 ** (-(max_exponent_bits - 1) + i)
        data += (scale * means).tolist()
        if signed:
            data += (-scale * means).tolist()
    if additional_items > 0:
        bounds = np.linspace(0.1, 1, additional_items + 1, dtype=np.float32)
        means = (bounds[:-1] + bounds[1:]) / 2.0
        scale = 10 ** (-(max_exponent_bits - 1) + i)
        data += (scale * means).tolist()
        if signed:
            data += (-scale * means).tolist()
    data += [0.0, 1.0]
    data += [0.0] * (256 - len(data))
    data.sort()
    return np.array(data, np.float32)
