"""The C ABI library loads and exports every entry point include/bnbq.h
declares; host-only entry points answer without a GPU. No compute is called."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "bnbq.h"
LIB = ROOT / "bitsandbytes-jax_b200" / "bnb_b200" / "libbnbq.so"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BNBQ_API\s+[\w\s\*]*?\b(bnbq_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ["bnbq_quantize_nf4", "bnbq_quantize_blockwise", "bnbq_dequantize_nf4",
              "bnbq_dequantize_blockwise", "bnbq_dequantize_nf4_nested", "bnbq_gemv_nf4",
              "bnbq_matmul_nf4", "bnbq_error_string"]:
        assert s in syms


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        pytest.fail(f"{LIB} not built (python bitsandbytes-jax_b200/build.py)")
    return ctypes.CDLL(str(LIB))


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from bnb_b200 import _lib
    assert sorted(_lib.exported_symbols()) == declared_symbols()


def test_host_only_entry_points(lib):
    lib.bnbq_error_string.restype = ctypes.c_char_p
    assert lib.bnbq_error_string(0) == b"ok"
    assert b"misaligned" in lib.bnbq_error_string(-3)
    assert lib.bnbq_error_string(12345) == b"unknown status"
    assert lib.bnbq_version() >= 100


def test_argument_errors_need_no_device(lib):
    """Bad arguments are rejected before any CUDA call (status, no launch)."""
    P = ctypes.c_void_p
    f = lib.bnbq_quantize_nf4
    f.argtypes = [ctypes.c_int, P, ctypes.c_int64, ctypes.c_int32, P, P, P]
    assert f(7, None, 16, 64, None, None, None) == -2        # unknown dtype
    assert f(0, None, 16, 48, None, None, None) == -1        # blocksize not a power of two
    assert f(0, None, 16, 64, None, None, None) == -1        # null pointers
    assert f(0, P(8), 16, 64, P(16), P(16), None) == -3      # x not 16-byte aligned
    assert f(0, None, 0, 64, None, None, None) == 0          # empty input: nothing to do
    g = lib.bnbq_gemv_nf4
    g.argtypes = [ctypes.c_int, P, ctypes.c_int32, ctypes.c_int32, P, ctypes.c_int64, ctypes.c_int32,
                  P, P, P, P, P, ctypes.c_int32, ctypes.c_int64, P, ctypes.c_int64, P]
    args = [2, P(256), 1, 100, P(256), 8, 64, P(256), None, None, None, None, 0, 0, P(256), 8, None]
    assert g(*args) == -1                                     # K % 32 != 0
    args[3] = 128; args[0] = 0
    assert g(*args) == -2                                     # float32 x
    args[0] = 2; args[2] = 21
    assert g(*args) == -1                                     # M above the GEMV limit


def test_gemv_blockwise_host_checks(lib):
    """The 8-bit-weight GEMV: workspace size and argument errors, no device."""
    P = ctypes.c_void_p
    n = ctypes.c_int64(0)
    w = lib.bnbq_gemv_blockwise_workspace_bytes
    w.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, P]
    assert w(1, 14336, 4096, ctypes.byref(n)) == 0
    assert n.value == 4096 // 32 * (14336 // 128) * 1 * 32 * 4  # one float per (unit, row, x row)
    assert w(5, 14336, 4096, ctypes.byref(n)) == -1            # above BNBQ_GEMV8_MAX_M
    assert w(1, 14336 + 32, 4096, ctypes.byref(n)) == -2       # K % 128 != 0
    g = lib.bnbq_gemv_blockwise_ws
    g.argtypes = [ctypes.c_int, P, ctypes.c_int32, ctypes.c_int32, P, ctypes.c_int64, ctypes.c_int32, P,
                  P, P, P, P, P, ctypes.c_int32, ctypes.c_int64, P, ctypes.c_int64, P, ctypes.c_int64, P]
    args = [2, P(256), 1, 256, P(256), 8, 64, P(256), P(256), None, None, None, None, 0, 0, P(256), 8,
            P(256), 1 << 20, None]
    args[2] = 5
    assert g(*args) == -1                                      # M above the 8-bit GEMV limit
    args[2] = 1; args[7] = None
    assert g(*args) == -1                                      # no codebook
    args[7] = P(258)
    assert g(*args) == -3                                      # codebook not 4-byte aligned
    args[7] = P(256); args[3] = 288
    assert g(*args) == -2                                      # K % 128 != 0


def test_quantize_nf4_dq_host_checks(lib):
    """The single-pass NF4 + double quantization: workspace size and argument
    errors, no device."""
    P = ctypes.c_void_p
    lib.bnbq_quantize_nf4_dq_workspace_bytes.restype = ctypes.c_int64
    assert 16 <= lib.bnbq_quantize_nf4_dq_workspace_bytes() <= 1 << 17
    f = lib.bnbq_quantize_nf4_dq
    f.argtypes = [ctypes.c_int, P, ctypes.c_int64, ctypes.c_int32, P, ctypes.c_int32, P, P, P, P, P, P,
                  ctypes.c_int64, P]
    ok = [2, P(256), 1024, 64, P(256), 256, P(256), P(256), P(256), P(256), P(256), P(256), 1 << 20, None]
    args = list(ok); args[0] = 7
    assert f(*args) == -2                                      # unknown dtype
    args = list(ok); args[2] = 0
    assert f(*args) == -1                                      # nothing to quantize
    args = list(ok); args[11] = None
    assert f(*args) == -1                                      # no workspace
    args = list(ok); args[12] = 8
    assert f(*args) == -1                                      # workspace too small
    args = list(ok); args[5] = 512
    assert f(*args) == -2                                      # nested blocks above 256
    args = list(ok); args[11] = P(264)
    assert f(*args) == -3                                      # workspace not 16-byte aligned


def test_gemv_t_host_checks(lib):
    """The fused backward's argument errors, before any device call."""
    P = ctypes.c_void_p
    f = lib.bnbq_gemv_t_nf4_ws
    f.argtypes = [ctypes.c_int, P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, P,
                  ctypes.c_int32, P, P, P, P, P, ctypes.c_int32, ctypes.c_int64, P, ctypes.c_int64, P,
                  ctypes.c_int64, P]
    ok = [2, P(256), 1, 64, 64, 512, P(256), 64, P(256), None, None, None, None, 0, 0, P(256), 512,
          P(256), 1 << 24, None]
    args = list(ok); args[0] = 0
    assert f(*args) == -2                                      # float32 g
    args = list(ok); args[2] = 5
    assert f(*args) == -1                                      # more than 4 rows of g
    args = list(ok); args[16] = 256
    assert f(*args) == -1                                      # ldo < k
    args = list(ok); args[5] = 320; args[16] = 320
    assert f(*args) == -2                                      # K % 256 != 0
    args = list(ok); args[7] = 16
    assert f(*args) == -1                                      # blocksize below 32
    args = list(ok); args[8] = P(258)
    assert f(*args) == -3                                      # absmax not 4-byte aligned
