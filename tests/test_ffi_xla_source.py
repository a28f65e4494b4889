"""The XLA FFI handlers (csrc/ffi_xla.cc) type-check against include/bnbq.h.

jaxlib is absent here, so the file is compiled with g++ -fsyntax-only against
a minimal stand-in for its FFI header (tests/ffi_stub): every handler's call
into the C ABI -- argument count, order and types -- is checked; the binding
itself needs the real headers (build.py compiles the handlers where they are
found)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


CUDA_INC = Path(shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc").resolve().parent.parent / "include"


@pytest.mark.skipif(shutil.which("g++") is None or not (CUDA_INC / "cuda_runtime_api.h").exists(),
                    reason="needs g++ and the CUDA headers")
def test_ffi_handlers_type_check():
    cuda_inc = CUDA_INC
    cmd = ["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
           f"-I{ROOT / 'tests' / 'ffi_stub'}", f"-I{cuda_inc}", str(ROOT / "bitsandbytes-jax_b200/csrc/ffi_xla.cc")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_ffi_handlers_cover_every_reference_call_site():
    src = (ROOT / "bitsandbytes-jax_b200/csrc/ffi_xla.cc").read_text()
    for entry in ("bnbq_quantize_nf4(", "bnbq_quantize_blockwise(", "bnbq_absmax_mean(", "bnbq_dequantize_nf4(",
                  "bnbq_dequantize_blockwise(", "bnbq_dequantize_nf4_nested(", "bnbq_dequantize_blockwise_nested(",
                  "bnbq_matmul_nf4_ws(", "bnbq_gemv_blockwise_ws(", "bnbq_gemv_t_nf4_ws(", "bnbq_quantize_nf4_dq("):
        assert entry in src, entry
