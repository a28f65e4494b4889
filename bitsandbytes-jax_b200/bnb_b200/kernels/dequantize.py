"""Blockwise NF4 / 8-bit dequantization on flat CUDA tensors (sm_100a kernels).

Mirrors the reference's bnb_jax.kernels.dequantize (kernels/dequantize.py):
element i decodes as ``T(table[q_i] * absmax[i // blocksize])`` with a
flush-to-zero float32 multiply and a round-to-nearest conversion, bitwise the
reference's values. The ``cutejax.call`` (:110-116) is replaced by the C ABI;
the pad (:105-109) and slice (:117) copies do not exist.

``dequantize_nf4_nested`` / ``dequantize_blockwise_nested`` (extensions) decode
a double-quantized array in one kernel, bitwise equal to the reference's chain
``absmax.dequantize(float32)`` -> ``+ offset`` -> decode (array.py:95-108).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib

NF4_TABLE = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
], dtype=np.float32)

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _log2_blocksize(blocksize: int) -> int:
    if blocksize < 8 or blocksize & (blocksize - 1):
        raise ValueError(f"blocksize must be a power of two >= 8, got {blocksize}")
    return blocksize.bit_length() - 1


def _check(quantized: torch.Tensor, absmax: torch.Tensor | None, n: int, blocksize: int, dtype):
    if dtype not in _DTYPES:
        raise NotImplementedError(f"dequantization to {dtype} is not implemented")
    _log2_blocksize(blocksize)
    assert quantized.dtype == torch.uint8, quantized.dtype
    if absmax is not None:
        if absmax.numel() * blocksize < n:
            raise ValueError(f"{absmax.numel()} absmax values do not cover {n} elements "
                             f"with blocksize {blocksize}")


def dequantize_nf4(quantized: torch.Tensor, absmax: torch.Tensor, blocksize: int = 64,
                   dtype: torch.dtype = torch.float16, n: int | None = None) -> torch.Tensor:
    """Dequantize packed NF4 codes (two per byte) to a flat ``dtype`` tensor of
    ``n`` elements (default ``2 * quantized.numel()``; one fewer when the last
    byte holds a single code). (reference kernels/dequantize.py:120-134)"""
    if n is None:
        n = quantized.numel() * 2
    assert -(-n // 2) == quantized.numel(), f"{quantized.numel()} bytes do not hold {n} codes"
    assert absmax.dtype == torch.float32, absmax.dtype
    _check(quantized, absmax, n, blocksize, dtype)
    _lib.require_cuda(quantized, absmax)
    q = _lib.aligned(quantized.reshape(-1))
    a = _lib.aligned(absmax.reshape(-1), 4)
    out = torch.empty(n, dtype=dtype, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("bnbq_dequantize_nf4", _lib.DTYPE_CODE[dtype], q.data_ptr(), a.data_ptr(), n,
                  blocksize, out.data_ptr(), _lib.stream_of(q))
    return out


def dequantize_blockwise(quantized: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor,
                         blocksize: int = 64, dtype: torch.dtype = torch.float16, *,
                         offset: torch.Tensor | None = None) -> torch.Tensor:
    """Dequantize an 8-bit blockwise quantized tensor with codebook ``code``.
    ``offset`` (keyword extension, float32 output only) adds the nested offset
    in the same pass. (reference kernels/dequantize.py:137-148)"""
    n = quantized.numel()
    assert absmax.dtype == torch.float32, absmax.dtype
    _check(quantized, absmax, n, blocksize, dtype)
    _lib.require_cuda(quantized, absmax)
    code = _lib.aligned(torch.as_tensor(code, dtype=torch.float32).reshape(-1).to(quantized.device), 4)
    assert code.numel() == 256, f"codebook must have 256 entries, got {code.numel()}"
    q = _lib.aligned(quantized.reshape(-1))
    a = _lib.aligned(absmax.reshape(-1), 4)
    off = None if offset is None else _lib.aligned(offset.reshape(1).to(torch.float32), 4)
    out = torch.empty(n, dtype=dtype, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("bnbq_dequantize_blockwise", _lib.DTYPE_CODE[dtype], q.data_ptr(), a.data_ptr(),
                  code.data_ptr(), n, blocksize, _lib.ptr(off), out.data_ptr(), _lib.stream_of(q))
    return out


def _nested_args(absmax_q, absmax2, code2, offset, device):
    aq = _lib.aligned(absmax_q.reshape(-1))
    a2 = _lib.aligned(absmax2.reshape(-1).to(torch.float32), 4)
    c2 = _lib.aligned(torch.as_tensor(code2, dtype=torch.float32).reshape(-1).to(device), 4)
    off = _lib.aligned(torch.as_tensor(offset, dtype=torch.float32).reshape(1).to(device), 4)
    return aq, a2, c2, off


def dequantize_nf4_nested(quantized: torch.Tensor, absmax_q: torch.Tensor, absmax2: torch.Tensor,
                          code2: torch.Tensor, offset: torch.Tensor, blocksize: int, blocksize2: int,
                          dtype: torch.dtype, n: int) -> torch.Tensor:
    """NF4 decode of a double-quantized array in one pass."""
    assert -(-n // 2) == quantized.numel(), f"{quantized.numel()} bytes do not hold {n} codes"
    _check(quantized, None, n, blocksize, dtype)
    _log2_blocksize(blocksize2)
    if absmax_q.numel() * blocksize < n:
        raise ValueError(f"{absmax_q.numel()} absmax values do not cover {n} elements "
                         f"with blocksize {blocksize}")
    _lib.require_cuda(quantized, absmax_q, absmax2)
    q = _lib.aligned(quantized.reshape(-1))
    aq, a2, c2, off = _nested_args(absmax_q, absmax2, code2, offset, q.device)
    out = torch.empty(n, dtype=dtype, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("bnbq_dequantize_nf4_nested", _lib.DTYPE_CODE[dtype], q.data_ptr(), aq.data_ptr(),
                  a2.data_ptr(), c2.data_ptr(), off.data_ptr(), n, blocksize, blocksize2,
                  out.data_ptr(), _lib.stream_of(q))
    return out


def dequantize_blockwise_nested(quantized: torch.Tensor, code: torch.Tensor, absmax_q: torch.Tensor,
                                absmax2: torch.Tensor, code2: torch.Tensor, offset: torch.Tensor,
                                blocksize: int, blocksize2: int, dtype: torch.dtype) -> torch.Tensor:
    """8-bit decode of a double-quantized array in one pass."""
    n = quantized.numel()
    _check(quantized, None, n, blocksize, dtype)
    _log2_blocksize(blocksize2)
    if absmax_q.numel() * blocksize < n:
        raise ValueError(f"{absmax_q.numel()} absmax values do not cover {n} elements "
                         f"with blocksize {blocksize}")
    _lib.require_cuda(quantized, absmax_q, absmax2)
    q = _lib.aligned(quantized.reshape(-1))
    code = _lib.aligned(torch.as_tensor(code, dtype=torch.float32).reshape(-1).to(q.device), 4)
    aq, a2, c2, off = _nested_args(absmax_q, absmax2, code2, offset, q.device)
    out = torch.empty(n, dtype=dtype, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("bnbq_dequantize_blockwise_nested", _lib.DTYPE_CODE[dtype], q.data_ptr(),
                  code.data_ptr(), aq.data_ptr(), a2.data_ptr(), c2.data_ptr(), off.data_ptr(), n,
                  blocksize, blocksize2, out.data_ptr(), _lib.stream_of(q))
    return out
