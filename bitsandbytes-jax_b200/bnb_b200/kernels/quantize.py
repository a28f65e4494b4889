"""Blockwise NF4 / 8-bit quantization on flat CUDA tensors (sm_100a kernels).

Mirrors the reference's bnb_jax.kernels.quantize (kernels/quantize.py):
same function names, arguments, return values and errors, with the
``cutejax.call`` custom call (:226-233) replaced by the C ABI
``bnbq_quantize_nf4`` / ``bnbq_quantize_blockwise``. The kernels write the exact
output sizes, so the reference's pad (:221-225) and slice (:234-235) copies do
not exist. Per block: ``absmax = max |x|`` (flush-to-zero), ``r =
rcp.approx(absmax)``, ``q = code(x * r)`` -- bitwise the reference's codes.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib
from .dequantize import _log2_blocksize

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def create_dynamic_map(signed: bool = True, max_exponent_bits: int = 7, total_bits: int = 8,
                       device: torch.device | str | None = None) -> torch.Tensor:
    """The 256-entry dynamic codebook of 8-bit blockwise quantization
    (reference kernels/quantize.py:53-88; bitsandbytes' create_dynamic_map).

    Per exponent level i, the float32 midpoints of ``linspace(0.1, 1)`` scaled
    by ``10**(i - max_exponent_bits + 1)`` (mirrored when signed), then 0 and
    1, zero-filled to 256 entries and sorted. Returned as float32 on
    ``device`` (default: the CPU)."""
    data: list[float] = []
    non_sign_bits = total_bits - 1
    additional_items = 2 ** (non_sign_bits - max_exponent_bits) - 1
    i = 0
    for i in range(max_exponent_bits):
        items = (2 ** (i + non_sign_bits - max_exponent_bits) + 1 if signed
                 else 2 ** (i + non_sign_bits - max_exponent_bits + 1) + 1)
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
    return torch.tensor(np.array(data, np.float32), device=device)


def _check_input(input: torch.Tensor, blocksize: int) -> torch.Tensor:
    if input.dtype not in _DTYPES:
        raise NotImplementedError(f"quantization of {input.dtype} is not implemented")
    _log2_blocksize(blocksize)
    if blocksize > 4096:
        raise ValueError(f"blocksize must be at most 4096, got {blocksize}")
    _lib.require_cuda(input)
    return _lib.aligned(input.reshape(-1))


def quantize_nf4(input: torch.Tensor, blocksize: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize a tensor to NF4.

    Returns (quantized_u8, absmax_f32): ``ceil(n / 2)`` bytes, each holding two
    4-bit codes (high nibble first), and one absmax per block.
    (reference kernels/quantize.py:238-248)"""
    x = _check_input(input, blocksize)
    n = x.numel()
    q = torch.empty(-(-n // 2), dtype=torch.uint8, device=x.device)
    absmax = torch.empty(-(-n // blocksize), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("bnbq_quantize_nf4", _lib.DTYPE_CODE[x.dtype], x.data_ptr(), n, blocksize,
                  q.data_ptr(), absmax.data_ptr(), _lib.stream_of(x))
    return q, absmax


def quantize_nf4_dq(input: torch.Tensor, blocksize: int = 64, code2: torch.Tensor | None = None,
                    blocksize2: int = 256):
    """NF4 quantization with double-quantized scales in one kernel launch
    (``bnbq_quantize_nf4_dq``).

    Returns ``(q, absmax, absmax_q, absmax2, offset)``: the NF4 codes and the
    float32 block maxima as :func:`quantize_nf4` gives them, then
    ``offset = absmax_mean(absmax)`` and ``quantize_blockwise(absmax - offset,
    code2, blocksize2)``, all bitwise the three separate calls (the reference's
    ``quantize(..., double_quant=True)``, array.py:199-202). ``code2`` defaults
    to the dynamic map; ``blocksize2 <= 256``."""
    x = _check_input(input, blocksize)
    n = x.numel()
    if n == 0:
        raise ValueError("nothing to quantize")
    if code2 is None:
        code2 = create_dynamic_map(device=x.device)
    c2 = _lib.aligned(torch.as_tensor(code2, dtype=torch.float32).reshape(-1).to(x.device), 4)
    nb = -(-n // blocksize)
    q = torch.empty(-(-n // 2), dtype=torch.uint8, device=x.device)
    absmax = torch.empty(nb, dtype=torch.float32, device=x.device)
    absmax_q = torch.empty(nb, dtype=torch.uint8, device=x.device)
    absmax2 = torch.empty(-(-nb // blocksize2), dtype=torch.float32, device=x.device)
    offset = torch.empty((), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        stream = _lib.stream_of(x)
        ws = _lib.workspace(x.device, stream, int(_lib.lib().bnbq_quantize_nf4_dq_workspace_bytes()))
        _lib.call("bnbq_quantize_nf4_dq", _lib.DTYPE_CODE[x.dtype], x.data_ptr(), n, blocksize, c2.data_ptr(),
                  blocksize2, q.data_ptr(), absmax.data_ptr(), absmax_q.data_ptr(), absmax2.data_ptr(),
                  offset.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    return q, absmax, absmax_q, absmax2, offset


def quantize_blockwise(input: torch.Tensor, code: torch.Tensor, blocksize: int = 64, *,
                       offset: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize with 8-bit blockwise quantization and codebook ``code``.

    Returns (quantized_u8, absmax_f32). ``offset`` (a float32 scalar on the
    device, keyword-only extension) quantizes ``input - offset`` without
    materialising the difference -- the centring step of double quantization.
    (reference kernels/quantize.py:251-262)"""
    code = torch.as_tensor(code, dtype=torch.float32).reshape(-1)
    assert code.numel() == 256, f"codebook must have 256 entries, got {code.numel()}"
    x = _check_input(input, blocksize)
    code = _lib.aligned(code.to(x.device))
    n = x.numel()
    q = torch.empty(n, dtype=torch.uint8, device=x.device)
    absmax = torch.empty(-(-n // blocksize), dtype=torch.float32, device=x.device)
    off = None
    if offset is not None:
        off = _lib.aligned(torch.as_tensor(offset, dtype=torch.float32).reshape(1).to(x.device))
    with torch.cuda.device(x.device):
        _lib.call("bnbq_quantize_blockwise", _lib.DTYPE_CODE[x.dtype], x.data_ptr(), n, blocksize,
                  code.data_ptr(), _lib.ptr(off), q.data_ptr(), absmax.data_ptr(), _lib.stream_of(x))
    return q, absmax


def absmax_mean(absmax: torch.Tensor) -> torch.Tensor:
    """mean(absmax) as a float32 scalar on the device (double accumulation,
    deterministic): the offset of double quantization (reference array.py:200)."""
    a = _lib.aligned(absmax.reshape(-1).to(torch.float32))
    _lib.require_cuda(a)
    out = torch.empty((), dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        _lib.call("bnbq_absmax_mean", a.data_ptr(), a.numel(), out.data_ptr(), _lib.stream_of(a))
    return out
