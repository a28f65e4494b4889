"""Fused NF4 dequantize-matmul: ``y = x @ W.T`` with W kept quantized.

Mirrors the reference's bnb_jax.kernels.gemv (kernels/gemv.py): ``gemv_nf4``
with the same arguments and errors, its ``cutejax.call`` (:195-204) replaced by
``bnbq_gemv_nf4``. Numerics as the reference: float32 partial sums per
32-element chunk, each block's scale applied once per chunk, one rounding to
x's dtype; a one-hot x returns the dequantized weights bitwise.

``matmul_nf4`` (extension) takes any number of rows: the GEMV up to
``GEMV_MAX_M``, the tcgen05 fused dequantize-GEMM above it.
"""
from __future__ import annotations

import torch

from .. import _lib
from .dequantize import _log2_blocksize

_CHUNK = 32
GEMV_MAX_M = _lib.GEMV_MAX_M
GEMV8_MAX_M = _lib.GEMV8_MAX_M  # rows of x the fused 8-bit-weight GEMV takes
_GROUP8 = 128  # elements of K per unit of the 8-bit-weight GEMV (K must be a multiple)


def _rows_per_warp(m: int) -> int:
    """The reference's tuning knob (kernels/gemv.py:207-215), kept for API
    compatibility; the sm_100a kernel chooses its own rows per CTA."""
    return 2 if m <= 2 else 4


def _f32_on(t, device) -> torch.Tensor:
    """``t`` as a float32 tensor on ``device``; no conversion call when it
    already is one (the common case: the arrays of a QuantizedArray)."""
    if isinstance(t, torch.Tensor) and t.dtype == torch.float32 and t.device == device:
        return t
    return torch.as_tensor(t, dtype=torch.float32).to(device)


def _prepare(x, data, absmax, n_rows, blocksize, nested, what):
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D (M, K), got shape {tuple(x.shape)}")
    m, k = x.shape
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"{what} of {x.dtype} x is not implemented")
    if k % _CHUNK:
        raise ValueError(f"K must be a multiple of {_CHUNK}, got {k}")
    _log2_blocksize(blocksize)
    if blocksize < _CHUNK:
        raise ValueError(f"blocksize must be >= {_CHUNK}, got {blocksize}")
    assert data.dtype == torch.uint8 and data.numel() * 2 == n_rows * k, (tuple(data.shape), n_rows, k)
    _lib.require_cuda(x, data, absmax)
    xs = _lib.aligned(x)
    w = _lib.aligned(data.reshape(-1))
    if nested is None:
        assert absmax.dtype == torch.float32, absmax.dtype
        a = _lib.aligned(absmax.reshape(-1), 4)
        extra = (a, None, None, None, None, 0)
    else:
        absmax2, code2, offset, blocksize2 = nested
        assert absmax.dtype == torch.uint8, absmax.dtype
        _log2_blocksize(blocksize2)
        aq = _lib.aligned(absmax.reshape(-1))
        a2 = _lib.aligned(_f32_on(absmax2, x.device).reshape(-1), 4)
        c2 = _lib.aligned(_f32_on(code2, x.device).reshape(-1), 4)
        off = _lib.aligned(_f32_on(offset, x.device).reshape(1), 4)
        extra = (None, aq, a2, c2, off, blocksize2)
    return xs, w, extra


def _run(entry, x, data, absmax, n_rows, blocksize, nested, absmax2_block0, out):
    xs, w, (a, aq, a2, c2, off, bs2) = _prepare(x, data, absmax, n_rows, blocksize, nested, entry)
    m, k = xs.shape
    if out is None:
        out = torch.empty((m, n_rows), dtype=x.dtype, device=x.device)
    ldy = out.stride(0)
    assert out.dtype == x.dtype and out.stride(1) == 1 and out.shape == (m, n_rows)
    stream = _lib.stream_of(xs)
    wsb = _lib.gemv_workspace_bytes(m, k, n_rows) if m <= GEMV_MAX_M else 0
    ws = _lib.workspace(x.device, stream, wsb) if wsb else None
    args = (entry + "_ws", _lib.DTYPE_CODE[x.dtype], xs.data_ptr(), m, k, w.data_ptr(), n_rows, blocksize,
            _lib.ptr(a), _lib.ptr(aq), _lib.ptr(a2), _lib.ptr(c2), _lib.ptr(off), bs2, absmax2_block0,
            out.data_ptr(), ldy, _lib.ptr(ws), 0 if ws is None else ws.numel(), stream)
    if x.device.index == torch.cuda.current_device():
        _lib.call(*args)
    else:
        with torch.cuda.device(x.device):
            _lib.call(*args)
    return out


def gemv_nf4(
    x: torch.Tensor,
    data: torch.Tensor,
    absmax: torch.Tensor,
    n_rows: int,
    blocksize: int,
    *,
    nested: tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None = None,
    rows_per_warp: int | None = None,
    absmax2_block0: int = 0,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x @ W.T`` for an NF4 weight W (n_rows, K), never materialized.

    Args:
        x: float16 or bfloat16 ``(M, K)``, ``1 <= M <= GEMV_MAX_M``,
            ``K % 32 == 0``; the result is ``(M, n_rows)`` of the same dtype.
        data: the packed NF4 codes of the row-major flattened W.
        absmax: float32 scale per block, or, if ``nested`` is given, the
            uint8 codes of the double-quantized scales.
        blocksize: power of two >= 32.
        nested: ``(absmax2, code2, offset, blocksize2)`` of a double-quantized
            absmax.
        rows_per_warp: accepted for compatibility; ignored.
        absmax2_block0: global index of this weight's first block within
            ``absmax2``'s indexing (non-zero for a row shard).
        out: optional ``(M, n_rows)`` output with unit column stride (a row
            stride larger than n_rows writes into a wider buffer).
    (reference kernels/gemv.py:148-204)"""
    del rows_per_warp
    if not 0 < x.shape[0] <= GEMV_MAX_M:
        raise ValueError(f"gemv_nf4 takes 1..{GEMV_MAX_M} rows of x, got {x.shape[0]}")
    return _run("bnbq_gemv_nf4", x, data, absmax, n_rows, blocksize, nested, absmax2_block0, out)


def matmul_nf4(
    x: torch.Tensor,
    data: torch.Tensor,
    absmax: torch.Tensor,
    n_rows: int,
    blocksize: int,
    *,
    nested: tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None = None,
    absmax2_block0: int = 0,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x @ W.T`` for any M >= 1: the GEMV up to GEMV_MAX_M rows, the fused
    tcgen05 dequantize-GEMM above (weights decoded to x's dtype in tensor
    memory, float32 accumulation: the precision of the reference's fallback
    ``x @ w.dequantize().T``). K not a multiple of 64 runs as GEMV passes."""
    if x.shape[0] < 1:
        raise ValueError("matmul_nf4 needs at least one row of x")
    return _run("bnbq_matmul_nf4", x, data, absmax, n_rows, blocksize, nested, absmax2_block0, out)


class FusedPlan:
    """The C-ABI arguments of one NF4 weight, prepared once: its codes and
    (nested) scales as aligned float32/uint8 device tensors and their
    addresses. :meth:`run` is then one ctypes call per matmul, with checks on
    x only (dtype, device, contiguity, alignment). Built by :func:`plan_for`
    and cached on the weight object."""

    __slots__ = ("data", "absmax", "n", "k", "bs", "ptrs", "bs2", "keep", "device", "_dev", "_ws", "_fn")

    def __init__(self, data, absmax, scales, n_rows, k, blocksize, nested, device):
        self.data, self.absmax = data, absmax  # the weight's own fields (identity checked on reuse)
        self.n, self.k, self.bs = n_rows, k, blocksize
        self.device = device
        self._dev = device.index
        w = _lib.aligned(data.reshape(-1))
        if nested is None:
            a = _lib.aligned(scales.reshape(-1), 4)
            self.keep = (w, a)
            self.ptrs = (w.data_ptr(), a.data_ptr(), None, None, None, None)
            self.bs2 = 0
        else:
            absmax2, code2, offset, blocksize2 = nested
            _log2_blocksize(blocksize2)
            aq = _lib.aligned(scales.reshape(-1))
            a2 = _lib.aligned(_f32_on(absmax2, device).reshape(-1), 4)
            c2 = _lib.aligned(_f32_on(code2, device).reshape(-1), 4)
            off = _lib.aligned(_f32_on(offset, device).reshape(1), 4)
            self.keep = (w, aq, a2, c2, off)
            self.ptrs = (w.data_ptr(), None, aq.data_ptr(), a2.data_ptr(), c2.data_ptr(), off.data_ptr())
            self.bs2 = blocksize2
        # (m, stream) -> (workspace pointer, bytes, the tensor: held, so that the
        # pointer stays valid even if the shared workspace is later replaced)
        self._ws: dict[tuple[int, int], tuple] = {}
        self._fn = _lib.lib().bnbq_matmul_nf4_ws

    def _workspace(self, m: int, stream: int) -> tuple:
        if m > GEMV_MAX_M:
            return None, 0, None
        nb = _lib.gemv_workspace_bytes(m, self.k, self.n)
        if not nb:
            return None, 0, None
        ws = _lib.workspace(self.device, stream, nb)
        return ws.data_ptr(), ws.numel(), ws

    def run(self, x: torch.Tensor) -> torch.Tensor:
        m = x.shape[0]
        xp = x.data_ptr()
        if xp & 15 or not x.is_contiguous():
            x = _lib.aligned(x)
            xp = x.data_ptr()
        out = x.new_empty((m, self.n))
        di = self._dev
        stream = torch._C._cuda_getCurrentRawStream(di)
        ws = self._ws.get((m, stream))
        if ws is None:
            ws = self._ws[(m, stream)] = self._workspace(m, stream)
        wp, ap, aqp, a2p, c2p, offp = self.ptrs
        args = (_lib.DTYPE_CODE[x.dtype], xp, m, self.k, wp, self.n, self.bs, ap, aqp, a2p, c2p, offp,
                self.bs2, 0, out.data_ptr(), self.n, ws[0], ws[1], stream)
        if torch._C._cuda_getDevice() == di:
            st = self._fn(*args)
        else:
            with torch.cuda.device(di):
                st = self._fn(*args)
        if st:
            _lib.check(st, "bnbq_matmul_nf4_ws")
        return out


def plan_for(w, scales, nested, device) -> FusedPlan:
    """The FusedPlan of the 2-D NF4 QuantizedArray `w` (`scales`: its float32
    absmax, or the codes of its nested absmax; `nested`: the rest of the
    nested absmax or None), cached on `w` and re-made when `w`'s data or
    absmax object is no longer the one it was made from."""
    plan = w.__dict__.get("_bnbq_plan")
    if plan is None or plan.data is not w.data or plan.absmax is not w.absmax or plan.device != device:
        n, k = w.shape
        if k % _CHUNK:
            raise ValueError(f"K must be a multiple of {_CHUNK}, got {k}")
        _log2_blocksize(w.blocksize)
        plan = FusedPlan(w.data, w.absmax, scales, n, k, w.blocksize, nested, device)
        w.__dict__["_bnbq_plan"] = plan
    return plan


def gemv_blockwise_applies(m: int, k: int, blocksize: int) -> bool:
    """Whether :func:`gemv_blockwise` takes an (m x k) x with this blocksize."""
    return 1 <= m <= GEMV8_MAX_M and k % _GROUP8 == 0 and blocksize >= _CHUNK


def gemv_blockwise(
    x: torch.Tensor,
    data: torch.Tensor,
    absmax: torch.Tensor,
    code: torch.Tensor,
    n_rows: int,
    blocksize: int,
    *,
    nested: tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None = None,
    absmax2_block0: int = 0,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x @ W.T`` for an 8-bit blockwise-quantized weight W (n_rows, K) with
    codebook ``code``, never materialized (``bnbq_gemv_blockwise_ws``).

    The reference has no such kernel: it computes ``x @ w.dequantize().T``
    for 8-bit weights (_matmul.py:58-59, routed by _matmul.py:74-79). Same
    arguments and numerics as :func:`gemv_nf4` (float32 products with the
    exact codebook value, each block's scale applied once, one rounding), plus
    the codebook; ``1 <= M <= GEMV8_MAX_M`` and ``K % 128 == 0``."""
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D (M, K), got shape {tuple(x.shape)}")
    m, k = x.shape
    if not 0 < m <= GEMV8_MAX_M:
        raise ValueError(f"gemv_blockwise takes 1..{GEMV8_MAX_M} rows of x, got {m}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"gemv_blockwise of {x.dtype} x is not implemented")
    if k % _GROUP8:
        raise ValueError(f"K must be a multiple of {_GROUP8}, got {k}")
    _log2_blocksize(blocksize)
    if blocksize < _CHUNK:
        raise ValueError(f"blocksize must be >= {_CHUNK}, got {blocksize}")
    assert data.dtype == torch.uint8 and data.numel() == n_rows * k, (tuple(data.shape), n_rows, k)
    _lib.require_cuda(x, data, absmax)
    xs = _lib.aligned(x)
    w = _lib.aligned(data.reshape(-1))
    cb = _lib.aligned(_f32_on(code, x.device).reshape(-1), 4)
    if cb.numel() != 256:
        raise ValueError(f"code must have 256 entries, got {cb.numel()}")
    if nested is None:
        assert absmax.dtype == torch.float32, absmax.dtype
        a, aq, a2, c2, off, bs2 = _lib.aligned(absmax.reshape(-1), 4), None, None, None, None, 0
    else:
        absmax2, code2, offset, bs2 = nested
        assert absmax.dtype == torch.uint8, absmax.dtype
        _log2_blocksize(bs2)
        a = None
        aq = _lib.aligned(absmax.reshape(-1))
        a2 = _lib.aligned(_f32_on(absmax2, x.device).reshape(-1), 4)
        c2 = _lib.aligned(_f32_on(code2, x.device).reshape(-1), 4)
        off = _lib.aligned(_f32_on(offset, x.device).reshape(1), 4)
    if out is None:
        out = torch.empty((m, n_rows), dtype=x.dtype, device=x.device)
    assert out.dtype == x.dtype and out.stride(1) == 1 and out.shape == (m, n_rows)
    stream = _lib.stream_of(xs)
    ws = _lib.workspace(x.device, stream, _lib.gemv8_workspace_bytes(m, k, n_rows))
    args = ("bnbq_gemv_blockwise_ws", _lib.DTYPE_CODE[x.dtype], xs.data_ptr(), m, k, w.data_ptr(), n_rows,
            blocksize, cb.data_ptr(), _lib.ptr(a), _lib.ptr(aq), _lib.ptr(a2), _lib.ptr(c2), _lib.ptr(off), bs2,
            absmax2_block0, out.data_ptr(), out.stride(0), ws.data_ptr(), ws.numel(), stream)
    if x.device.index == torch.cuda.current_device():
        _lib.call(*args)
    else:
        with torch.cuda.device(x.device):
            _lib.call(*args)
    return out


GEMV_T_MAX_M = 4  # rows of g the fused backward takes


def gemv_t_applies(m: int, k: int, n_rows: int) -> bool:
    """Whether :func:`gemv_t_nf4` takes this shape."""
    return 1 <= m <= GEMV_T_MAX_M and k % 256 == 0 and n_rows <= (1 << 29)


def gemv_t_nf4(
    g: torch.Tensor,
    data: torch.Tensor,
    absmax: torch.Tensor,
    n_rows: int,
    k: int,
    blocksize: int,
    *,
    nested: tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None = None,
    absmax2_block0: int = 0,
) -> torch.Tensor:
    """``g @ W`` for an NF4 weight W (n_rows, k), never materialized
    (``bnbq_gemv_t_nf4_ws``): the backward of :func:`bnb_b200.matmul` for up to
    GEMV_T_MAX_M rows of g. The reference computes ``g @ w.dequantize(g.dtype)``
    (_matmul.py:67-68); here every weight is its exact float32 dequantized
    value, accumulated in float32 and rounded once, so a one-hot g returns the
    dequantized weight row bitwise."""
    if g.dim() != 2 or g.shape[1] != n_rows:
        raise ValueError(f"g must be (M, {n_rows}), got {tuple(g.shape)}")
    m = g.shape[0]
    if g.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"gemv_t_nf4 of {g.dtype} g is not implemented")
    if not gemv_t_applies(m, k, n_rows):
        raise ValueError(f"gemv_t_nf4 takes 1..{GEMV_T_MAX_M} rows, K % 256 == 0, got M={m}, K={k}")
    _log2_blocksize(blocksize)
    if blocksize < _CHUNK:
        raise ValueError(f"blocksize must be >= {_CHUNK}, got {blocksize}")
    assert data.dtype == torch.uint8 and data.numel() * 2 == n_rows * k, (tuple(data.shape), n_rows, k)
    _lib.require_cuda(g, data, absmax)
    gs = g if g.stride(1) == 1 and g.data_ptr() % 2 == 0 else g.contiguous()
    w = _lib.aligned(data.reshape(-1))
    if nested is None:
        assert absmax.dtype == torch.float32, absmax.dtype
        a, aq, a2, c2, off, bs2 = _lib.aligned(absmax.reshape(-1), 4), None, None, None, None, 0
    else:
        absmax2, code2, offset, bs2 = nested
        assert absmax.dtype == torch.uint8, absmax.dtype
        _log2_blocksize(bs2)
        a = None
        aq = _lib.aligned(absmax.reshape(-1))
        a2 = _lib.aligned(_f32_on(absmax2, g.device).reshape(-1), 4)
        c2 = _lib.aligned(_f32_on(code2, g.device).reshape(-1), 4)
        off = _lib.aligned(_f32_on(offset, g.device).reshape(1), 4)
    out = torch.empty((m, k), dtype=g.dtype, device=g.device)
    stream = _lib.stream_of(gs)
    ws = _lib.workspace(g.device, stream, _lib.gemv_t_workspace_bytes(m, k, n_rows))
    args = ("bnbq_gemv_t_nf4_ws", _lib.DTYPE_CODE[g.dtype], gs.data_ptr(), m, n_rows, gs.stride(0), k, w.data_ptr(),
            blocksize, _lib.ptr(a), _lib.ptr(aq), _lib.ptr(a2), _lib.ptr(c2), _lib.ptr(off), bs2, absmax2_block0,
            out.data_ptr(), k, ws.data_ptr(), ws.numel(), stream)
    if g.device.index == torch.cuda.current_device():
        _lib.call(*args)
    else:
        with torch.cuda.device(g.device):
            _lib.call(*args)
    return out
