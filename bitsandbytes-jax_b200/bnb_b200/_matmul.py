"""``x @ w.T`` for a quantized ``w``, picking the route.

Mirrors the reference's ``bnb_jax._matmul`` (_matmul.py): same ``matmul``
signature, shape checks and errors, and the same custom backward
(``g @ w.dequantize(g.dtype)``, no gradient to ``w``, only the quantized weight
kept for the backward pass); for up to 4 rows of g (an NF4 weight, K % 256 ==
0) that product runs fused, the weight never materialized.

Routing. An NF4 weight with a bfloat16/float16 x, K % 32 == 0 and blocksize >=
32: up to GEMV_MAX_M rows of x run the fused GEMV (float32 weights, closer to
the exact product than the fallback), up to FUSED_GEMM_MAX_M rows the fused
tcgen05 dequantize-GEMM (weights decoded to x's dtype in tensor memory, the
fallback's precision, float32 accumulation), where the weight never
materializes. Above that, and for everything else, ``x @ w.dequantize(x.dtype).T``
with the dequantize on the sm_100a kernels and the product on cuBLAS: measured
on a B200, the fused GEMM wins up to M = 512 (1.03-1.75x on the Llama-3-8B
and -70B MLP shapes) and loses from M = 768 on (0.67-0.95x at 768-2048),
because each 128-row weight tile is decoded once per 256 rows of x.
"""
from __future__ import annotations

import torch

from .array import QuantizedArray
from .kernels.gemv import _CHUNK, gemv_blockwise, gemv_blockwise_applies, gemv_t_applies, gemv_t_nf4, plan_for

__all__ = ["matmul"]

FUSED_GEMM_MAX_M = 512  # rows of x up to which the fused GEMM beats dequantize + cuBLAS (B200, measured)

def matmul(x: torch.Tensor, w: QuantizedArray) -> torch.Tensor:
    """``x @ w.T`` for a 2-D quantized weight ``w`` (N, K).

    ``x`` is ``(..., K)``; the result is ``(..., N)`` in ``x.dtype``.
    Differentiable in ``x``: the gradient is ``g @ w.dequantize(g.dtype)``.
    No gradient flows to ``w``. (reference _matmul.py:19-43)"""
    if w.ndim != 2:
        raise ValueError(f"w must be a 2-D weight, got shape {w.shape}")
    n, k = w.shape
    if x.shape[-1] != k:
        raise ValueError(f"contraction mismatch: x {tuple(x.shape)} @ w.T {w.shape[::-1]}")
    flat = x.dim() == 2  # the common (M, K) case needs no reshapes (host time per call)
    xm = x if flat else x.reshape(-1, k)
    if torch.is_grad_enabled() and xm.requires_grad:
        out = _Matmul2d.apply(xm, w)
    else:  # no gradient wanted: skip the autograd node
        out = _forward(xm, w)
    return out if flat else out.reshape(*x.shape[:-1], n)


def _fused_args(w: QuantizedArray):
    absmax = w.absmax
    if isinstance(absmax, QuantizedArray):
        assert absmax.code is not None and absmax.offset is not None
        assert not isinstance(absmax.absmax, QuantizedArray)
        return absmax.data, (absmax.absmax, absmax.code, absmax.offset, absmax.blocksize)
    return absmax, None


def _forward(xm: torch.Tensor, w: QuantizedArray) -> torch.Tensor:
    if w.qtype == "8bit" and _fused8_applies(xm, w):
        scales, nested = _fused_args(w)
        return gemv_blockwise(xm, w.data, scales, w.code, w.shape[0], w.blocksize, nested=nested)
    if xm.shape[0] <= FUSED_GEMM_MAX_M and _fused_applies(xm, w):
        plan = w.__dict__.get("_bnbq_plan")
        if plan is None or plan.data is not w.data or plan.absmax is not w.absmax or plan.device != xm.device:
            scales, nested = _fused_args(w)
            plan = plan_for(w, scales, nested, xm.device)
        return plan.run(xm)
    return xm @ w.dequantize(xm.dtype).T


class _Matmul2d(torch.autograd.Function):
    """custom_vjp of the reference (_matmul.py:46-71)."""

    @staticmethod
    def forward(ctx, xm: torch.Tensor, w: QuantizedArray) -> torch.Tensor:
        ctx.w = w
        return _forward(xm, w)

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        w = ctx.w
        if (w.qtype == "nf4" and g.dtype in (torch.bfloat16, torch.float16) and g.is_cuda
                and w.blocksize >= _CHUNK and gemv_t_applies(g.shape[0], w.shape[1], w.shape[0])):
            # the reference's rule with the weight kept NF4 (measured on a B200:
            # 23.8 us against 58.0 us for dequantize + cuBLAS on config 2's weight)
            scales, nested = _fused_args(w)
            try:
                return gemv_t_nf4(g, w.data, scales, w.shape[0], w.shape[1], w.blocksize, nested=nested), None
            except NotImplementedError:
                pass  # the kernel declined this call (BNBQ_ERR_UNSUPPORTED): the rule below
        return g @ w.dequantize(g.dtype), None


def _fused_applies(xm: torch.Tensor, w: QuantizedArray) -> bool:
    return (w.qtype == "nf4"
            and xm.dtype in (torch.bfloat16, torch.float16)
            and xm.is_cuda
            and xm.shape[0] > 0
            and xm.shape[1] % _CHUNK == 0
            and w.blocksize >= _CHUNK)


def _fused8_applies(xm: torch.Tensor, w: QuantizedArray) -> bool:
    """An 8-bit weight with a 16-bit x of up to GEMV8_MAX_M rows: the fused
    8-bit GEMV (the reference always takes the fallback for 8-bit weights,
    _matmul.py:74-79)."""
    return (xm.dtype in (torch.bfloat16, torch.float16)
            and xm.is_cuda
            and w.code is not None
            and gemv_blockwise_applies(xm.shape[0], xm.shape[1], w.blocksize))
