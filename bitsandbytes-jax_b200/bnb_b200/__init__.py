"""bitsandbytes quantization on B200 (sm_100a), the reference bnb_jax's API on torch.

Quantized tensors are :class:`QuantizedArray` pytrees, made by :func:`quantize`
or loaded from a HuggingFace bnb-4bit checkpoint with
:meth:`QuantizedArray.from_dict`, and decoded with
:meth:`QuantizedArray.dequantize` -- bitwise equal to bitsandbytes either way.
:func:`matmul` multiplies by an NF4 weight without materializing it. The
kernels themselves, on flat tensors, are in :mod:`bnb_b200.kernels`; the C ABI
they call is ``include/bnbq.h``.
(reference src/bnb_jax/__init__.py:10-20)
"""

from ._matmul import matmul
from .array import QType, QuantizedArray, quantize
from .kernels import create_dynamic_map

__all__ = [
    "QType",
    "QuantizedArray",
    "create_dynamic_map",
    "matmul",
    "quantize",
]
