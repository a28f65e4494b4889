"""The sm_100a kernels behind :class:`bnb_b200.QuantizedArray`, on flat CUDA tensors.

Same names as the reference's ``bnb_jax.kernels`` (kernels/__init__.py:6-18);
each is bitwise equal to the reference kernel of the same name.
"""

from .dequantize import (
    NF4_TABLE,
    dequantize_blockwise,
    dequantize_blockwise_nested,
    dequantize_nf4,
    dequantize_nf4_nested,
)
from .gemv import GEMV8_MAX_M, GEMV_MAX_M, GEMV_T_MAX_M, gemv_blockwise, gemv_nf4, gemv_t_nf4, matmul_nf4
from .quantize import absmax_mean, create_dynamic_map, quantize_blockwise, quantize_nf4, quantize_nf4_dq

__all__ = [
    "GEMV8_MAX_M",
    "GEMV_MAX_M",
    "GEMV_T_MAX_M",
    "NF4_TABLE",
    "absmax_mean",
    "create_dynamic_map",
    "dequantize_blockwise",
    "dequantize_blockwise_nested",
    "dequantize_nf4",
    "dequantize_nf4_nested",
    "gemv_blockwise",
    "gemv_nf4",
    "gemv_t_nf4",
    "matmul_nf4",
    "quantize_blockwise",
    "quantize_nf4",
    "quantize_nf4_dq",
]
