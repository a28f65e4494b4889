"""Compatibility: QuantizedArray used to live here, and downstream code still
imports it as ``from bnb_b200.dequantize import QuantizedArray``
(the reference's src/bnb_jax/dequantize.py:1-6)."""

from .array import QuantizedArray

__all__ = ["QuantizedArray"]
