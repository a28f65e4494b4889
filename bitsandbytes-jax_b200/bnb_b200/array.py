"""QuantizedArray: a bitsandbytes-quantized tensor on a CUDA device.

Mirrors the reference's ``bnb_jax.array`` (array.py): the same dataclass
fields, properties, ``dequantize``, ``from_dict`` and ``quantize`` with the
same arguments and errors. Leaves are torch tensors; the class is registered as
a torch pytree node (leaves ``data, absmax, code, offset``; static ``qtype,
blocksize, shape, dtype``), as the reference registers a JAX pytree.

Differences of mechanism, not of result:
* a double-quantized array decodes in ONE kernel (the nested scale is decoded
  in-kernel), bitwise equal to the reference's three-step chain (:95-108);
* double quantization computes the offset with a deterministic on-device mean
  and centres the absmax inside the 8-bit quantize kernel (:199-202).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field, replace
from typing import Any, Literal

import numpy as np
import torch
import torch.utils._pytree as pytree

from .kernels import (
    absmax_mean,
    create_dynamic_map,
    dequantize_blockwise,
    dequantize_blockwise_nested,
    dequantize_nf4,
    dequantize_nf4_nested,
    quantize_blockwise,
    quantize_nf4,
    quantize_nf4_dq,
)

__all__ = ["QType", "QuantizedArray", "quantize"]

QType = Literal["nf4", "8bit"]
"""``"nf4"``: 4-bit NormalFloat, two codes per byte (bitsandbytes'
``quantize_4bit``). ``"8bit"``: 8-bit blockwise with a 256-entry codebook
(``quantize_blockwise``)."""

# bitsandbytes' double quantization: absmax is itself 8-bit quantized in
# blocks of this size, around its mean (reference array.py:30).
_NESTED_BLOCKSIZE = 256
# Largest tensor that double-quantizes in the single launch: measured on a
# B200, the one-launch kernel matches the three launches at 2^24 elements
# (35.3 vs 35.8 us) and falls behind above (90 vs 78 us at 4096 x 14336): its
# NF4 pass runs with the occupancy of the whole kernel and without the CTAs
# that do the nested pass.
_SINGLE_PASS_MAX = 1 << 24

_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _dtype_name(dtype: torch.dtype) -> str:
    return str(dtype).removeprefix("torch.")


@dataclass
class QuantizedArray:
    """Codes of a flattened tensor, the scale of each block of ``blocksize``
    codes, and what it takes to turn them back into values.

    Decoding element ``i``: look its code up (the built-in NF4 table, or the
    256-entry ``code`` of an 8-bit array), multiply by its block's scale
    ``absmax[i // blocksize]``, and add ``offset`` when there is one.

    Fields:
        data: the uint8 codes. NF4 packs two per byte, the even element in
            the high nibble (``ceil(size / 2)`` bytes); 8-bit uses one byte
            per element.
        absmax: the block scales, float32 -- or, for a double-quantized
            array, an 8-bit QuantizedArray that holds them.
        code: an 8-bit array's float32 codebook; None for NF4.
        offset: a float32 scalar added after decoding; only the nested absmax
            of a double-quantized array has one (its values were centred on
            their mean before quantizing).
        qtype: ``"nf4"`` or ``"8bit"``.
        blocksize: codes per scale.
        shape: the decoded tensor's shape.
        dtype: what :meth:`dequantize` returns unless told otherwise.
    Same fields and meaning as the reference's dataclass (array.py:35-68).
    """

    data: torch.Tensor
    absmax: torch.Tensor | QuantizedArray
    code: torch.Tensor | None
    offset: torch.Tensor | None
    qtype: QType = field(metadata={"static": True})
    blocksize: int = field(metadata={"static": True})
    shape: tuple[int, ...] = field(metadata={"static": True})
    dtype: torch.dtype = field(default=torch.bfloat16, metadata={"static": True})

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def size(self) -> int:
        return math.prod(self.shape)

    @property
    def nbytes(self) -> int:
        """Bytes held by all the leaves: codes, scales, codebook."""
        return sum(t.numel() * t.element_size() for t in pytree.tree_leaves(self)
                   if isinstance(t, torch.Tensor))

    @property
    def double_quantized(self) -> bool:
        return isinstance(self.absmax, QuantizedArray)

    @property
    def device(self) -> torch.device:
        return self.data.device

    def astype(self, dtype) -> QuantizedArray:
        """Return a copy whose default dequantization dtype is ``dtype``."""
        return replace(self, dtype=dtype)

    def dequantize(self, dtype=None) -> torch.Tensor:
        """Decode to a dense tensor of ``dtype`` (default: ``self.dtype``),
        bitwise equal to bitsandbytes' dequantization (reference array.py:91-109)."""
        dtype = self.dtype if dtype is None else dtype
        absmax = self.absmax
        if self.qtype not in ("nf4", "8bit"):
            raise NotImplementedError(f"dequantization of {self.qtype!r} is not implemented")
        if self.qtype == "8bit":
            assert self.code is not None, "8bit QuantizedArray without a codebook"
        if isinstance(absmax, QuantizedArray) and _fusable(absmax):
            assert absmax.code is not None and absmax.offset is not None
            if self.qtype == "nf4":
                out = dequantize_nf4_nested(self.data, absmax.data, absmax.absmax, absmax.code,
                                            absmax.offset, self.blocksize, absmax.blocksize,
                                            dtype, self.size)
            else:
                out = dequantize_blockwise_nested(self.data, self.code, absmax.data, absmax.absmax,
                                                  absmax.code, absmax.offset, self.blocksize,
                                                  absmax.blocksize, dtype)
        else:
            if isinstance(absmax, QuantizedArray):
                absmax = absmax.dequantize(torch.float32)
            if self.qtype == "nf4":
                out = dequantize_nf4(self.data, absmax, blocksize=self.blocksize, dtype=dtype,
                                     n=self.size)
            elif self.offset is not None and dtype == torch.float32:
                # the nested-absmax decode + its offset, in one pass (:103-108)
                return dequantize_blockwise(self.data, absmax, self.code, blocksize=self.blocksize,
                                            dtype=dtype, offset=self.offset).reshape(self.shape)
            else:
                out = dequantize_blockwise(self.data, absmax, self.code, blocksize=self.blocksize,
                                           dtype=dtype)
        if self.offset is not None:
            out = out + self.offset.to(out.dtype)
        return out.reshape(self.shape)

    def __repr__(self) -> str:
        nested = ", double_quantized" if self.double_quantized else ""
        return (f"QuantizedArray({self.qtype}, shape={self.shape}, "
                f"dtype={_dtype_name(self.dtype)}, blocksize={self.blocksize}{nested})")

    @classmethod
    def from_dict(cls, weight: torch.Tensor, qs_dict: dict[str, Any]) -> QuantizedArray:
        """A QuantizedArray over a 4-bit weight saved by HuggingFace with
        bitsandbytes (keys as the reference reads them, array.py:116-163).

        ``weight``: the uint8 tensor of packed codes. ``qs_dict``: the entries
        stored next to it, keyed by what follows the weight's name --
        ``absmax``, ``quant_map``, the ``nested_*`` entries of a
        double-quantized weight, and the metadata, given either as separate
        keys or packed into one ``quant_state.bitsandbytes__nf4`` tensor of
        JSON bytes.
        """
        qs_dict = dict(qs_dict)  # the caller's dict is left as it was
        packed = [k for k, v in qs_dict.items() if "quant_state" in k and isinstance(v, torch.Tensor)]
        if "quant_type" not in qs_dict:
            if len(packed) != 1:
                raise ValueError(f"expected exactly one packed quant_state item, found {packed}")
            qs_dict.update(_unpack_tensor_to_dict(qs_dict.pop(packed[0])))
        qs_dict = {k.split(".")[-1]: v for k, v in qs_dict.items()}  # keep the last dotted part of each key

        if qs_dict["quant_type"] != "nf4":
            raise NotImplementedError(f"quant_type {qs_dict['quant_type']!r} is not supported")

        absmax = qs_dict["absmax"]
        if "nested_absmax" in qs_dict:
            assert qs_dict["nested_dtype"] == "float32", qs_dict["nested_dtype"]
            absmax = cls(
                data=absmax.reshape(-1),
                absmax=qs_dict["nested_absmax"].reshape(-1),
                code=qs_dict["nested_quant_map"].reshape(-1),
                offset=torch.tensor(float(qs_dict["nested_offset"]), dtype=torch.float32,
                                    device=absmax.device),
                qtype="8bit",
                blocksize=int(qs_dict["nested_blocksize"]),
                shape=tuple(absmax.shape),
                dtype=torch.float32,
            )
        else:
            absmax = absmax.reshape(-1)

        # the saved quant_map is not stored: decoding always uses the NF4
        # table built into the kernels (so does bitsandbytes)
        return cls(
            data=weight.reshape(-1),
            absmax=absmax,
            code=None,
            offset=None,
            qtype="nf4",
            blocksize=int(qs_dict["blocksize"]),
            shape=tuple(int(s) for s in qs_dict["shape"]),
            dtype=_DTYPES[qs_dict["dtype"]],
        )


def _fusable(absmax: QuantizedArray) -> bool:
    """A nested absmax the one-pass kernels decode: 8-bit, centred, flat scales."""
    return (absmax.qtype == "8bit" and absmax.offset is not None and absmax.code is not None
            and isinstance(absmax.absmax, torch.Tensor))


def _flatten(qa: QuantizedArray):
    return [qa.data, qa.absmax, qa.code, qa.offset], (qa.qtype, qa.blocksize, qa.shape, qa.dtype)


def _unflatten(leaves, ctx):
    qtype, blocksize, shape, dtype = ctx
    data, absmax, code, offset = leaves
    return QuantizedArray(data, absmax, code, offset, qtype, blocksize, shape, dtype)


pytree.register_pytree_node(
    QuantizedArray, _flatten, _unflatten,
    serialized_type_name="bnb_b200.array.QuantizedArray",
)


def quantize(
    array: torch.Tensor,
    qtype: QType = "nf4",
    blocksize: int = 64,
    *,
    code: torch.Tensor | None = None,
    double_quant: bool = False,
    dtype=None,
) -> QuantizedArray:
    """Blockwise quantization with bitsandbytes' codes and scales, bit for bit
    (same arguments as the reference's ``quantize``, array.py:166-213).

    Args:
        array: the values (a CUDA tensor of float16, bfloat16 or float32, any
            shape), quantized as one flat run.
        qtype: ``"nf4"`` (bitsandbytes' ``quantize_4bit``) or ``"8bit"``
            (``quantize_blockwise``).
        blocksize: a power of two (bitsandbytes accepts 32..4096 for NF4 and
            64..4096 for 8-bit).
        code: the 8-bit codebook; the dynamic map when omitted.
        double_quant: quantize the block scales as well, 8-bit in blocks of
            256 around their mean (bitsandbytes' ``compress_statistics``).
            That mean is a float32 rounding of its own, which may differ from
            torch's in the last bit, so this one value is not bitwise.
        dtype: the result's default decoding dtype (``array.dtype`` when
            omitted).
    """
    x = array.reshape(-1)
    if qtype == "nf4" and double_quant and 0 < x.numel() <= _SINGLE_PASS_MAX:
        # the three steps below in one launch (bnbq_quantize_nf4_dq), bitwise the same
        code2 = create_dynamic_map(device=x.device)
        data, absmax, q2, absmax2, offset = quantize_nf4_dq(x, blocksize, code2, _NESTED_BLOCKSIZE)
        absmax = QuantizedArray(data=q2, absmax=absmax2, code=code2, offset=offset,
                                qtype="8bit", blocksize=_NESTED_BLOCKSIZE, shape=tuple(absmax.shape),
                                dtype=torch.float32)
        return QuantizedArray(data=data, absmax=absmax, code=None, offset=None, qtype=qtype, blocksize=blocksize,
                              shape=tuple(array.shape), dtype=array.dtype if dtype is None else dtype)
    if qtype == "nf4":
        data, absmax = quantize_nf4(x, blocksize=blocksize)
        code = None
    elif qtype == "8bit":
        code = (create_dynamic_map(device=x.device) if code is None
                else torch.as_tensor(code, dtype=torch.float32).reshape(-1).to(x.device))
        data, absmax = quantize_blockwise(x, code, blocksize=blocksize)
    else:
        raise NotImplementedError(f"quantization to {qtype!r} is not implemented")

    if double_quant:
        offset = absmax_mean(absmax)
        code2 = create_dynamic_map(device=x.device)
        q2, absmax2 = quantize_blockwise(absmax, code2, blocksize=_NESTED_BLOCKSIZE, offset=offset)
        absmax = QuantizedArray(data=q2, absmax=absmax2, code=code2, offset=offset, qtype="8bit",
                                blocksize=_NESTED_BLOCKSIZE, shape=tuple(absmax.shape),
                                dtype=torch.float32)

    return QuantizedArray(
        data=data,
        absmax=absmax,
        code=code,
        offset=None,
        qtype=qtype,
        blocksize=blocksize,
        shape=tuple(array.shape),
        dtype=array.dtype if dtype is None else dtype,
    )


def _unpack_tensor_to_dict(tensor: torch.Tensor) -> dict[str, Any]:
    return json.loads(bytes(np.asarray(tensor.detach().cpu().numpy(), dtype=np.uint8)).decode("utf-8"))
