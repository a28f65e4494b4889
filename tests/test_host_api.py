"""Host-side behaviour of the reference-shaped API that needs no GPU: argument
errors (same exception types and messages as the reference), the
QuantizedArray container, pytree round trip, from_dict parsing."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch
import torch.utils._pytree as pytree

import bnb_b200
from bnb_b200 import QuantizedArray
from bnb_b200.kernels import dequantize_nf4, gemv_nf4, quantize_blockwise, quantize_nf4


def test_quantize_rejects_dtype_and_blocksize():
    with pytest.raises(NotImplementedError, match="quantization of torch.int32"):
        quantize_nf4(torch.zeros(8, dtype=torch.int32))
    with pytest.raises(ValueError, match="power of two"):
        quantize_nf4(torch.zeros(8), blocksize=48)
    with pytest.raises(ValueError, match="CUDA tensor"):
        quantize_nf4(torch.zeros(64))  # host tensors never run anywhere
    with pytest.raises(NotImplementedError, match="quantization to 'int4'"):
        bnb_b200.quantize(torch.zeros(64), "int4")
    with pytest.raises(AssertionError, match="256 entries"):
        quantize_blockwise(torch.zeros(64), torch.zeros(10), 64)


def test_dequantize_rejects():
    q = torch.zeros(8, dtype=torch.uint8)
    a = torch.zeros(1, dtype=torch.float32)
    with pytest.raises(NotImplementedError, match="dequantization to torch.int8"):
        dequantize_nf4(q, a, 64, torch.int8)
    with pytest.raises(ValueError, match="do not cover"):
        dequantize_nf4(torch.zeros(64, dtype=torch.uint8), a, 64, torch.float16)
    with pytest.raises(AssertionError, match="do not hold"):
        dequantize_nf4(q, a, 64, torch.float16, n=100)


def test_gemv_rejects():
    x = torch.zeros(1, 100, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="multiple of 32"):
        gemv_nf4(x, torch.zeros(50, dtype=torch.uint8), torch.zeros(2), 1, 64)
    with pytest.raises(NotImplementedError, match="float32 x"):
        gemv_nf4(torch.zeros(1, 64), torch.zeros(32, dtype=torch.uint8), torch.zeros(1), 1, 64)
    with pytest.raises(ValueError, match="blocksize must be >= 32"):
        gemv_nf4(torch.zeros(1, 64, dtype=torch.bfloat16), torch.zeros(32, dtype=torch.uint8),
                 torch.zeros(4), 1, 16)


def _qa(shape=(64, 96), nested=False):
    n = int(np.prod(shape))
    nb = n // 64
    absmax = torch.rand(nb)
    if nested:
        absmax = QuantizedArray(data=torch.zeros(nb, dtype=torch.uint8), absmax=torch.rand(-(-nb // 256)),
                                code=bnb_b200.create_dynamic_map(), offset=torch.tensor(0.1),
                                qtype="8bit", blocksize=256, shape=(nb,), dtype=torch.float32)
    return QuantizedArray(data=torch.zeros(n // 2, dtype=torch.uint8), absmax=absmax, code=None,
                          offset=None, qtype="nf4", blocksize=64, shape=shape, dtype=torch.bfloat16)


def test_container_properties():
    qa = _qa()
    assert qa.shape == (64, 96) and qa.ndim == 2 and qa.size == 64 * 96
    assert repr(qa) == "QuantizedArray(nf4, shape=(64, 96), dtype=bfloat16, blocksize=64)"
    assert qa.nbytes == 64 * 96 // 2 + 64 * 96 // 64 * 4  # reference tests/test_quantize.py:211
    assert not qa.double_quantized
    assert qa.astype(torch.float16).dtype == torch.float16
    qn = _qa(nested=True)
    assert qn.double_quantized
    assert repr(qn).endswith("blocksize=64, double_quantized)")


def test_pytree_round_trip():
    qa = _qa(nested=True)
    leaves, spec = pytree.tree_flatten(qa)
    tensors = [t for t in leaves if isinstance(t, torch.Tensor)]
    assert len(tensors) == 5  # data + the nested array's data, absmax, code, offset
    back = pytree.tree_unflatten(leaves, spec)
    assert isinstance(back, QuantizedArray) and back.double_quantized
    assert back.shape == qa.shape and back.blocksize == 64
    doubled = pytree.tree_map(lambda t: t * 2 if t is not None and t.dtype.is_floating_point else t, qa)
    assert torch.equal(doubled.absmax.absmax, qa.absmax.absmax * 2)


def _state_dict(compress: bool, packed: bool):
    qs = {"absmax": torch.rand(192), "quant_map": torch.zeros(16)}
    meta = {"quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [96, 128]}
    if compress:
        qs["absmax"] = torch.zeros(192, dtype=torch.uint8)
        qs["nested_absmax"] = torch.rand(1)
        qs["nested_quant_map"] = bnb_b200.create_dynamic_map()
        meta.update({"nested_blocksize": 256, "nested_offset": 0.0312, "nested_dtype": "float32"})
    if packed:
        raw = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8).copy()
        qs["quant_state.bitsandbytes__nf4"] = torch.from_numpy(raw)
    else:
        qs.update(meta)
    return qs


@pytest.mark.parametrize("packed", [True, False])
@pytest.mark.parametrize("compress", [True, False])
def test_from_dict_parsing(packed, compress):
    qs = _state_dict(compress, packed)
    q = QuantizedArray.from_dict(torch.zeros(96 * 128 // 2, dtype=torch.uint8), qs)
    assert q.shape == (96, 128) and q.dtype == torch.bfloat16 and q.blocksize == 64
    assert q.double_quantized == compress
    if compress:
        assert q.absmax.blocksize == 256 and q.absmax.qtype == "8bit"
        assert abs(float(q.absmax.offset) - 0.0312) < 1e-7


def test_from_dict_errors():
    qs = _state_dict(False, False)
    qs["quant_type"] = "fp4"
    with pytest.raises(NotImplementedError, match="fp4"):
        QuantizedArray.from_dict(torch.zeros(8, dtype=torch.uint8), qs)
    qs = _state_dict(False, True)
    qs["another.quant_state.x"] = torch.zeros(3, dtype=torch.uint8)
    with pytest.raises(ValueError, match="exactly one packed"):
        QuantizedArray.from_dict(torch.zeros(8, dtype=torch.uint8), qs)


def test_legacy_import():
    from bnb_b200.dequantize import QuantizedArray as Q
    assert Q is bnb_b200.QuantizedArray


def test_matmul_shape_errors_before_any_compute():
    w = _qa((256, 512))
    with pytest.raises(ValueError, match="contraction"):
        bnb_b200.matmul(torch.zeros(1, 256, dtype=torch.bfloat16), w)
    w1 = _qa((512 * 64,))
    with pytest.raises(ValueError, match="2-D"):
        bnb_b200.matmul(torch.zeros(1, 512, dtype=torch.bfloat16), w1)


@pytest.mark.parametrize("compress", [True, False])
def test_shard_from_dict_takes_only_the_rank_rows(compress):
    """parallel.shard_from_dict: each rank's codes and scales are exactly its
    rows' slices of the whole weight's (host tensors here; the device copy is
    the shard's .to()), the ranks tile the rows, and a nested weight keeps
    the whole second level with the shard's first global block."""
    from bnb_b200.parallel import shard_from_dict
    n, k = 1024, 512  # 8192 blocks of 64; nested blocks of 256 -> row unit 32
    g = torch.Generator().manual_seed(1)
    weight = torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, generator=g)
    nb = n * k // 64
    qs = {"quant_map": torch.zeros(16), "quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [n, k]}
    if compress:
        qs.update({"absmax": torch.randint(0, 256, (nb,), dtype=torch.uint8, generator=g),
                   "nested_absmax": torch.rand(nb // 256, generator=g), "nested_quant_map": bnb_b200.create_dynamic_map(),
                   "nested_blocksize": 256, "nested_offset": 0.02, "nested_dtype": "float32"})
    else:
        qs["absmax"] = torch.rand(nb, generator=g)
    world, covered = 3, 0
    for rank in range(world):
        sh = shard_from_dict(weight, qs, rank, world)
        assert sh.start == covered and sh.n_rows_total == n and sh.k == k
        covered = sh.stop
        assert torch.equal(sh.data, weight[sh.start * k // 2:sh.stop * k // 2])
        b0, b1 = sh.start * k // 64, sh.stop * k // 64
        assert sh.block0 == b0
        assert torch.equal(sh.absmax, qs["absmax"][b0:b1])
        if compress:
            assert sh.start % 32 == 0  # whole nested blocks per rank
            a2, c2, off, bs2 = sh.nested
            assert torch.equal(a2, qs["nested_absmax"]) and bs2 == 256 and abs(float(off) - 0.02) < 1e-7
        else:
            assert sh.nested is None
    assert covered == n


def test_new_kernel_entries_reject_before_any_compute():
    """The 8-bit GEMV, the fused backward and the one-launch double
    quantization check shapes and dtypes on the host (no device needed)."""
    from bnb_b200.kernels import GEMV8_MAX_M, GEMV_T_MAX_M, gemv_blockwise, gemv_t_nf4, quantize_nf4_dq
    from bnb_b200.kernels.gemv import gemv_blockwise_applies, gemv_t_applies

    assert gemv_blockwise_applies(1, 256, 64) and gemv_blockwise_applies(GEMV8_MAX_M, 128, 32)
    assert not gemv_blockwise_applies(GEMV8_MAX_M + 1, 256, 64)
    assert not gemv_blockwise_applies(1, 320, 64)           # K % 128 != 0
    assert not gemv_blockwise_applies(1, 256, 16)           # blocks below 32
    assert gemv_t_applies(GEMV_T_MAX_M, 512, 1000) and not gemv_t_applies(GEMV_T_MAX_M + 1, 512, 1000)
    assert not gemv_t_applies(1, 320, 1000)                 # K % 256 != 0

    codes = torch.zeros(64 * 256, dtype=torch.uint8)
    absmax = torch.ones(64 * 256 // 64)
    code = torch.linspace(-1, 1, 256)
    with pytest.raises(ValueError):                         # more rows than the kernel takes
        gemv_blockwise(torch.zeros(GEMV8_MAX_M + 1, 256, dtype=torch.bfloat16), codes, absmax, code, 64, 64)
    with pytest.raises(NotImplementedError):                # float32 x
        gemv_blockwise(torch.zeros(1, 256), codes, absmax, code, 64, 64)
    with pytest.raises(ValueError):                         # K % 128 != 0
        gemv_blockwise(torch.zeros(1, 192, dtype=torch.bfloat16), codes[:64 * 192], absmax, code, 64, 64)
    with pytest.raises(ValueError):                         # host tensors
        gemv_blockwise(torch.zeros(1, 256, dtype=torch.bfloat16), codes, absmax, code, 64, 64)

    nf4 = torch.zeros(64 * 512 // 2, dtype=torch.uint8)
    scales = torch.ones(64 * 512 // 64)
    with pytest.raises(ValueError):                         # g must be (M, n_rows)
        gemv_t_nf4(torch.zeros(1, 63, dtype=torch.bfloat16), nf4, scales, 64, 512, 64)
    with pytest.raises(ValueError):                         # more rows of g than the kernel takes
        gemv_t_nf4(torch.zeros(GEMV_T_MAX_M + 1, 64, dtype=torch.bfloat16), nf4, scales, 64, 512, 64)
    with pytest.raises(NotImplementedError):                # float32 g
        gemv_t_nf4(torch.zeros(1, 64), nf4, scales, 64, 512, 64)
    with pytest.raises(ValueError):                         # blocks below 32
        gemv_t_nf4(torch.zeros(1, 64, dtype=torch.bfloat16), nf4, scales, 64, 512, 16)
    with pytest.raises(ValueError):                         # host tensors
        gemv_t_nf4(torch.zeros(1, 64, dtype=torch.bfloat16), nf4, scales, 64, 512, 64)

    with pytest.raises(ValueError):                         # nothing to quantize
        quantize_nf4_dq(torch.zeros(0, dtype=torch.bfloat16), 64)
