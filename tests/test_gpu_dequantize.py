"""Dequantize parity on the B200: every decoded value bit-exact against the
CPU oracle, for every dtype, blocksize and partial last block (reference
tests/test_dequantize.py:68-86), the fused double-quantized decode against the
reference's three-step chain, and quantize -> dequantize round trips."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200 import QuantizedArray, _lib
from bnb_b200.kernels import (dequantize_blockwise, dequantize_blockwise_nested, dequantize_nf4,
                              dequantize_nf4_nested)
from helpers import DTYPE_IDS, TORCH_DTYPES, bits, host_input, mixed_outliers, randn, to_device, to_host
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [O.F32, O.F16, O.BF16]
BLOCKSIZES = [8, 32, 64, 128, 256, 512, 1024, 2048, 4096]


def host_quantized(nf4, n, bs, seed):
    x = randn(n, seed)
    if nf4:
        q, am = O.quantize_nf4(x, O.F32, bs)
    else:
        q, am = O.quantize_8bit(mixed_outliers(n, seed), O.F32, bs, O.create_dynamic_map())
    return q, am


@pytest.mark.parametrize("out", DTYPES, ids=DTYPE_IDS.get)
@pytest.mark.parametrize("qtype", ["nf4", "8bit"])
def test_dequantize_basic(cuda, out, qtype):
    q, am = host_quantized(qtype == "nf4", 256, 64, seed=1)
    qt, at = torch.from_numpy(q).cuda(), torch.from_numpy(am).cuda()
    if qtype == "nf4":
        got = dequantize_nf4(qt, at, 64, TORCH_DTYPES[out], n=256)
        want = O.dequantize_nf4(q, am, 256, 64, out)
    else:
        code = O.create_dynamic_map()
        got = dequantize_blockwise(qt, at, torch.from_numpy(code).cuda(), 64, TORCH_DTYPES[out])
        want = O.dequantize_8bit(q, am, code, 64, out)
    assert got.dtype == TORCH_DTYPES[out]
    assert np.array_equal(bits(to_host(got)), bits(want))


@pytest.mark.parametrize("out", DTYPES, ids=DTYPE_IDS.get)
@pytest.mark.parametrize("bs", BLOCKSIZES)
@pytest.mark.parametrize("qtype", ["nf4", "8bit"])
def test_dequantize_blocksizes(cuda, qtype, bs, out):
    """Every blocksize, with a partial odd-length last block, and 2^18."""
    code = O.create_dynamic_map()
    for n in [bs, 3 * bs + 5, (1 << 18) + 3]:
        q, am = host_quantized(qtype == "nf4", n, bs, seed=bs + n)
        qt, at = torch.from_numpy(q).cuda(), torch.from_numpy(am).cuda()
        if qtype == "nf4":
            got = dequantize_nf4(qt, at, bs, TORCH_DTYPES[out], n=n)
            want = O.dequantize_nf4(q, am, n, bs, out)
        else:
            got = dequantize_blockwise(qt, at, torch.from_numpy(code).cuda(), bs, TORCH_DTYPES[out])
            want = O.dequantize_8bit(q, am, code, bs, out)
        assert np.array_equal(bits(to_host(got)), bits(want)), n


def nested_host(n, bs, seed):
    """A double-quantized NF4 array built by the oracle (reference array.py:199-202)."""
    x = randn(n, seed, scale=0.02)
    q, am = O.quantize_nf4(x, O.F32, bs)
    off = O.mean_f32(am)
    code = O.create_dynamic_map()
    q2, am2 = O.quantize_8bit(am, O.F32, 256, code, offset=off)
    return q, q2, am2, code, off


@pytest.mark.parametrize("out", DTYPES, ids=DTYPE_IDS.get)
@pytest.mark.parametrize("n", [64, 3 * 64 + 5, 256 * 64 * 3 + 101])
def test_dequantize_nf4_nested_fused(cuda, n, out):
    """One kernel == nested 8-bit dequantize(f32) + offset, then NF4 decode."""
    q, q2, am2, code, off = nested_host(n, 64, seed=n)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    got = dequantize_nf4_nested(dev(q), dev(q2), dev(am2), dev(code),
                                torch.tensor(off, device="cuda"), 64, 256, TORCH_DTYPES[out], n)
    scales = O.dequantize_8bit(q2, am2, code, 256, O.F32, offset=off)
    want = O.dequantize_nf4(q, scales, n, 64, out)
    assert np.array_equal(bits(to_host(got)), bits(want))


def test_dequantize_blockwise_nested_fused(cuda):
    n = 5 * 256 * 256 + 9
    x = mixed_outliers(n, 3)
    code = O.create_dynamic_map()
    q, am = O.quantize_8bit(x, O.F32, 256, code)
    off = O.mean_f32(am)
    q2, am2 = O.quantize_8bit(am, O.F32, 256, code, offset=off)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    for out in DTYPES:
        got = dequantize_blockwise_nested(dev(q), dev(code), dev(q2), dev(am2), dev(code),
                                          torch.tensor(off, device="cuda"), 256, 256, TORCH_DTYPES[out])
        scales = O.dequantize_8bit(q2, am2, code, 256, O.F32, offset=off)
        assert np.array_equal(bits(to_host(got)), bits(O.dequantize_8bit(q, scales, code, 256, out)))


@pytest.mark.parametrize("dtype", DTYPES, ids=DTYPE_IDS.get)
@pytest.mark.parametrize("qtype", ["nf4", "8bit"])
def test_roundtrip(cuda, qtype, dtype):
    """quantize -> dequantize at the input dtype equals the oracle's round
    trip (reference tests/test_quantize.py:134-167)."""
    x = host_input(randn(4096 + 64, seed=21), dtype)
    qa = bnb_b200.quantize(to_device(x, dtype), qtype, 64)
    got = qa.dequantize()
    assert got.dtype == TORCH_DTYPES[dtype]
    am = to_host(qa.absmax)
    if qtype == "nf4":
        want = O.dequantize_nf4(to_host(qa.data), am, x.size, 64, dtype)
    else:
        want = O.dequantize_8bit(to_host(qa.data), am, O.create_dynamic_map(), 64, dtype)
    assert np.array_equal(bits(to_host(got)), bits(want))


@pytest.mark.parametrize("qtype", ["nf4", "8bit"])
def test_double_quant_dequantize_chain(cuda, qtype):
    """QuantizedArray.dequantize on a double-quantized array (fused kernel)
    equals the explicit chain: nested absmax decode, + offset, decode."""
    x = host_input(randn(1 << 16, seed=7), O.BF16)
    bs = 64 if qtype == "nf4" else 256
    qa = bnb_b200.quantize(to_device(x, O.BF16), qtype, bs, double_quant=True)
    fused = qa.dequantize(torch.float32)
    a = qa.absmax
    scales = dequantize_blockwise(a.data, a.absmax, a.code, 256, torch.float32) + a.offset
    chained = QuantizedArray(qa.data, scales, qa.code, None, qa.qtype, bs, qa.shape, qa.dtype)
    assert torch.equal(fused.view(torch.int32), chained.dequantize(torch.float32).view(torch.int32))
    # and the nested absmax alone, decoded at float32 in one pass
    assert torch.equal(a.dequantize().view(torch.int32), scales.view(torch.int32))


def test_dequantize_vmap_like_stack(cuda):
    """Decoding each of several stacked arrays (the reference's jit+vmap test,
    tests/test_dequantize.py:89-96) gives each array's own decode."""
    xs = torch.randn(3, 4096, device="cuda", generator=torch.Generator("cuda").manual_seed(0))
    qs = [bnb_b200.quantize(x) for x in xs]
    out = torch.stack([q.dequantize() for q in qs])
    for q, o in zip(qs, out):
        assert torch.equal(o, q.dequantize())


def test_no_writes_past_output(cuda):
    n, bs = 7 * 64 + 5, 64
    q, am = host_quantized(True, n, bs, seed=2)
    out = torch.full((n + 64,), -3.0, dtype=torch.float32, device="cuda")
    qt, at = torch.from_numpy(q).cuda(), torch.from_numpy(am).cuda()
    with torch.cuda.device(qt.device):
        _lib.call("bnbq_dequantize_nf4", O.F32, qt.data_ptr(), at.data_ptr(), n, bs, out.data_ptr(),
                  _lib.stream_of(qt))
    assert torch.all(out[n:] == -3.0)
    assert np.array_equal(bits(to_host(out[:n])), bits(O.dequantize_nf4(q, am, n, bs, O.F32)))


def test_from_dict_dequantize_matches_chain(cuda):
    """A bnb-4bit style state dict (nested) decodes as the explicit chain."""
    n = 96 * 128
    q, q2, am2, code, off = nested_host(n, 64, seed=5)
    qs = {"absmax": torch.from_numpy(q2).cuda(), "nested_absmax": torch.from_numpy(am2).cuda(),
          "nested_quant_map": torch.from_numpy(code).cuda(), "quant_map": torch.zeros(16).cuda(),
          "quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [96, 128],
          "nested_blocksize": 256, "nested_offset": float(off), "nested_dtype": "float32"}
    w = QuantizedArray.from_dict(torch.from_numpy(q).cuda(), qs)
    got = w.dequantize()
    scales = O.dequantize_8bit(q2, am2, code, 256, O.F32, offset=off)
    assert got.shape == (96, 128) and got.dtype == torch.bfloat16
    assert np.array_equal(bits(to_host(got).reshape(-1)), bits(O.dequantize_nf4(q, scales, n, 64, O.BF16)))
