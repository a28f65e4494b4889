"""Quantize parity on the B200: codes and absmax bit-exact against the CPU
oracle (which takes the device's own rcp.approx values, so nothing is left to
model), for every dtype and blocksize, one block / a partial odd last block /
2^18 elements (reference tests/test_quantize.py:35-79), plus the reference's
known-answer tests and double quantization."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200 import _lib
from bnb_b200.kernels import absmax_mean, quantize_blockwise, quantize_nf4
from helpers import DTYPE_IDS, bits, host_input, mixed_outliers, randn, to_device, to_host
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [O.F32, O.F16, O.BF16]
NF4_BLOCKSIZES = [8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]
BLOCKWISE_BLOCKSIZES = [64, 128, 256, 512, 1024, 2048, 4096]


def sizes(bs):
    return [bs, 3 * bs + 5, 1 << 18]


def device_rcp(absmax: torch.Tensor) -> np.ndarray:
    out = torch.empty_like(absmax)
    with torch.cuda.device(absmax.device):
        _lib.call("bnbq_rcp_approx_ftz", absmax.data_ptr(), out.data_ptr(), absmax.numel(),
                  _lib.stream_of(absmax))
    return to_host(out)


def check_nf4(x_host, dtype, bs):
    xt = to_device(x_host, dtype)
    q, am = quantize_nf4(xt, bs)
    am_h = to_host(am)
    assert np.array_equal(bits(am_h), bits(O.absmax(x_host, dtype, bs)))
    q_o, _ = O.quantize_nf4(x_host, dtype, bs, rcp=device_rcp(am))
    assert np.array_equal(to_host(q), q_o)
    return q, am


def check_8bit(x_host, dtype, bs, code, offset=None):
    xt = to_device(x_host, dtype)
    ct = torch.from_numpy(code).cuda()
    off_t = None if offset is None else torch.tensor(offset, dtype=torch.float32, device="cuda")
    q, am = quantize_blockwise(xt, ct, bs, offset=off_t)
    q_o, am_o = O.quantize_8bit(x_host, dtype, bs, code, offset=offset, rcp=device_rcp(am))
    assert np.array_equal(bits(to_host(am)), bits(am_o))
    assert np.array_equal(to_host(q), q_o)
    return q, am


@pytest.mark.parametrize("dtype", DTYPES, ids=DTYPE_IDS.get)
@pytest.mark.parametrize("bs", NF4_BLOCKSIZES)
def test_quantize_nf4(cuda, dtype, bs):
    for i, n in enumerate(sizes(bs)):
        check_nf4(host_input(randn(n, seed=1000 * bs + i), dtype), dtype, bs)


@pytest.mark.parametrize("dtype", DTYPES, ids=DTYPE_IDS.get)
@pytest.mark.parametrize("bs", BLOCKWISE_BLOCKSIZES)
def test_quantize_blockwise(cuda, dtype, bs):
    code = O.create_dynamic_map()
    for i, n in enumerate(sizes(bs)):
        check_8bit(host_input(mixed_outliers(n, seed=2000 * bs + i), dtype), dtype, bs, code)


def test_quantize_blockwise_user_codebooks(cuda):
    """A strictly increasing random codebook (thresholds too close for the
    bucket table: the literal search), an unsorted one and one with a
    repeated value (both the literal search)."""
    rng = np.random.default_rng(9)
    sorted_code = np.sort(rng.uniform(-1, 1, 256).astype(np.float32))
    sorted_code = np.sort(np.sign(sorted_code) * np.abs(sorted_code) ** 3).astype(np.float32)
    unsorted = O.create_dynamic_map().copy()
    unsorted[[3, 200]] = unsorted[[200, 3]]
    dup = O.create_dynamic_map().copy()
    dup[5] = dup[6]
    for code in (sorted_code, unsorted, dup):
        check_8bit(randn(3 * 256 + 5, seed=4), O.F32, 256, code)
        check_8bit(host_input(randn(1 << 14, seed=5), O.BF16), O.BF16, 64, code)


def _common_codebooks():
    from statistics import NormalDist
    nd = NormalDist()
    q = np.array([nd.inv_cdf((i + 0.5) / 256) for i in range(256)])
    return {"dynamic_unsigned": O.create_dynamic_map(False).astype(np.float32),
            "linear": np.linspace(-1.0, 1.0, 256).astype(np.float32),
            "quantile": (q / np.abs(q).max()).astype(np.float32)}


def _blocks_of(vals, bs):
    """vals in blocks of bs - 1 with a 1.0 closing each block (absmax 1)."""
    x = np.zeros(-(-len(vals) // (bs - 1)) * bs, np.float32)
    for i, start in enumerate(range(0, len(vals), bs - 1)):
        chunk = vals[start:start + bs - 1]
        x[i * bs:i * bs + len(chunk)] = chunk
        x[(i + 1) * bs - 1] = 1.0
    return x


@pytest.mark.parametrize("name", ["dynamic_unsigned", "linear", "quantile"])
def test_quantize_blockwise_common_codebooks(cuda, name):
    """Codebooks of the bitsandbytes family besides the signed dynamic map:
    the bucket table, and for the symmetric ones (middle threshold just below
    0) the table plus one direct compare. Every code, every midpoint and one
    ulp either side, zeros and the smallest denormals, and random values."""
    code = _common_codebooks()[name]
    mid = ((code[1:] + code[:-1]) * np.float32(0.5)).astype(np.float32)
    tiny = np.array([0.0, -0.0, 1e-45, -1e-45, 1.2e-38, -1.2e-38], np.float32)
    vals = np.concatenate([code, mid, np.nextafter(mid, np.float32(np.inf)),
                           np.nextafter(mid, np.float32(-np.inf)), tiny])
    check_8bit(_blocks_of(vals, 256), O.F32, 256, code)
    for dtype in (O.F16, O.BF16):
        check_8bit(host_input(mixed_outliers(3 * 4096 + 7, seed=77), dtype), dtype, 4096, code)
        check_8bit(host_input(mixed_outliers(1 << 16, seed=78), dtype), dtype, 256, code)


def test_quantize_nf4_thresholds(cuda):
    """On and one ulp either side of each threshold, absmax 1 (reference
    tests/test_quantize.py:90-99)."""
    t = O.NF4_THRESHOLDS
    vals = np.concatenate([t, np.nextafter(t, np.float32(np.inf)), np.nextafter(t, np.float32(-np.inf))])
    x = np.zeros(128, np.float32)
    x[:len(vals)] = vals
    x[63] = x[127] = 1.0
    q, am = check_nf4(x, O.F32, 64)
    codes = to_host(q)
    codes = np.stack([codes >> 4, codes & 15], 1).reshape(-1)
    j = np.arange(15)
    assert np.array_equal(codes[:15], j) and np.array_equal(codes[15:30], j + 1)
    assert np.array_equal(codes[30:45], j)


def test_quantize_blockwise_midpoints(cuda):
    code = O.create_dynamic_map()
    mid = ((code[1:] + code[:-1]) * np.float32(0.5)).astype(np.float32)
    vals = np.concatenate([code, mid, np.nextafter(mid, np.float32(np.inf)),
                           np.nextafter(mid, np.float32(-np.inf))])
    bs = 256
    x = np.zeros(-(-len(vals) // (bs - 1)) * bs, np.float32)
    for i, start in enumerate(range(0, len(vals), bs - 1)):
        chunk = vals[start:start + bs - 1]
        x[i * bs:i * bs + len(chunk)] = chunk
        x[(i + 1) * bs - 1] = 1.0
    check_8bit(x, O.F32, bs, code)


@pytest.mark.parametrize("nf4", [True, False])
def test_quantize_special_values(cuda, nf4):
    """All-zero blocks, denormal-only blocks, huge values, -0.0
    (reference tests/test_quantize.py:117-131)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal(64 * 6).astype(np.float32)
    x[0:64] = 0.0
    x[64:128] = (rng.standard_normal(64) * 1e-39).astype(np.float32)
    x[128:192] *= np.float32(1e30)
    x[192:256] = -x[192:256] * np.float32(1e-30)
    x[256] = -0.0
    if nf4:
        check_nf4(x, O.F32, 64)
        check_nf4(host_input(x, O.BF16), O.BF16, 64)
    else:
        check_8bit(x, O.F32, 64, O.create_dynamic_map())


def test_quantize_nonfinite_inputs(cuda):
    """NaN and inf inputs follow the reference's arithmetic (absmax ignores
    NaN; NaN scaled values take code 0)."""
    x = randn(64 * 4 + 3, seed=8)
    x[3] = np.nan
    x[70] = np.inf
    x[140:204] = np.nan
    check_nf4(x, O.F32, 64)
    check_8bit(x, O.F32, 64, O.create_dynamic_map())


def test_quantize_empty(cuda):
    q, am = quantize_nf4(torch.empty(0, device="cuda"), 64)
    assert q.numel() == 0 and am.numel() == 0


def test_no_writes_past_outputs(cuda):
    """Outputs are written at their exact sizes: guard bytes after q and
    absmax keep their canary values (odd n, partial last block)."""
    n, bs = 5 * 64 + 7, 64
    x = to_device(randn(n, seed=3), O.F32)
    nq, nb = -(-n // 2), -(-n // bs)
    qbuf = torch.full((nq + 64,), 0xA5, dtype=torch.uint8, device="cuda")
    abuf = torch.full((nb + 16,), -7.0, dtype=torch.float32, device="cuda")
    with torch.cuda.device(x.device):
        _lib.call("bnbq_quantize_nf4", O.F32, x.data_ptr(), n, bs, qbuf.data_ptr(), abuf.data_ptr(),
                  _lib.stream_of(x))
    assert torch.all(qbuf[nq:] == 0xA5) and torch.all(abuf[nb:] == -7.0)
    q8 = torch.full((n + 64,), 0x5A, dtype=torch.uint8, device="cuda")
    code = torch.from_numpy(O.create_dynamic_map()).cuda()
    with torch.cuda.device(x.device):
        _lib.call("bnbq_quantize_blockwise", O.F32, x.data_ptr(), n, bs, code.data_ptr(), None,
                  q8.data_ptr(), abuf.data_ptr(), _lib.stream_of(x))
    assert torch.all(q8[n:] == 0x5A) and torch.all(abuf[nb:] == -7.0)


@pytest.mark.parametrize("qtype", ["nf4", "8bit"])
def test_quantize_double_quant(cuda, qtype):
    """double_quant=True: codes bitwise; the nested absmax is the 8-bit
    quantization of (absmax - mean) with bs 256 (reference array.py:199-202)."""
    x_host = host_input(randn(1 << 16, seed=6), O.BF16)
    bs = 64 if qtype == "nf4" else 256
    qa = bnb_b200.quantize(to_device(x_host, O.BF16), qtype, bs, double_quant=True)
    assert qa.double_quantized
    absmax = qa.absmax
    assert absmax.qtype == "8bit" and absmax.blocksize == 256 and absmax.offset is not None
    # first level: same codes as without double quant
    plain = bnb_b200.quantize(to_device(x_host, O.BF16), qtype, bs)
    assert torch.equal(qa.data, plain.data)
    am = to_host(plain.absmax)
    off = to_host(absmax.offset).reshape(())
    assert abs(float(off) - float(np.mean(am.astype(np.float64)))) <= 1e-7 * float(off)
    # second level: bitwise the oracle's centred 8-bit quantization
    q2, am2 = O.quantize_8bit(am, O.F32, 256, O.create_dynamic_map(), offset=off,
                              rcp=device_rcp(absmax.absmax))
    assert np.array_equal(to_host(absmax.data), q2)
    assert np.array_equal(bits(to_host(absmax.absmax)), bits(am2))
    # the decoded absmax is close to the original
    dec = to_host(absmax.dequantize())
    assert np.allclose(dec, am, rtol=1e-2, atol=1e-6 * np.abs(am).max() + 2e-3 * np.abs(am).max())


def test_absmax_mean_matches_oracle(cuda):
    a = np.abs(randn(917_504, seed=12, scale=0.03))
    got = to_host(absmax_mean(torch.from_numpy(a).cuda())).reshape(())
    assert got == O.mean_f32(a)


def test_quantize_jit_shape(cuda):
    """Multi-dimensional input (reference tests/test_quantize.py:201-211)."""
    x = torch.randn(64, 96, device="cuda", generator=torch.Generator("cuda").manual_seed(0)).to(torch.bfloat16)
    qa = bnb_b200.quantize(x)
    assert qa.shape == (64, 96) and qa.ndim == 2 and qa.size == 64 * 96
    assert qa.dtype == torch.bfloat16
    expected = bnb_b200.quantize(x.reshape(-1))
    assert torch.equal(qa.data, expected.data)
    assert qa.dequantize().shape == (64, 96)
    assert repr(qa) == "QuantizedArray(nf4, shape=(64, 96), dtype=bfloat16, blocksize=64)"
    assert qa.nbytes == 64 * 96 // 2 + 64 * 96 // 64 * 4
