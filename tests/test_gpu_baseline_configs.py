"""Parity at the benchmark configurations themselves, at their full sizes,
against the CPU oracle (reference tests/test_quantize.py:35-79 and
tests/test_matmul.py:18-44 for the checks; the sizes and distributions are
the benchmark's):

* config 1 -- one 4096 x 4096 bf16 tensor, N(0, 0.02^2) from seed 0, NF4
  blocksize 64, float32 absmax: codes, absmax and the dequantized bf16 values
  bitwise;
* config 3 -- 2^28 + 37 elements (a partial last block) of 90% N(0, 1) and 10%
  Laplace(0, 8), in f32 / f16 / bf16, 8-bit dynamic map at blocksizes 256 and
  4096: codes, absmax and decoded values bitwise;
* config 2 -- the 4096 x 14336 double-quantized GEMV at every benchmarked M
  (1, 2, 4, 8, 16, 20), against the oracle's float64 product computed from the
  raw codes and the oracle's own decode of the nested scales;
* config 5 -- both Llama-3-70B MLP shapes (28672 x 8192 and 8192 x 28672,
  N(0, 0.015^2)) at M = 64 and 2048, on sampled weight rows, against the
  float64 product of x and the oracle-decoded weight rounded to bf16 (the
  fallback's operands).

The oracle takes the device's own rcp.approx reciprocals for the code choice
(bnbq_rcp_approx_ftz), so code comparisons are exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200 import _lib
from bnb_b200.kernels import dequantize_blockwise, dequantize_nf4, quantize_blockwise, quantize_nf4
from helpers import GEMV_ATOL, GEMV_RTOL, bits, host_input, mixed_outliers, to_device, to_host
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


def device_rcp(absmax: torch.Tensor) -> np.ndarray:
    out = torch.empty_like(absmax)
    _lib.call("bnbq_rcp_approx_ftz", absmax.data_ptr(), out.data_ptr(), absmax.numel(), _lib.stream_of(absmax))
    return to_host(out)


def test_config1_nf4_round_trip_bitwise(cuda):
    n = 4096 * 4096
    w = (np.random.default_rng(0).standard_normal(n) * 0.02).astype(np.float32)
    xh = host_input(w, O.BF16)
    q, am = quantize_nf4(to_device(xh, O.BF16), 64)
    am_h = to_host(am)
    assert np.array_equal(bits(am_h), bits(O.absmax(xh, O.BF16, 64)))
    q_o, _ = O.quantize_nf4(xh, O.BF16, 64, rcp=device_rcp(am))
    assert np.array_equal(to_host(q), q_o)
    out = dequantize_nf4(q, am, 64, torch.bfloat16)
    assert np.array_equal(bits(to_host(out)), bits(O.dequantize_nf4(q_o, am_h, n, 64, O.BF16)))


@pytest.fixture(scope="module")
def config3_values():
    return mixed_outliers((1 << 28) + 37, seed=3)


@pytest.mark.parametrize("bs", [256, 4096])
@pytest.mark.parametrize("dtype", [O.F32, O.F16, O.BF16], ids=["f32", "f16", "bf16"])
def test_config3_8bit_full_size_bitwise(cuda, config3_values, dtype, bs):
    code = O.create_dynamic_map()
    xh = host_input(config3_values, dtype)
    xt = to_device(xh, dtype)
    ct = torch.from_numpy(code).to(cuda)
    q, am = quantize_blockwise(xt, ct, bs)
    del xt
    am_h = to_host(am)
    q_o, am_o = O.quantize_8bit(xh, dtype, bs, code, rcp=device_rcp(am))
    assert np.array_equal(bits(am_h), bits(am_o))
    assert np.array_equal(to_host(q), q_o)
    out = dequantize_blockwise(q, am, ct, bs, {O.F32: torch.float32, O.F16: torch.float16,
                                                O.BF16: torch.bfloat16}[dtype])
    assert np.array_equal(bits(to_host(out)), bits(O.dequantize_8bit(q_o, am_o, code, bs, dtype)))


def _nested_on_host(w: bnb_b200.QuantizedArray) -> np.ndarray:
    """The oracle's own decode of a double-quantized weight's scales."""
    a = w.absmax
    return O.nested_absmax(to_host(a.data), to_host(a.absmax), to_host(a.code), float(to_host(a.offset).reshape(())),
                           a.blocksize)


@pytest.fixture(scope="module")
def config2_weight():
    g = torch.Generator("cuda").manual_seed(0)
    wt = (torch.randn(4096, 14336, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w = bnb_b200.quantize(wt, "nf4", 64, double_quant=True)
    return w, to_host(w.data), _nested_on_host(w)


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 20])
def test_config2_gemv_every_m_against_oracle(cuda, config2_weight, m):
    w, codes, scales = config2_weight
    g = torch.Generator("cuda").manual_seed(50 + m)
    x = torch.randn(m, 14336, device="cuda", generator=g).to(torch.bfloat16)
    y = bnb_b200.matmul(x, w)
    xh = to_host(x)
    y64, yabs = O.gemv_f64(xh, O.BF16, codes, 4096, 64, scales)
    yd = O.bf16_to_f32(to_host(y)).reshape(m, 4096).astype(np.float64)
    err = np.abs(yd - y64)
    assert np.all(err <= GEMV_RTOL * np.abs(y64) + GEMV_ATOL * yabs), float(err.max())
    if m == 1:  # the reference's own float32 chunked numerics, same tolerance
        yr = O.bf16_to_f32(O.gemv_ref(xh, O.BF16, codes, 4096, 64, scales)).reshape(1, 4096).astype(np.float64)
        assert np.all(np.abs(yd - yr) <= 2 * GEMV_RTOL * np.abs(y64) + 2 * GEMV_ATOL * yabs)


@pytest.mark.parametrize("shape", [(28672, 8192), (8192, 28672)], ids=["gate_up", "down"])
def test_config5_gemm_sampled_rows_against_oracle(cuda, shape, timeouts_at_start):
    n, k = shape
    g = torch.Generator("cuda").manual_seed(n)
    wt = (torch.randn(n, k, device="cuda", generator=g) * 0.015).to(torch.bfloat16)
    w = bnb_b200.quantize(wt, "nf4", 64, double_quant=True)
    del wt
    rows = np.arange(5, n, n // 48)
    scales = _nested_on_host(w)
    codes = to_host(w.data).reshape(n, k // 2)
    spr = k // 64
    w_rows = np.stack([O.bf16_to_f32(O.dequantize_nf4(codes[r], scales[r * spr:(r + 1) * spr], k, 64, O.BF16))
                       for r in rows]).astype(np.float64)
    for m in (64, 2048):
        x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        y = bnb_b200.matmul(x, w)
        xd = O.bf16_to_f32(to_host(x)).reshape(m, k).astype(np.float64)
        y64 = xd @ w_rows.T
        yabs = np.abs(xd) @ np.abs(w_rows).T
        yd = O.bf16_to_f32(to_host(y[:, torch.from_numpy(rows).to(cuda)].contiguous())).reshape(m, rows.size)
        err = np.abs(yd.astype(np.float64) - y64)
        assert np.all(err <= 2.0 ** -8 * np.abs(y64) + 2.0 ** -12 * yabs), (m, float(err.max()))
    assert _lib.wait_timeouts() == timeouts_at_start
