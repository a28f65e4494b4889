"""Fused GEMV for 8-bit blockwise-quantized weights (bnbq_gemv_blockwise_ws).

The reference has no fused kernel for 8-bit weights: its router sends them
to x @ w.dequantize().T (_matmul.py:74-79, tested by the reference's
tests/test_matmul.py:55-67). The fused kernel must therefore agree with the
oracle's 8-bit decode (oracle/bnbq_oracle.c, the reference's arithmetic):
a one-hot x returns the decoded weights bitwise, a random x is within the
GEMV tolerance of the float64 product of x and the oracle-decoded weights,
and closer to it than dequantize-then-matmul."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200 import _lib
from bnb_b200.kernels import GEMV8_MAX_M, gemv_blockwise
from helpers import GEMV_ATOL, GEMV_RTOL, bits, to_host
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


def weight8(n, k, blocksize, double_quant, seed=0, scale=0.02):
    g = torch.Generator("cuda").manual_seed(seed)
    w = (torch.randn(n, k, device="cuda", generator=g) * scale).to(torch.bfloat16)
    return bnb_b200.quantize(w, "8bit", blocksize, double_quant=double_quant)


def oracle_weight(w) -> np.ndarray:
    """The weight decoded to float32 by the oracle, from the raw codes and scales."""
    q = w.data.cpu().numpy()
    code = w.code.cpu().numpy()
    if isinstance(w.absmax, bnb_b200.QuantizedArray):
        a = w.absmax
        absmax = O.nested_absmax(a.data.cpu().numpy(), a.absmax.cpu().numpy(), a.code.cpu().numpy(),
                                 float(a.offset.item()), a.blocksize)
    else:
        absmax = w.absmax.cpu().numpy()
    return O.dequantize_8bit(q, absmax, code, w.blocksize, O.F32).reshape(w.shape)


def x_rand(m, k, dtype, seed):
    g = torch.Generator("cuda").manual_seed(2000 + seed)
    return torch.randn(m, k, device="cuda", generator=g).to(dtype)


@pytest.mark.parametrize("double_quant", [False, True])
@pytest.mark.parametrize("blocksize", [64, 128, 256, 1024])
def test_gemv8_one_hot_is_the_oracle_decode(cuda, blocksize, double_quant):
    """One-hot rows of x return the decoded weight columns bitwise."""
    n, k = 544, 1024
    w = weight8(n, k, blocksize, double_quant, seed=blocksize)
    dense = O.f32_to_bf16(oracle_weight(w))  # the oracle's decode, rounded once to bf16
    eye = torch.eye(k, dtype=torch.bfloat16, device="cuda")
    for i0 in range(0, k, 4 * 37):
        m = min(GEMV8_MAX_M, k - i0)
        y = to_host(bnb_b200.matmul(eye[i0:i0 + m], w))
        assert np.array_equal(bits(y), bits(np.ascontiguousarray(dense[:, i0:i0 + m].T))), i0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("double_quant", [False, True])
def test_gemv8_accuracy_against_oracle(cuda, m, dtype, double_quant):
    """Within the GEMV tolerance of the float64 product with the oracle-decoded
    weight, and closer to it than dequantize-then-matmul (the reference's path)."""
    n, k = 1000, 4096  # rows not a multiple of the 32-row unit
    w = weight8(n, k, 64, double_quant, seed=m)
    x = x_rand(m, k, dtype, m)
    wd = oracle_weight(w).astype(np.float64)
    xd = x.double().cpu().numpy()
    exact, yabs = xd @ wd.T, np.abs(xd) @ np.abs(wd).T
    fused = bnb_b200.matmul(x, w)
    assert fused.dtype == dtype and fused.shape == (m, n)
    f = fused.double().cpu().numpy()
    assert np.all(np.abs(f - exact) <= GEMV_RTOL * np.abs(exact) + GEMV_ATOL * yabs)
    unfused = (x @ w.dequantize(dtype).T).double().cpu().numpy()
    assert np.abs(f - exact).mean() < np.abs(unfused - exact).mean()


@pytest.mark.parametrize("shape", [(4096, 14336), (14336, 4096)])
def test_gemv8_llama_shapes(cuda, shape):
    """The config-2 shape and its transpose, double-quantized, M = 1 and 4."""
    n, k = shape
    w = weight8(n, k, 64, True, seed=7)
    wd = oracle_weight(w).astype(np.float64)
    for m in (1, 4):
        x = x_rand(m, k, torch.bfloat16, 10 + m)
        xd = x.double().cpu().numpy()
        exact, yabs = xd @ wd.T, np.abs(xd) @ np.abs(wd).T
        f = bnb_b200.matmul(x, w).double().cpu().numpy()
        assert np.all(np.abs(f - exact) <= GEMV_RTOL * np.abs(exact) + GEMV_ATOL * yabs)


def test_gemv8_user_codebook_and_strided_output(cuda):
    """A non-default codebook, and y written into columns of a wider buffer."""
    n, k = 256, 512
    g = torch.Generator("cuda").manual_seed(3)
    code = torch.sort(torch.rand(256, device="cuda", generator=g) * 2 - 1).values
    code[0], code[-1] = -1.0, 1.0
    wf = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    w = bnb_b200.quantize(wf, "8bit", 128, code=code)
    x = x_rand(2, k, torch.float16, 3)
    wide = torch.full((2, n + 64), 7.0, dtype=torch.float16, device="cuda")
    out = wide[:, 16:16 + n]
    gemv_blockwise(x, w.data, w.absmax, w.code, n, 128, out=out)
    ref = bnb_b200.matmul(x, w)
    assert torch.equal(out, ref)
    assert torch.all(wide[:, :16] == 7.0) and torch.all(wide[:, 16 + n:] == 7.0)  # nothing written outside


def test_gemv8_routes_and_errors(cuda):
    """More rows than the fused kernel takes, or K % 128 != 0, go to the
    reference's fallback; the kernel entry itself rejects them."""
    w = weight8(64, 512, 64, False)
    x = x_rand(GEMV8_MAX_M + 1, 512, torch.bfloat16, 1)
    assert torch.equal(bnb_b200.matmul(x, w), x @ w.dequantize(torch.bfloat16).T)
    with pytest.raises(ValueError):
        gemv_blockwise(x, w.data, w.absmax, w.code, 64, 64)
    w96 = weight8(64, 96 * 4, 32, False)  # K = 384: a multiple of 128
    assert bnb_b200.matmul(x[:1, :384], w96).shape == (1, 64)
    w_odd = weight8(64, 320, 64, False)  # K = 320: not a multiple of 128
    xo = x_rand(1, 320, torch.bfloat16, 2)
    assert torch.equal(bnb_b200.matmul(xo, w_odd), xo @ w_odd.dequantize(torch.bfloat16).T)
    with pytest.raises(ValueError):
        gemv_blockwise(xo, w_odd.data, w_odd.absmax, w_odd.code, 64, 64)
    assert _lib.wait_timeouts() >= 0


def test_gemv8_in_cuda_graph(cuda):
    """Captured and replayed: the same bits as eager calls."""
    w = weight8(512, 1024, 64, True, seed=5)
    x = x_rand(2, 1024, torch.bfloat16, 5)
    ref = bnb_b200.matmul(x, w)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        bnb_b200.matmul(x, w)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            y = bnb_b200.matmul(x, w)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
