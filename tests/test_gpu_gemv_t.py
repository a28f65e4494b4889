"""The fused backward of matmul for a few rows of g (bnbq_gemv_t_nf4_ws):
out = g @ W with W kept NF4. The reference computes g @ w.dequantize(g.dtype)
(_matmul.py:67-68); here a one-hot g returns the dequantized weight rows
bitwise, a random g is within the GEMV tolerance of the float64 product with
the weight as the CPU oracle decodes it and closer to it than the reference's
rule, and autograd uses it."""
from __future__ import annotations

import pytest
import torch

import bnb_b200
from bnb_b200 import _lib
from bnb_b200.kernels import GEMV_T_MAX_M, gemv_t_nf4
from helpers import GEMV_ATOL, GEMV_RTOL
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


def weight(n, k, blocksize=64, double_quant=True, seed=0):
    gen = torch.Generator("cuda").manual_seed(seed)
    w = (torch.randn(n, k, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    return bnb_b200.quantize(w, "nf4", blocksize, double_quant=double_quant)


def args(w):
    a = w.absmax
    if isinstance(a, bnb_b200.QuantizedArray):
        return a.data, (a.absmax, a.code, a.offset, a.blocksize)
    return a, None


def call(g, w):
    scales, nested = args(w)
    return gemv_t_nf4(g, w.data, scales, w.shape[0], w.shape[1], w.blocksize, nested=nested)


def oracle_weight(w) -> torch.Tensor:
    """The weight decoded to float32 by the CPU oracle from the raw codes and
    scales (the reference's arithmetic), as a float64 CUDA tensor."""
    a = w.absmax
    if isinstance(a, bnb_b200.QuantizedArray):
        absmax = O.nested_absmax(a.data.cpu().numpy(), a.absmax.cpu().numpy(), a.code.cpu().numpy(),
                                 float(a.offset.item()), a.blocksize)
    else:
        absmax = a.cpu().numpy()
    n, k = w.shape
    dense = O.dequantize_nf4(w.data.cpu().numpy(), absmax, n * k, w.blocksize, O.F32).reshape(n, k)
    return torch.from_numpy(dense).to("cuda").double()


def check_tolerance(g, w, out):
    wd = oracle_weight(w)
    gd = g.double()
    exact = gd @ wd
    bound = GEMV_RTOL * exact.abs() + GEMV_ATOL * (gd.abs() @ wd.abs())
    err = (out.double() - exact).abs()
    assert torch.all(err <= bound), float((err / bound).max())
    rule = (g @ w.dequantize(g.dtype)).double()
    assert err.mean() <= (rule - exact).abs().mean()


@pytest.mark.parametrize("double_quant", [False, True])
@pytest.mark.parametrize("blocksize", [32, 64, 256, 1024])
def test_one_hot_rows_are_the_weight(cuda, blocksize, double_quant):
    n, k = 1000, 1024  # rows not a multiple of anything
    w = weight(n, k, blocksize, double_quant, seed=blocksize)
    dense = w.dequantize(torch.bfloat16)
    eye = torch.eye(n, dtype=torch.bfloat16, device="cuda")
    for r0 in (0, 1, 333, 996):
        out = call(eye[r0:r0 + GEMV_T_MAX_M], w)
        assert torch.equal(out, dense[r0:r0 + GEMV_T_MAX_M])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("double_quant", [False, True])
def test_tolerance(cuda, m, dtype, double_quant):
    w = weight(777, 2048, 64, double_quant, seed=m)
    g = torch.randn(m, 777, device="cuda", generator=torch.Generator("cuda").manual_seed(m)).to(dtype)
    out = call(g, w)
    assert out.shape == (m, 2048) and out.dtype == dtype
    check_tolerance(g, w, out)


@pytest.mark.parametrize("shape", [(4096, 14336), (14336, 4096)])
def test_llama_shapes(cuda, shape):
    """Config 2's weight and its transpose (the backward of the forward GEMV)."""
    n, k = shape
    w = weight(n, k, 64, True, seed=9)
    for m in (1, 4):
        g = torch.randn(m, n, device="cuda", generator=torch.Generator("cuda").manual_seed(m)).to(torch.bfloat16)
        check_tolerance(g, w, call(g, w))


def test_strided_g_and_repeat(cuda):
    """g a column slice of a wider tensor; two calls in a row agree bitwise
    (deterministic order, a workspace with old contents)."""
    w = weight(512, 768, 64, True, seed=4)
    wide = torch.randn(3, 600, device="cuda", generator=torch.Generator("cuda").manual_seed(4)).to(torch.bfloat16)
    g = wide[:, 40:552]
    a = call(g, w)
    b = call(g.contiguous(), w)
    assert torch.equal(a, b)
    check_tolerance(g, w, a)


def test_autograd_uses_it(cuda):
    w = weight(512, 768, 64, True, seed=2)
    x = torch.randn(3, 768, device="cuda", generator=torch.Generator("cuda").manual_seed(2)).to(torch.bfloat16)
    x.requires_grad_(True)
    y = bnb_b200.matmul(x, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    assert torch.equal(x.grad, call(gy, w))


def test_autograd_gradient_small_weight(cuda):
    """A 256 x 512 weight: the gradient is either the reference's rule
    g @ w.dequantize(g.dtype), bitwise (where the fused kernel declines the
    call), or the fused kernel's, within the GEMV tolerance of the float64
    product with the oracle's weight."""
    w = weight(256, 512, 64, True, seed=2)
    x = torch.randn(3, 512, device="cuda", generator=torch.Generator("cuda").manual_seed(2)).to(torch.bfloat16)
    x.requires_grad_(True)
    y = bnb_b200.matmul(x, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    if torch.equal(x.grad, gy @ w.dequantize(gy.dtype)):
        return
    wd = oracle_weight(w)
    exact = gy.double() @ wd
    bound = GEMV_RTOL * exact.abs() + GEMV_ATOL * (gy.double().abs() @ wd.abs())
    assert torch.all((x.grad.double() - exact).abs() <= bound)


def test_errors(cuda):
    w = weight(64, 512, 64, False)
    with pytest.raises(ValueError):
        call(torch.zeros(GEMV_T_MAX_M + 1, 64, device="cuda", dtype=torch.bfloat16), w)
    w2 = weight(64, 320, 64, False)  # K % 256 != 0
    with pytest.raises(ValueError):
        call(torch.zeros(1, 64, device="cuda", dtype=torch.bfloat16), w2)
    with pytest.raises(NotImplementedError):
        call(torch.zeros(1, 64, device="cuda", dtype=torch.float32), w)
    assert _lib.wait_timeouts() >= 0
