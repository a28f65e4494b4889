"""Fused tcgen05 NF4 dequantize-GEMM (more than GEMV_MAX_M rows of x) on the B200.

A one-hot x returns the dequantized weights bitwise (the test of every layout:
codes, scales, tensor-memory operand, swizzled x tile, accumulator lanes). A
random x matches the float64 product of x and ``w.dequantize(x.dtype)`` -- the
operands of the reference's fallback (_matmul.py:58-59) -- within float32
accumulation error and one rounding. Tile edges in M, N and K, blocksizes 32..4096,
plain and double-quantized scales, row shards and a wider output buffer."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200.kernels.gemv import GEMV_MAX_M, matmul_nf4

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]

# |y - y64| <= REL[dtype] * |y64| + ACC * (|x| @ |w|): one rounding of the output
# plus float32 accumulation over K terms.
REL = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -10}
ACC = 2.0 ** -12


def weight(n, k, blocksize=64, double_quant=True, seed=0, std=1.0):
    g = torch.Generator("cuda").manual_seed(seed)
    w = (torch.randn(n, k, device="cuda", generator=g) * std).to(torch.bfloat16)
    return bnb_b200.quantize(w, "nf4", blocksize, double_quant=double_quant)


def x_rand(m, k, dtype, seed):
    g = torch.Generator("cuda").manual_seed(2000 + seed)
    return torch.randn(m, k, device="cuda", generator=g).to(dtype)


def one_hot(m, k, dtype):
    x = torch.zeros(m, k, dtype=dtype, device="cuda")
    cols = (torch.arange(m, device="cuda") * 37 + 5) % k
    x[torch.arange(m, device="cuda"), cols] = 1.0
    return x, cols


def check_close(y, x, w):
    wd = w.dequantize(x.dtype).double()
    y64 = x.double() @ wd.T
    yabs = x.double().abs() @ wd.abs().T
    err = (y.double() - y64).abs()
    bound = REL[x.dtype] * y64.abs() + ACC * yabs
    assert bool((err <= bound).all()), float((err - bound).max())
    return err


SHAPES = [  # (m, n, k): every BN (32, 64, 128, 256), partial tiles in M and N
    (GEMV_MAX_M + 1, 200, 512),
    (32, 128, 64),
    (33, 256, 1024),
    (64, 130, 512),
    (65, 384, 256),
    (128, 128, 2048),
    (129, 1000, 512),
    (256, 256, 512),
    (300, 520, 1024),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_one_hot_exact(cuda, m, n, k, dtype):
    w = weight(n, k, seed=m + n)
    x, cols = one_hot(m, k, dtype)
    y = bnb_b200.matmul(x, w)
    assert y.dtype == dtype and y.shape == (m, n)
    assert torch.equal(y, w.dequantize(dtype)[:, cols].T)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_random_within_tolerance(cuda, m, n, k, dtype):
    w = weight(n, k, seed=7 * m + n)
    x = x_rand(m, k, dtype, m + k)
    check_close(bnb_b200.matmul(x, w), x, w)


@pytest.mark.parametrize("double_quant", [False, True])
@pytest.mark.parametrize("blocksize", [32, 64, 128, 256, 4096])
def test_gemm_blocksizes(cuda, blocksize, double_quant):
    """blocksize 32 puts two scale blocks in a 64-wide stage."""
    n, k, m = 256, 4096, 96
    w = weight(n, k, blocksize, double_quant, seed=blocksize)
    x, cols = one_hot(m, k, torch.bfloat16)
    assert torch.equal(bnb_b200.matmul(x, w), w.dequantize(torch.bfloat16)[:, cols].T)
    x = x_rand(m, k, torch.bfloat16, blocksize)
    check_close(bnb_b200.matmul(x, w), x, w)


def test_gemm_error_like_fallback(cuda):
    """Against the exact product (float32 weights, float64 sums) the fused GEMM is
    as accurate as dequantize-then-matmul: both use x-dtype weights."""
    n, k, m = 512, 4096, 200
    w = weight(n, k, seed=31, std=0.02)
    x = x_rand(m, k, torch.bfloat16, 31)
    exact = x.double() @ w.dequantize(torch.float32).double().T
    fused = (bnb_b200.matmul(x, w).double() - exact).abs().mean().item()
    fallback = ((x @ w.dequantize(torch.bfloat16).T).double() - exact).abs().mean().item()
    assert fused <= 1.1 * fallback, (fused, fallback)


def test_gemm_k_not_multiple_of_64(cuda):
    """K % 64 != 0: the same call runs as GEMV passes of GEMV_MAX_M rows."""
    n, k, m = 300, 1056, 50
    w = weight(n, k, seed=5)
    x, cols = one_hot(m, k, torch.bfloat16)
    assert torch.equal(bnb_b200.matmul(x, w), w.dequantize(torch.bfloat16)[:, cols].T)
    x = x_rand(m, k, torch.bfloat16, 5)
    y = bnb_b200.matmul(x, w).double()
    y64 = x.double() @ w.dequantize(torch.float32).double().T
    yabs = x.double().abs() @ w.dequantize(torch.float32).double().abs().T
    assert bool(((y - y64).abs() <= 2.0 ** -8 * y64.abs() + 2.0 ** -18 * yabs).all())


@pytest.mark.parametrize("shards", [2, 4])
def test_gemm_row_shards_concatenate(cuda, shards):
    """Row shards (own slices of codes and nested codes, the whole absmax2 with the
    shard's first global block) reproduce the unsharded product bitwise."""
    n, k, m = 1024, 2048, 100
    w = weight(n, k, 64, True, seed=11)
    x = x_rand(m, k, torch.bfloat16, 11)
    full = bnb_b200.matmul(x, w)
    a = w.absmax
    rows = n // shards
    parts = []
    for s in range(shards):
        r0 = s * rows
        b0 = r0 * k // 64
        parts.append(matmul_nf4(x, w.data[r0 * k // 2:(r0 + rows) * k // 2], a.data[b0:b0 + rows * k // 64],
                                rows, 64, nested=(a.absmax, a.code, a.offset, a.blocksize), absmax2_block0=b0))
    assert torch.equal(torch.cat(parts, dim=1), full)


def test_gemm_writes_into_wider_output(cuda):
    n, k, m = 256, 512, 40
    w = weight(n, k, seed=12)
    x = x_rand(m, k, torch.bfloat16, 12)
    big = torch.full((m, 1024), 7.0, dtype=torch.bfloat16, device="cuda")
    a = w.absmax
    matmul_nf4(x, w.data, a.data, n, 64, nested=(a.absmax, a.code, a.offset, a.blocksize), out=big[:, 256:512])
    assert torch.equal(big[:, 256:512], bnb_b200.matmul(x, w))
    assert bool((big[:, :256] == 7.0).all()) and bool((big[:, 512:] == 7.0).all())


def test_gemm_llama70b_mlp_shape(cuda):
    """The prefill benchmark's gate/up shape (28672 x 8192, double-quantized,
    blocksize 64, N(0, 0.015^2)) at M = 512; a one-hot slice checks exactness."""
    n, k, m = 28672, 8192, 512
    w = weight(n, k, seed=70, std=0.015)
    x = x_rand(m, k, torch.bfloat16, 70)
    y = bnb_b200.matmul(x, w)
    rows = torch.arange(0, n, 97, device="cuda")
    wd = w.dequantize(torch.bfloat16)[rows].double()
    y64 = x.double() @ wd.T
    yabs = x.double().abs() @ wd.abs().T
    assert bool(((y[:, rows].double() - y64).abs() <= REL[torch.bfloat16] * y64.abs() + ACC * yabs).all())
    xo, cols = one_hot(m, k, torch.bfloat16)
    assert torch.equal(bnb_b200.matmul(xo, w), w.dequantize(torch.bfloat16)[:, cols].T)


def test_gemm_grad_matches_fallback(cuda):
    w = weight(256, 512)
    x = x_rand(2 * 64, 512, torch.bfloat16, 4).reshape(2, 64, 512).requires_grad_(True)
    bnb_b200.matmul(x, w).float().sum().backward()
    g = x.grad.clone()
    x.grad = None
    (x @ w.dequantize(x.dtype).T).float().sum().backward()
    assert torch.equal(g, x.grad)


def test_gemm_no_wait_timeouts(cuda, timeouts_at_start):
    """The GEMM's bounded waits never expired during these tests."""
    from bnb_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == timeouts_at_start


def test_large_m_routes_to_the_fallback(cuda):
    """Above FUSED_GEMM_MAX_M rows of x (the measured crossover), matmul is the
    reference's fallback: dequantize on the sm_100a kernels, then a dense
    matmul; up to it, the fused GEMM."""
    from bnb_b200._matmul import FUSED_GEMM_MAX_M
    n, k = 256, 1024
    w = weight(n, k, seed=7)
    x = x_rand(FUSED_GEMM_MAX_M + 1, k, torch.bfloat16, 7)
    assert torch.equal(bnb_b200.matmul(x, w), x @ w.dequantize(torch.bfloat16).T)
    xs = x[:FUSED_GEMM_MAX_M]
    a = w.absmax
    fused = matmul_nf4(xs, w.data, a.data, n, 64, nested=(a.absmax, a.code, a.offset, a.blocksize))
    assert torch.equal(bnb_b200.matmul(xs, w), fused)
