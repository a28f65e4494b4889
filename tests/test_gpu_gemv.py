"""Fused NF4 GEMV / matmul on the B200 (reference tests/test_matmul.py):
one-hot x returns the dequantized weights bitwise, the product matches the
float64 product within the stated tolerance and is closer to it than
dequantize-then-matmul, batch dims, the fallback routes, gradients, shards."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200.kernels import gemv_nf4
from bnb_b200.kernels.gemv import GEMV8_MAX_M, GEMV_MAX_M, GEMV_T_MAX_M
from helpers import GEMV_ATOL, GEMV_RTOL, TORCH_DTYPES, bits, to_host
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


def weight(n, k, blocksize=64, double_quant=True, qtype="nf4", seed=0):
    g = torch.Generator("cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    return bnb_b200.quantize(w, qtype, blocksize, double_quant=double_quant)


def x_rand(m, k, dtype, seed):
    g = torch.Generator("cuda").manual_seed(1000 + seed)
    return torch.randn(m, k, device="cuda", generator=g).to(dtype)


def f64_product(x: torch.Tensor, w) -> tuple[np.ndarray, np.ndarray]:
    """Oracle: x (as stored) times the float32 dequantized weight, in float64."""
    wd = w.dequantize(torch.float32).double()
    xd = x.double()
    return (xd @ wd.T).cpu().numpy(), (xd.abs() @ wd.abs().T).cpu().numpy()


@pytest.mark.parametrize("double_quant", [False, True])
@pytest.mark.parametrize("blocksize", [32, 64, 256])
def test_gemv_exact_weights(cuda, blocksize, double_quant):
    """One-hot x -> the dequantized weights, bitwise (reference test_matmul.py:18-27)."""
    w = weight(1000, 1056, blocksize, double_quant)
    dense = w.dequantize(torch.bfloat16)
    for m in [1, 3, GEMV_MAX_M]:
        x = torch.eye(1056, dtype=torch.bfloat16, device="cuda")[:m]
        y = bnb_b200.matmul(x, w)
        assert torch.equal(y, dense[:, :m].T)  # value equality, as assert_array_equal


@pytest.mark.parametrize("m", list(range(1, GEMV_MAX_M + 1)))
def test_gemv_every_m_exact_and_tolerance(cuda, m):
    w = weight(160, 512, 64, True, seed=m)
    x = torch.zeros(m, 512, dtype=torch.float16, device="cuda")
    cols = torch.arange(m, device="cuda") * 7 % 512
    x[torch.arange(m, device="cuda"), cols] = 1.0
    assert torch.equal(bnb_b200.matmul(x, w), w.dequantize(torch.float16)[:, cols].T)
    x = x_rand(m, 512, torch.bfloat16, m)
    y = bnb_b200.matmul(x, w).double().cpu().numpy()
    y64, yabs = f64_product(x, w)
    assert np.all(np.abs(y - y64) <= GEMV_RTOL * np.abs(y64) + GEMV_ATOL * yabs)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m", [1, 2, 3, 8, GEMV_MAX_M])
def test_gemv_accuracy(cuda, m, dtype):
    """Within tolerance of the float64 product and closer to it than
    dequantize-then-matmul (reference test_matmul.py:30-44)."""
    w = weight(1000, 4096)
    x = x_rand(m, 4096, dtype, m)
    exact, yabs = f64_product(x, w)
    fused = bnb_b200.matmul(x, w)
    unfused = x @ w.dequantize(dtype).T
    assert fused.dtype == dtype and fused.shape == (m, 1000)
    f = fused.double().cpu().numpy()
    err_fused = np.abs(f - exact).mean()
    err_unfused = np.abs(unfused.double().cpu().numpy() - exact).mean()
    assert err_fused < err_unfused, (err_fused, err_unfused)
    assert np.all(np.abs(f - exact) <= GEMV_RTOL * np.abs(exact) + GEMV_ATOL * yabs)


def test_gemv_config2_shape(cuda):
    """The benchmark's weight shape (4096 x 14336, double-quantized, bs 64)."""
    w = weight(4096, 14336, seed=3)
    for m in [1, GEMV_MAX_M]:
        x = x_rand(m, 14336, torch.bfloat16, 40 + m)
        y = bnb_b200.matmul(x, w).double().cpu().numpy()
        y64, yabs = f64_product(x, w)
        assert np.all(np.abs(y - y64) <= GEMV_RTOL * np.abs(y64) + GEMV_ATOL * yabs)


def test_gemv_against_oracle_numerics(cuda):
    """Independent of torch: the host oracle's float64 product from the raw
    codes and float32 scales."""
    n, k = 300, 2048
    w = weight(n, k, 64, double_quant=False, seed=9)
    x = x_rand(4, k, torch.bfloat16, 9)
    y = gemv_nf4(x, w.data, w.absmax, n, 64)
    xh = to_host(x)
    y64, yabs = O.gemv_f64(xh, O.BF16, to_host(w.data), n, 64, to_host(w.absmax))
    yd = O.bf16_to_f32(to_host(y)).reshape(4, n).astype(np.float64)
    assert np.all(np.abs(yd - y64) <= GEMV_RTOL * np.abs(y64) + GEMV_ATOL * yabs)


def test_matmul_batch_dims(cuda):
    w = weight(512, 1024)
    x = x_rand(6, 1024, torch.bfloat16, 1).reshape(2, 3, 1024)
    out = bnb_b200.matmul(x, w)
    assert out.shape == (2, 3, 512)
    assert torch.equal(out, bnb_b200.matmul(x.reshape(6, 1024), w).reshape(2, 3, 512))


@pytest.mark.parametrize("case", ["8bit", "float32_x"])
def test_matmul_fallback(cuda, case):
    """Where no fused kernel applies, x @ w.dequantize(x.dtype).T exactly
    (reference test_matmul.py:55-67). 8-bit weights take the fallback above
    GEMV8_MAX_M rows of x (below it, the fused 8-bit GEMV: test_gpu_gemv_8bit.py)."""
    m, dtype, qtype = 4, torch.bfloat16, "nf4"
    if case == "8bit":
        qtype = "8bit"
        m = GEMV8_MAX_M + 1
    else:
        dtype = torch.float32
    w = weight(256, 512, qtype=qtype)
    x = x_rand(m, 512, dtype, 2)
    assert torch.equal(bnb_b200.matmul(x, w), x @ w.dequantize(dtype).T)


def test_matmul_large_m(cuda):
    """Above GEMV_MAX_M: the fused GEMM (decoded to bf16, the fallback's
    precision) within tolerance of the fallback."""
    w = weight(256, 512)
    x = x_rand(GEMV_MAX_M + 1, 512, torch.bfloat16, 3)
    got = bnb_b200.matmul(x, w).double().cpu().numpy()
    ref = (x @ w.dequantize(torch.bfloat16).T).double().cpu().numpy()
    y64, yabs = f64_product(x, w)
    assert np.all(np.abs(got - ref) <= 2 * GEMV_RTOL * np.abs(ref) + 4 * GEMV_ATOL * yabs + 2.0 ** -7 * yabs / 512)


@pytest.mark.parametrize("m", [1, GEMV_MAX_M + 1])
def test_matmul_grad(cuda, m):
    """Gradient in x (reference test_matmul.py:70-79). More than GEMV_T_MAX_M
    rows of g: the reference's rule g @ w.dequantize(g.dtype), bitwise. Up to
    it: the fused backward (exact float32 weights), within the GEMV tolerance
    of the float64 product and closer to it than the rule."""
    w = weight(256, 512)
    x = x_rand(2 * m, 512, torch.bfloat16, 4).reshape(2, m, 512).requires_grad_(True)
    bnb_b200.matmul(x, w).float().sum().backward()
    g = x.grad.clone()
    x.grad = None
    (x @ w.dequantize(x.dtype).T).float().sum().backward()
    assert g.dtype == torch.bfloat16
    if 2 * m > GEMV_T_MAX_M:
        assert torch.equal(g, x.grad)
        return
    wd = w.dequantize(torch.float32).double()
    exact = torch.ones(2 * m, 256, dtype=torch.float64, device="cuda") @ wd
    bound = GEMV_RTOL * exact.abs() + GEMV_ATOL * wd.abs().sum(0, keepdim=True)
    got = g.reshape(2 * m, 512).double()
    assert torch.all((got - exact).abs() <= bound)
    assert (got - exact).abs().mean() <= (x.grad.reshape(2 * m, 512).double() - exact).abs().mean()


def test_matmul_saves_no_dense_weight(cuda):
    """Only the quantized weight is kept for the backward pass (reference
    test_matmul.py:82-89): no (N, K) dense tensor is saved."""
    w = weight(256, 512)
    x = x_rand(GEMV_MAX_M + 1, 512, torch.bfloat16, 5).requires_grad_(True)
    saved = []
    with torch.autograd.graph.saved_tensors_hooks(lambda t: saved.append(t) or t, lambda t: t):
        y = bnb_b200.matmul(x, w).float().sum()
    assert not any(t.shape == (256, 512) for t in saved), [t.shape for t in saved]
    y.backward()


@pytest.mark.parametrize("shards", [2, 4])
def test_gemv_row_shards_concatenate(cuda, shards):
    """Row shards (own slices of codes / nested codes, the whole absmax2 with
    the shard's first global block) reproduce the unsharded output bitwise."""
    n, k = 1024, 2048
    w = weight(n, k, 64, True, seed=11)
    x = x_rand(3, k, torch.bfloat16, 11)
    full = bnb_b200.matmul(x, w)
    a = w.absmax
    rows = n // shards
    parts = []
    for s in range(shards):
        r0 = s * rows
        b0 = r0 * k // 64
        parts.append(gemv_nf4(x, w.data[r0 * k // 2:(r0 + rows) * k // 2], a.data[b0:b0 + rows * k // 64],
                              rows, 64, nested=(a.absmax, a.code, a.offset, a.blocksize), absmax2_block0=b0))
    assert torch.equal(torch.cat(parts, dim=1), full)


def test_gemv_writes_into_wider_output(cuda):
    """ldy > n_rows: a shard writes its columns of a shared output buffer."""
    w = weight(256, 512, seed=12)
    x = x_rand(2, 512, torch.bfloat16, 12)
    big = torch.full((2, 1024), 7.0, dtype=torch.bfloat16, device="cuda")
    a = w.absmax
    gemv_nf4(x, w.data, a.data, 256, 64, nested=(a.absmax, a.code, a.offset, 256), out=big[:, 256:512])
    assert torch.equal(big[:, 256:512], bnb_b200.matmul(x, w))
    assert torch.all(big[:, :256] == 7.0) and torch.all(big[:, 512:] == 7.0)


def test_no_wait_timeouts(cuda, timeouts_at_start):
    """The pipelined kernels' bounded waits never expired during these tests."""
    from bnb_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == timeouts_at_start
