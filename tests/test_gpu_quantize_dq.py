"""NF4 quantization with double-quantized scales in one launch
(bnbq_quantize_nf4_dq): every output bitwise the three-call chain it
replaces -- bnbq_quantize_nf4, bnbq_absmax_mean, bnbq_quantize_blockwise with
the offset (the reference's quantize(..., double_quant=True), array.py:199-202)
-- which the other quantize tests pin to the oracle; and the offset equal to
the oracle's float64 mean."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from bnb_b200 import _lib
from bnb_b200.kernels import absmax_mean, create_dynamic_map, quantize_blockwise, quantize_nf4, quantize_nf4_dq
from helpers import DTYPE_IDS, TORCH_DTYPES, bits, host_input, randn, to_device, to_host
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


def chain(x: torch.Tensor, bs: int, bs2: int):
    """The three separate launches."""
    q, absmax = quantize_nf4(x, bs)
    offset = absmax_mean(absmax)
    q2, absmax2 = quantize_blockwise(absmax, create_dynamic_map(device=x.device), bs2, offset=offset)
    return q, absmax, q2, absmax2, offset


def assert_same(got, want):
    for g, w in zip(got, want):
        assert g.shape == w.shape and g.dtype == w.dtype
        assert np.array_equal(bits(to_host(g).reshape(-1)), bits(to_host(w).reshape(-1)))


@pytest.mark.parametrize("dtype", [O.F32, O.F16, O.BF16], ids=DTYPE_IDS.get)
@pytest.mark.parametrize("bs", [8, 32, 64, 256, 512, 4096])
def test_single_pass_equals_chain(cuda, dtype, bs):
    for n in (bs, 3 * bs + 5, (1 << 18) + 37):
        x = to_device(host_input(randn(n, seed=n + bs, scale=0.02), dtype), dtype)
        assert_same(quantize_nf4_dq(x, bs), chain(x, bs, 256))


@pytest.mark.parametrize("bs2", [64, 128, 256])
def test_single_pass_nested_blocksizes(cuda, bs2):
    """More than 8192 blocks (every mean slot used more than once)."""
    n = (1 << 20) + 13
    x = to_device(host_input(randn(n, seed=5, scale=0.02), O.BF16), O.BF16)
    got = quantize_nf4_dq(x, 64, blocksize2=bs2)
    assert_same(got, chain(x, 64, bs2))
    assert to_host(got[4]).reshape(()) == O.mean_f32(to_host(got[1]))


@pytest.mark.parametrize("shape", [(4096, 4096), (4096, 14336)], ids=["config1", "config2"])
def test_single_pass_benchmark_shapes(cuda, shape):
    """Configs 1 and 2: W ~ N(0, 0.02^2) bf16, seed 0, NF4 bs 64, nested bs 256."""
    g = torch.Generator("cuda").manual_seed(0)
    w = (torch.randn(*shape, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    got = quantize_nf4_dq(w, 64)
    assert_same(got, chain(w.reshape(-1), 64, 256))
    assert to_host(got[4]).reshape(()) == O.mean_f32(to_host(got[1]))


def test_single_pass_through_quantize(cuda):
    """bnb_b200.quantize(..., double_quant=True) takes the single pass; its
    dequantized values equal those of the chain's arrays."""
    import bnb_b200
    x = torch.randn(1000, 256, device="cuda", generator=torch.Generator("cuda").manual_seed(3)).to(torch.float16)
    qa = bnb_b200.quantize(x, "nf4", 64, double_quant=True)
    q, absmax, q2, absmax2, offset = chain(x.reshape(-1), 64, 256)
    assert torch.equal(qa.data, q)
    assert torch.equal(qa.absmax.data, q2) and torch.equal(qa.absmax.absmax, absmax2)
    assert torch.equal(qa.absmax.offset, offset)
    assert qa.dequantize(torch.float16).shape == (1000, 256)


def test_single_pass_errors(cuda):
    x = torch.zeros(0, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        quantize_nf4_dq(x, 64)
    y = torch.ones(1024, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        quantize_nf4_dq(y, 64, blocksize2=512)  # nested blocks above 256
    assert TORCH_DTYPES[O.BF16] is torch.bfloat16
    assert _lib.wait_timeouts() >= 0
