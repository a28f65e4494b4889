"""Test helpers: seeded inputs and torch <-> numpy (bf16 as uint16 bits)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O

TORCH_DTYPES = {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}
DTYPE_IDS = {O.F32: "f32", O.F16: "f16", O.BF16: "bf16"}


def host_input(values_f32: np.ndarray, dtype: int) -> np.ndarray:
    """float32 values rounded to `dtype` (bf16 as uint16 bits, RNE)."""
    v = np.ascontiguousarray(values_f32, np.float32)
    if dtype == O.F32:
        return v
    if dtype == O.F16:
        return v.astype(np.float16)
    return O.f32_to_bf16(v)


def to_device(a: np.ndarray, dtype: int | None = None, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if dtype == O.BF16:
        return torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(a).to(device)


def to_host(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def bits(a: np.ndarray) -> np.ndarray:
    """Raw bit patterns (for bit-exact comparisons that see -0.0 and NaN payloads)."""
    a = np.ascontiguousarray(a)
    return a.view({1: np.uint8, 2: np.uint16, 4: np.uint32}[a.dtype.itemsize])


def randn(n: int, seed: int, scale: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


def mixed_outliers(n: int, seed: int) -> np.ndarray:
    """90% N(0, 1) and 10% Laplace(0, 8) at random positions (8-bit config)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    idx = rng.random(n) < 0.1
    x[idx] = rng.laplace(0.0, 8.0, int(idx.sum())).astype(np.float32)
    return x

# GEMV/GEMM tolerance against the float64 product of x and the float32
# dequantized weight, elementwise:
#   |y - y64| <= GEMV_RTOL * |y64| + GEMV_ATOL * sum_k |x_k * w_k|
# RTOL covers the final rounding to bf16 (half an ulp of an 8-bit significand);
# ATOL covers float32 accumulation over up to 28,672 products.
GEMV_RTOL = 2.0 ** -8
GEMV_ATOL = 2.0 ** -18
