"""The shared-memory pair-table GEMV (bnbq_gemv_nf4_ws, 1 <= M <= 4, K a
multiple of 256) on the B200: one-hot x returns the dequantized weights
bitwise at every blocksize, plain and double-quantized scales, both x dtypes;
random x matches the oracle's float64 product within the stated tolerance and
the workspace-free kernels' results within it too; results are deterministic
(bitwise equal across calls) and do not depend on the workspace's earlier
contents, eagerly and from a CUDA graph; partial row blocks, row shards of a
double-quantized weight and a wider output buffer."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import bnb_b200
from bnb_b200 import _lib
from helpers import GEMV_ATOL, GEMV_RTOL, to_host
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start", "table_policy")]


@pytest.fixture(scope="module")
def table_policy(cuda):
    """This module tests the table GEMV at every shape it applies to."""
    _lib.set_gemv_policy(_lib.POLICY_TABLE)
    yield
    _lib.set_gemv_policy(_lib.POLICY_AUTO)


def weight(n, k, blocksize=64, double_quant=True, seed=0, std=0.02):
    g = torch.Generator("cuda").manual_seed(seed)
    w = (torch.randn(n, k, device="cuda", generator=g) * std).to(torch.bfloat16)
    return bnb_b200.quantize(w, "nf4", blocksize, double_quant=double_quant)


def scales_args(w):
    a = w.absmax
    if isinstance(a, bnb_b200.QuantizedArray):
        return None, a.data, a.absmax, a.code, a.offset.reshape(1), a.blocksize
    return a, None, None, None, None, 0


def call(entry, x, w, n, ws=None, out=None, block0=0, data=None, scales=None):
    """One call through the C ABI (the table GEMV with a workspace, or the
    workspace-free entry point)."""
    m, k = x.shape
    if out is None:
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
    absmax, aq, a2, c2, off, bs2 = scales if scales is not None else scales_args(w)
    data = w.data if data is None else data
    args = [_lib.DTYPE_CODE[x.dtype], x.data_ptr(), m, k, data.data_ptr(), n, w.blocksize, _lib.ptr(absmax),
            _lib.ptr(aq), _lib.ptr(a2), _lib.ptr(c2), _lib.ptr(off), bs2, block0, out.data_ptr(), out.stride(0)]
    if entry == "bnbq_gemv_nf4_ws":
        args += [_lib.ptr(ws), 0 if ws is None else ws.numel()]
    args.append(_lib.stream_of(x))
    _lib.call(entry, *args)
    return out


def new_ws(m, k, n):
    """A workspace full of garbage (the kernels need no initial contents)."""
    nb = _lib.gemv_workspace_bytes(m, k, n)
    assert nb > 0
    return torch.full((nb,), 0xA5, dtype=torch.uint8, device="cuda")


@pytest.mark.parametrize("double_quant", [False, True])
@pytest.mark.parametrize("blocksize", [32, 64, 128, 256, 1024, 4096])
def test_table_gemv_one_hot_bitwise(cuda, blocksize, double_quant):
    n, k = 200, 4096
    w = weight(n, k, blocksize, double_quant, seed=blocksize)
    for dtype in (torch.bfloat16, torch.float16):
        dense = w.dequantize(dtype)
        for m in (1, 2, 3, 4):
            cols = (torch.arange(m, device="cuda") * 997 + 13) % k
            x = torch.zeros(m, k, dtype=dtype, device="cuda")
            x[torch.arange(m, device="cuda"), cols] = 1.0
            ws = new_ws(m, k, n)
            y = call("bnbq_gemv_nf4_ws", x, w, n, ws)
            torch.cuda.synchronize()
            assert torch.equal(y, dense[:, cols].T), (dtype, m)


@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("shape", [(4096, 14336), (1000, 4096), (33, 256)])
def test_table_gemv_tolerance_against_oracle(cuda, shape, m):
    n, k = shape
    w = weight(n, k, 64, True, seed=n + m, std=1.0)
    g = torch.Generator("cuda").manual_seed(m)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    ws = new_ws(m, k, n)
    y = call("bnbq_gemv_nf4_ws", x, w, n, ws)
    a = w.absmax
    scales = O.nested_absmax(to_host(a.data), to_host(a.absmax), to_host(a.code),
                             float(to_host(a.offset).reshape(())), a.blocksize)
    y64, yabs = O.gemv_f64(to_host(x), O.BF16, to_host(w.data), n, 64, scales)
    yd = O.bf16_to_f32(to_host(y)).reshape(m, n).astype(np.float64)
    err = np.abs(yd - y64)
    assert np.all(err <= GEMV_RTOL * np.abs(y64) + GEMV_ATOL * yabs), float(err.max())
    # the workspace-free kernels agree within the same tolerance
    y_old = O.bf16_to_f32(to_host(call("bnbq_gemv_nf4", x, w, n))).reshape(m, n).astype(np.float64)
    assert np.all(np.abs(yd - y_old) <= 2 * GEMV_RTOL * np.abs(y64) + 2 * GEMV_ATOL * yabs)


def test_table_gemv_takes_the_benchmark_shapes(cuda):
    """The table GEMV (not a fallback) runs for the benchmark's shapes, plain and
    double-quantized, M = 1..4."""
    for n, k in [(4096, 14336), (1024, 4096), (14336, 4096), (28672, 8192), (8192, 28672)]:
        for m in (1, 2, 3, 4):
            ws = new_ws(m, k, n)
            for dq in (True, False):
                aq = ws if dq else None  # only the pointer's alignment matters here
                route = _lib.gemv_route(m, k, n, 64, _lib.ptr(aq), 256, ws.data_ptr(), ws.numel())
                assert route == _lib.ROUTE_TABLE_GEMV, (n, k, m, dq, route)
    assert _lib.gemv_route(5, 14336, 4096, 64, None, 0, None, 0) == _lib.ROUTE_GEMV
    assert _lib.gemv_route(21, 14336, 4096, 64, None, 0, None, 0) == _lib.ROUTE_GEMM
    # the automatic policy: wide weights take the table GEMV, long rows the streaming kernels
    _lib.set_gemv_policy(_lib.POLICY_AUTO)
    try:
        ws = new_ws(1, 4096, 14336)
        assert _lib.gemv_route(1, 4096, 14336, 64, None, 256, ws.data_ptr(), ws.numel()) == _lib.ROUTE_TABLE_GEMV
        ws = new_ws(1, 14336, 4096)
        assert _lib.gemv_route(1, 14336, 4096, 64, None, 256, ws.data_ptr(), ws.numel()) == _lib.ROUTE_GEMV
    finally:
        _lib.set_gemv_policy(_lib.POLICY_TABLE)


def test_table_gemv_deterministic_and_reusable(cuda):
    """Bitwise equal results over repeated calls on one workspace (the fixed
    summation order)."""
    n, k = 4096, 14336
    w = weight(n, k, seed=5)
    x = torch.randn(1, k, device="cuda").to(torch.bfloat16)
    ws = new_ws(1, k, n)
    first = call("bnbq_gemv_nf4_ws", x, w, n, ws).clone()
    for _ in range(5):
        assert torch.equal(call("bnbq_gemv_nf4_ws", x, w, n, ws), first)


def test_table_gemv_in_cuda_graph(cuda):
    n, k = 1024, 4096
    ws_list = [weight(n, k, seed=s) for s in range(3)]
    x = torch.randn(2, k, device="cuda").to(torch.bfloat16)
    ws = new_ws(2, k, n)
    outs = [torch.empty(2, n, dtype=torch.bfloat16, device="cuda") for _ in ws_list]
    want = [bnb_b200.matmul(x, w) for w in ws_list]
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for w, o in zip(ws_list, outs):
                call("bnbq_gemv_nf4_ws", x, w, n, ws, out=o)
    for _ in range(3):
        for o in outs:
            o.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for o, ref in zip(outs, want):
            assert torch.equal(o, ref)
    del graph


def test_table_gemv_row_shard_and_wide_output(cuda):
    """Rows [1024, 3072) of a double-quantized weight with the whole absmax2
    and the shard's first global block; written into columns of a wider y."""
    n, k = 4096, 4096
    w = weight(n, k, seed=8)
    a = w.absmax
    r0, r1 = 1024, 3072
    bpr = k // 64
    data = w.data.reshape(-1)[r0 * k // 2:r1 * k // 2]
    scales = (None, a.data.reshape(-1)[r0 * bpr:r1 * bpr], a.absmax, a.code, a.offset.reshape(1), a.blocksize)
    x = torch.randn(3, k, device="cuda").to(torch.bfloat16)
    big = torch.full((3, 5000), 7.0, dtype=torch.bfloat16, device="cuda")
    ws = new_ws(3, k, r1 - r0)
    call("bnbq_gemv_nf4_ws", x, w, r1 - r0, ws, out=big[:, 100:100 + (r1 - r0)], block0=r0 * bpr, data=data,
         scales=scales)
    full = bnb_b200.matmul(x, w)
    torch.cuda.synchronize()
    assert torch.equal(big[:, 100:100 + (r1 - r0)], full[:, r0:r1])
    assert bool((big[:, :100] == 7.0).all()) and bool((big[:, 100 + (r1 - r0):] == 7.0).all())


def test_table_gemv_one_workspace_many_shapes(cuda):
    """One workspace shared by calls of different shapes, in turn."""
    shapes = [(160, 512), (4096, 14336), (1000, 4096), (14336, 4096), (33, 256)]
    nbytes = max(_lib.gemv_workspace_bytes(m, k, n) for n, k in shapes for m in (1, 2, 4))
    ws = torch.full((nbytes,), 0x5A, dtype=torch.uint8, device="cuda")
    for rep in range(2):
        for i, (n, k) in enumerate(shapes):
            w = weight(n, k, seed=30 + i)
            for m in (1, 2, 4):
                x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
                got = call("bnbq_gemv_nf4_ws", x, w, n, ws)
                fresh = call("bnbq_gemv_nf4_ws", x, w, n, new_ws(m, k, n))
                torch.cuda.synchronize()
                assert torch.equal(got, fresh), (rep, n, k, m)


def test_table_gemv_workspace_size_and_fallback(cuda):
    """The size query; a too-small workspace or K not a multiple of 256 runs
    the other kernels, with the same result."""
    assert _lib.gemv_workspace_bytes(1, 14336, 4096) >= 56 * 4096 * 4
    assert _lib.gemv_workspace_bytes(21, 14336, 4096) == 0
    n, k = 300, 2048
    w = weight(n, k, seed=2)
    x = torch.randn(1, k, device="cuda").to(torch.bfloat16)
    tiny = torch.zeros(256, dtype=torch.uint8, device="cuda")
    assert torch.equal(call("bnbq_gemv_nf4_ws", x, w, n, tiny), call("bnbq_gemv_nf4", x, w, n))
    n2, k2 = 128, 1056  # K % 256 != 0
    w2 = weight(n2, k2, seed=3)
    x2 = torch.randn(2, k2, device="cuda").to(torch.bfloat16)
    ws2 = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    assert torch.equal(call("bnbq_gemv_nf4_ws", x2, w2, n2, ws2), call("bnbq_gemv_nf4", x2, w2, n2))


def test_table_gemv_no_wait_timeouts(cuda, timeouts_at_start):
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == timeouts_at_start
