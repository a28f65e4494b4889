"""Failure detection of the bounded device-side waits, on one GPU and without
a fault: the peer all-gather is run as rank 0 of a group of two whose "rank
1" is a pair of local buffers nobody ever publishes to. The waits for rank 1
must run out after the (shortened) limit, the kernel must return, the expiry
must be counted by bnbq_wait_timeouts, and the device must stay usable for a
normal exchange right after.

Nothing here reaches another GPU's memory or waits on another kernel: the
flags rank 0 waits on are local, zero, and written by no one."""
from __future__ import annotations

import time

import pytest
import torch

from bnb_b200 import _lib

pytestmark = pytest.mark.gpu


def _group(world, m, ldy, dev):
    """y_full / flags of `world` ranks, all local buffers of this device."""
    ys = [torch.full((m, ldy), 3.0, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    flags = [torch.zeros(2 * world, dtype=torch.int32, device=dev) for _ in range(world)]
    y_ptrs = torch.tensor([y.data_ptr() for y in ys], dtype=torch.int64, device=dev)
    f_ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=dev)
    return ys, flags, y_ptrs, f_ptrs


def _gather(y_local, col0, ldy, y_ptrs, f_ptrs, state, world, rank):
    _lib.call("bnbq_peer_allgather_rows", _lib.BF16, y_local.data_ptr(), y_local.shape[0], y_local.shape[1],
              y_local.stride(0), col0, ldy, y_ptrs.data_ptr(), f_ptrs.data_ptr(), state.data_ptr(), world, rank,
              _lib.stream_of(y_local))


def test_peer_wait_expires_and_is_counted(cuda):
    m, n_local, ldy = 2, 512, 1024
    y_local = torch.randn(m, n_local, device=cuda).to(torch.bfloat16)
    ys, flags, y_ptrs, f_ptrs = _group(2, m, ldy, cuda)
    state = torch.zeros(2, dtype=torch.int32, device=cuda)
    before = _lib.wait_timeouts()
    _lib.set_wait_limit_ns(5_000_000)  # 5 ms
    try:
        t0 = time.perf_counter()
        _gather(y_local, 0, ldy, y_ptrs, f_ptrs, state, 2, 0)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        _lib.set_wait_limit_ns(0)
    after = _lib.wait_timeouts()
    assert after > before, "the wait for the silent rank did not expire"
    assert elapsed < 5.0, f"the kernel took {elapsed:.2f} s to give up"
    # rank 0 published its own ready and done epochs (1) in both ranks' flags
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1  # done[0]
    assert flags[0][2].item() == 1 and flags[1][2].item() == 1  # ready[0]
    # its own slice still reached its own buffer; the silent rank's did not
    assert torch.equal(ys[0][:, :n_local], y_local)
    assert bool((ys[1] == 3.0).all()), "stored into a rank that never said ready"
    assert state[1].item() == 1 and state[0].item() == 0
    # the device is still usable: a normal exchange (a group of one) works
    ys1, _, y1, f1 = _group(1, m, ldy, cuda)
    state1 = torch.zeros(2, dtype=torch.int32, device=cuda)
    _gather(y_local, 100, ldy, y1, f1, state1, 1, 0)
    torch.cuda.synchronize()
    assert torch.equal(ys1[0][:, 100:100 + n_local], y_local)
    assert _lib.wait_timeouts() == after, "a normal exchange counted a timeout"


def test_wait_limit_restores_default(cuda):
    """After set_wait_limit_ns(0), a normal exchange takes no time-outs."""
    _lib.set_wait_limit_ns(0)
    y_local = torch.randn(4, 64, device=cuda).to(torch.bfloat16)
    ys, _, y_ptrs, f_ptrs = _group(1, 4, 64, cuda)
    state = torch.zeros(2, dtype=torch.int32, device=cuda)
    before = _lib.wait_timeouts()
    for _ in range(3):
        _gather(y_local, 0, 64, y_ptrs, f_ptrs, state, 1, 0)
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == before
    assert state[1].item() == 3
