"""Failure detection of the bounded device-side waits, on one GPU and without
a fault: the peer all-gather is run as rank 0 of a group of two whose "rank
1" is a local inbox nobody ever sends to. The waits for rank 1's columns must
run out after the (shortened) limit, the kernel must return, the expiry must
be counted by bnbq_wait_timeouts, and the device must stay usable for a
normal exchange right after.

Nothing here reaches another GPU's memory or waits on another kernel: the
inbox words rank 0 polls are local, zero, and written by no one."""
from __future__ import annotations

import time

import pytest
import torch

from bnb_b200 import _lib

pytestmark = pytest.mark.gpu


class Group:
    """The inboxes of `world` ranks, all local buffers of this device, and
    rank 0's output and state."""

    def __init__(self, world, m, n_total, dev):
        self.inboxes = [torch.zeros(2 * m * n_total, dtype=torch.int64, device=dev) for _ in range(world)]
        self.ptrs = torch.tensor([b.data_ptr() for b in self.inboxes], dtype=torch.int64, device=dev)
        self.y = torch.full((m, n_total), 3.0, dtype=torch.bfloat16, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.world = world

    def gather(self, y_local, col0, rank=0):
        _lib.call("bnbq_peer_allgather_rows", _lib.BF16, y_local.data_ptr(), y_local.shape[0], y_local.shape[1],
                  y_local.stride(0), col0, self.y.data_ptr(), self.y.shape[1], self.y.stride(0),
                  self.ptrs.data_ptr(), self.inboxes[0].numel(), self.state.data_ptr(), self.world, rank,
                  _lib.stream_of(y_local))


def test_peer_wait_expires_and_is_counted(cuda):
    m, n_local, n_total = 2, 512, 1024
    y_local = torch.randn(m, n_local, device=cuda).to(torch.bfloat16)
    grp = Group(2, m, n_total, cuda)
    before = _lib.wait_timeouts()
    _lib.set_wait_limit_ns(5_000_000)  # 5 ms
    try:
        t0 = time.perf_counter()
        grp.gather(y_local, 0)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        _lib.set_wait_limit_ns(0)
    after = _lib.wait_timeouts()
    assert after > before, "the wait for the silent rank did not expire"
    assert elapsed < 5.0, f"the kernel took {elapsed:.2f} s to give up"
    # rank 0's own slice reached its output; the silent rank's columns were left alone
    assert torch.equal(grp.y[:, :n_local], y_local)
    assert bool((grp.y[:, n_local:] == 3.0).all()), "wrote columns that never arrived"
    # rank 0 sent its slice to rank 1 as {value, epoch 1} words in the odd half
    words = grp.inboxes[1].reshape(2, m, n_total)[1, :, :n_local]
    assert bool((words >> 32 == 1).all())
    low = words & 0xFFFF
    assert torch.equal((low - ((low & 0x8000) << 1)).to(torch.int16).view(torch.bfloat16), y_local)
    assert bool((grp.inboxes[1].reshape(2, m, n_total)[:, :, n_local:] == 0).all())
    assert grp.state.tolist() == [0, 1]
    # the device is still usable: a normal exchange (a group of one) works
    one = Group(1, m, n_local, cuda)
    one.gather(y_local, 0)
    torch.cuda.synchronize()
    assert torch.equal(one.y, y_local)
    assert _lib.wait_timeouts() == after, "a normal exchange counted a timeout"


def test_wait_limit_restores_default(cuda):
    """After set_wait_limit_ns(0), exchanges whose peer words are already
    there take no time-outs: rank 0 of two, with rank 1's words for epochs 1
    to 3 written into rank 0's inbox beforehand."""
    _lib.set_wait_limit_ns(0)
    m, n_total = 4, 64
    grp = Group(2, m, n_total, cuda)
    y_local = torch.randn(m, 32, device=cuda).to(torch.bfloat16)
    peer = torch.randn(3, m, 32, device=cuda).to(torch.bfloat16)
    before = _lib.wait_timeouts()
    halves = grp.inboxes[0].reshape(2, m, n_total)
    for call in range(3):
        epoch = call + 1
        bits = peer[call].view(torch.int16).to(torch.int64) & 0xFFFF
        halves[epoch & 1, :, 32:] = bits | (epoch << 32)
        grp.gather(y_local, 0)
        torch.cuda.synchronize()
        assert torch.equal(grp.y[:, :32], y_local)
        assert torch.equal(grp.y[:, 32:], peer[call]), f"call {call}"
    assert _lib.wait_timeouts() == before
    assert grp.state.tolist() == [0, 3]
