"""bnbq_matmul_nf4_allgather on one GPU: this rank's rows of an NF4 weight and
the exchange in one call, run as rank 0 of a group of two whose "rank 1" is
simulated. Rank 1's inbox is a local buffer, and its words for rank 1's
columns are written into rank 0's inbox beforehand, so nothing waits on
another GPU.

Checked for each route -- the streaming GEMV and the table GEMV with the
exchange in their epilogue (M = 1, 2), and the matmul followed by the
standalone exchange kernel (M = 3, 8) -- bitwise against matmul_rows (the
same kernels on the rank's rows): rank 0's columns of the output, the words
it sent to rank 1 (its values tagged with the call's epoch, in the epoch's
half), the columns it received, and the state (epoch advanced once per call,
counter reset). For M <= 2 the rank's rows also equal the whole weight's
product bitwise.
Then a peer that never sends: the fused kernel's bounded wait expires, is
counted, and the device stays usable."""
from __future__ import annotations

import pytest
import torch

import bnb_b200
from bnb_b200 import _lib
from bnb_b200.parallel import matmul_rows, row_partition, shard_rows

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


def _bits64(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int16).to(torch.int64) & 0xFFFF


class Rank0:
    def __init__(self, m, n_total, dev):
        self.inboxes = [torch.zeros(2 * m * n_total, dtype=torch.int64, device=dev) for _ in range(2)]
        self.ptrs = torch.tensor([b.data_ptr() for b in self.inboxes], dtype=torch.int64, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.y = torch.full((m, n_total), 5.0, dtype=torch.bfloat16, device=dev)

    def half(self, rank, epoch):
        m, n = self.y.shape
        return self.inboxes[rank].reshape(2, m, n)[epoch & 1]

    def call(self, x, sh):
        m, k = x.shape
        a = sh.nested
        nb = _lib.gemv_workspace_bytes(m, k, sh.n_rows) if m <= 20 else 0
        ws = torch.empty(max(nb, 16), dtype=torch.uint8, device=x.device)
        _lib.call("bnbq_matmul_nf4_allgather", _lib.BF16, x.data_ptr(), m, k, sh.data.data_ptr(), sh.n_rows,
                  sh.blocksize, None, sh.absmax.data_ptr(), a[0].data_ptr(), a[1].data_ptr(),
                  a[2].reshape(1).data_ptr(), a[3], sh.block0, self.y.data_ptr(), self.y.shape[1],
                  self.y.stride(0), sh.start, self.ptrs.data_ptr(), self.inboxes[0].numel(), self.state.data_ptr(),
                  2, 0, ws.data_ptr(), nb, _lib.stream_of(x))


def _weight(n, k, seed):
    g = torch.Generator("cuda").manual_seed(seed)
    return bnb_b200.quantize((torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16), "nf4", 64,
                             double_quant=True)


@pytest.mark.parametrize("shape", [(4096, 14336), (14336, 4096)], ids=["streaming", "table"])
def test_fused_exchange_rank0_of_two(cuda, shape):
    n, k = shape
    w = _weight(n, k, seed=n)
    (a0, b0), (a1, b1) = row_partition(n, k, 64 * 256, 2)
    sh = shard_rows(w, a0, b0)
    epoch = 0
    for m in (1, 2, 3, 8):
        r0 = Rank0(m, n, cuda)
        r0.state[1] = epoch  # carry the epoch on, as one group's calls would
        for rep in range(2):
            epoch += 1
            x = torch.randn(m, k, device=cuda).to(torch.bfloat16)
            mine = matmul_rows(x, sh)
            peer = torch.randn(m, b1 - a1, device=cuda).to(torch.bfloat16)
            r0.half(0, epoch)[:, a1:b1] = _bits64(peer) | (epoch << 32)  # rank 1's words
            r0.call(x, sh)
            torch.cuda.synchronize()
            assert torch.equal(r0.y[:, a0:b0], mine), (m, rep)
            assert torch.equal(r0.y[:, a1:b1], peer), (m, rep)
            if m <= 2:  # the row kernels: a row's result does not depend on how many rows run
                assert torch.equal(mine, bnb_b200.matmul(x, w)[:, a0:b0]), (m, rep)
            sent = r0.half(1, epoch)[:, a0:b0]
            assert bool((sent >> 32 == epoch).all()), (m, rep)
            assert torch.equal(sent & 0xFFFF, _bits64(mine)), (m, rep)
            assert r0.state.tolist() == [0, epoch], (m, rep)


def test_fused_exchange_wait_expires(cuda, timeouts_at_start):
    """Rank 1 never sends: the streaming GEMV's receive gives up after the
    (shortened) limit and counts it; rank 0's own columns are complete, the
    others untouched; a call of a group of one works right after."""
    n, k = 4096, 14336
    w = _weight(n, k, seed=3)
    (a0, b0), _ = row_partition(n, k, 64 * 256, 2)
    sh = shard_rows(w, a0, b0)
    x = torch.randn(1, k, device=cuda).to(torch.bfloat16)
    r0 = Rank0(1, n, cuda)
    _lib.set_wait_limit_ns(5_000_000)
    try:
        r0.call(x, sh)
        torch.cuda.synchronize()
    finally:
        _lib.set_wait_limit_ns(0)
    assert _lib.wait_timeouts() > timeouts_at_start
    full = bnb_b200.matmul(x, w)
    assert torch.equal(r0.y[:, a0:b0], full[:, a0:b0])
    assert bool((r0.y[:, b0:] == 5.0).all())
    assert r0.state.tolist() == [0, 1]
    # a group of one on the same device: no waits
    before = _lib.wait_timeouts()
    one = Rank0(1, n, cuda)
    y1 = torch.empty(1, n, dtype=torch.bfloat16, device=cuda)
    whole = shard_rows(w, 0, n)
    a = whole.nested
    _lib.call("bnbq_matmul_nf4_allgather", _lib.BF16, x.data_ptr(), 1, k, whole.data.data_ptr(), n, 64, None,
              whole.absmax.data_ptr(), a[0].data_ptr(), a[1].data_ptr(), a[2].reshape(1).data_ptr(), a[3], 0,
              y1.data_ptr(), n, n, 0, one.ptrs.data_ptr(), one.inboxes[0].numel(), one.state.data_ptr(), 1, 0,
              None, 0, _lib.stream_of(x))
    torch.cuda.synchronize()
    assert torch.equal(y1, full)
    assert _lib.wait_timeouts() == before
