"""bnbq_peer_allgather_rows_noalloc: the row-shard all-gather for callers that
may not allocate device memory (a custom-call handler inside a compiled
program whose runtime owns the device memory, or a serving loop held to a
fixed memory plan). It keeps the exchange's state words, which must outlive
every call, in a fixed per-device array inside the library instead of a
buffer the caller allocates.

Checked through the C ABI against bnbq_peer_allgather_rows (the entry point
that takes caller-allocated state) on two calls in a row: the second call
starts from what the first left in the shared array. The copy is exact, so
the tolerance is zero. This file is collected last on purpose."""
from __future__ import annotations

import pytest
import torch

from bnb_b200 import _lib
from dist_helpers import _free_port

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("timeouts_at_start")]


class Exchange:
    """The buffers a group of `world` ranks passes to either entry point, all
    on this device, from rank 0's side: the ranks' zeroed inboxes and a device
    array of their addresses, rank 0's output -- columns [out_col, out_col +
    n_total) of an m x ldy buffer filled with 7 -- and its `state` (used only
    by bnbq_peer_allgather_rows)."""

    def __init__(self, m, n_total, dtype, dev, world=1, ldy=None, out_col=0):
        self.world = world
        self.buf = torch.full((m, ldy or n_total), 7.0, dtype=dtype, device=dev)
        self.y_full = self.buf[:, out_col:out_col + n_total]
        self.inboxes = [torch.zeros(2 * m * n_total, dtype=torch.int64, device=dev) for _ in range(world)]
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.ptrs = torch.tensor([b.data_ptr() for b in self.inboxes], dtype=torch.int64, device=dev)

    def args(self, y_local, col0):
        return (_lib.DTYPE_CODE[y_local.dtype], y_local.data_ptr(), y_local.shape[0], y_local.shape[1],
                y_local.stride(0), col0, self.y_full.data_ptr(), self.y_full.shape[1], self.y_full.stride(0),
                self.ptrs.data_ptr(), self.inboxes[0].numel())

    def half(self, rank, epoch):
        m, n_total = self.y_full.shape
        return self.inboxes[rank].reshape(2, m, n_total)[epoch & 1]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n_local,out_col,ldy", [(1, 4096, 4096, 16384), (8, 1000, 3, 2011),
                                                   (20, 14336, 0, 14336)])
def test_noalloc_matches_existing_entry_point(cuda, m, n_local, out_col, ldy, dtype, timeouts_at_start):
    """Two calls in a row on one device (world 1, the output a column window
    of a wider buffer): bitwise the existing entry point's output, and the
    buffer's other columns stay untouched."""
    g = torch.Generator("cuda").manual_seed(m + n_local)
    ref = Exchange(m, n_local, dtype, cuda, ldy=ldy, out_col=out_col)
    new = Exchange(m, n_local, dtype, cuda, ldy=ldy, out_col=out_col)
    for call in range(2):
        y_local = torch.randn(m, n_local, device=cuda, generator=g).to(dtype)
        stream = _lib.stream_of(y_local)
        _lib.call("bnbq_peer_allgather_rows", *ref.args(y_local, 0), ref.state.data_ptr(), 1, 0, stream)
        _lib.call("bnbq_peer_allgather_rows_noalloc", *new.args(y_local, 0), 5, 1, 0, stream)
        torch.cuda.synchronize()
        assert torch.equal(new.buf, ref.buf), f"call {call}"
        assert torch.equal(new.y_full, y_local), f"call {call}"
    assert bool((new.buf[:, :out_col] == 7.0).all()) and bool((new.buf[:, out_col + n_local:] == 7.0).all())
    assert _lib.wait_timeouts() == timeouts_at_start


def test_world_one_slice_must_cover_the_output(cuda):
    e = Exchange(2, 128, torch.bfloat16, cuda)
    y = torch.zeros(2, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        _lib.call("bnbq_peer_allgather_rows", *e.args(y, 0), e.state.data_ptr(), 1, 0, _lib.stream_of(y))


def _calls(ex, y, peer, slot, epochs, stream):
    """Rank 0 of a group of two whose rank 1's words for `epochs` are written
    into rank 0's inbox beforehand (so nothing waits)."""
    for e in epochs:
        bits = peer.view(torch.int16).to(torch.int64) & 0xFFFF
        ex.half(0, e)[:, y.shape[1]:] = bits | (e << 32)
        _lib.call("bnbq_peer_allgather_rows_noalloc", *ex.args(y, 0), slot, 2, 0, stream)
    torch.cuda.synchronize()


def test_noalloc_setup_and_slot_reset(cuda, timeouts_at_start):
    """The set-up call alone succeeds; a reset slot starts its epochs from
    zero again, so a group with new zeroed inboxes can take it over. The
    epoch is visible in the words rank 0 sends to (local) rank 1."""
    _lib.call("bnbq_peer_allgather_noalloc_setup")
    y = torch.randn(2, 64, device=cuda).to(torch.bfloat16)
    peer = torch.randn(2, 64, device=cuda).to(torch.bfloat16)
    stream = _lib.stream_of(y)
    _lib.call("bnbq_peer_allgather_noalloc_reset", 11, stream)
    first = Exchange(2, 128, torch.bfloat16, cuda, world=2)
    _calls(first, y, peer, 11, (1, 2, 3), stream)
    assert bool((first.half(1, 1)[:, :64] >> 32 == 3).all()) and bool((first.half(1, 2)[:, :64] >> 32 == 2).all())
    second = Exchange(2, 128, torch.bfloat16, cuda, world=2)  # new inboxes: the slot must start over
    _lib.call("bnbq_peer_allgather_noalloc_reset", 11, stream)
    _calls(second, y, peer, 11, (1,), stream)
    assert bool((second.half(1, 1)[:, :64] >> 32 == 1).all()) and bool((second.half(1, 0) == 0).all())
    assert torch.equal(second.y_full, torch.cat([y, peer], dim=1))
    with pytest.raises(ValueError, match="fixed scratch"):
        _lib.call("bnbq_peer_allgather_noalloc_reset", 32, stream)
    assert _lib.wait_timeouts() == timeouts_at_start


def test_noalloc_rejects_slots_beyond_its_array(cuda):
    e = Exchange(1, 64, torch.bfloat16, cuda)
    y = torch.zeros(1, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="fixed scratch"):
        _lib.call("bnbq_peer_allgather_rows_noalloc", *e.args(y, 0), 32, 1, 0, _lib.stream_of(y))
    with pytest.raises(ValueError):
        _lib.call("bnbq_peer_allgather_rows_noalloc", *e.args(y, 0), -1, 1, 0, _lib.stream_of(y))


def _worker(rank, world, port, queue):
    import datetime
    import os
    import sys
    import traceback
    try:
        import torch.distributed as dist
        from bnb_b200.parallel import PeerGather
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        try:
            n_local, dtype = 1536, torch.bfloat16
            ref = PeerGather(8, world * n_local, dtype, dev)  # the existing entry point, its own state
            new = PeerGather(8, world * n_local, dtype, dev)  # its inboxes and output, the library's state
            g = torch.Generator(dev).manual_seed(10 + rank)
            for call, m in enumerate((8, 3)):
                y_local = torch.randn(m, n_local, device=dev, generator=g).to(dtype)
                want = ref.gather(y_local, rank * n_local).clone()
                _lib.call("bnbq_peer_allgather_rows_noalloc", _lib.DTYPE_CODE[dtype], y_local.data_ptr(), m,
                          n_local, y_local.stride(0), rank * n_local, new.y_full.data_ptr(), world * n_local,
                          new.y_full.stride(0), new.inbox_ptrs.data_ptr(), new.inbox.numel(), 7, world, rank,
                          _lib.stream_of(y_local))
                torch.cuda.synchronize()
                assert torch.equal(new.y_full[:m], want), f"call {call}"
            # a second group (new zeroed inboxes) takes the slot over after a reset
            other = PeerGather(8, world * n_local, dtype, dev)
            _lib.call("bnbq_peer_allgather_noalloc_reset", 7, _lib.stream_of(other.y_full))
            torch.cuda.synchronize()
            dist.barrier()
            for call in range(2):
                y_local = torch.randn(4, n_local, device=dev, generator=g).to(dtype)
                want = ref.gather(y_local, rank * n_local).clone()
                _lib.call("bnbq_peer_allgather_rows_noalloc", _lib.DTYPE_CODE[dtype], y_local.data_ptr(), 4,
                          n_local, y_local.stride(0), rank * n_local, other.y_full.data_ptr(), world * n_local,
                          other.y_full.stride(0), other.inbox_ptrs.data_ptr(), other.inbox.numel(), 7, world,
                          rank, _lib.stream_of(y_local))
                torch.cuda.synchronize()
                assert torch.equal(other.y_full[:4], want), f"second group, call {call}"
            assert _lib.wait_timeouts() == 0
            dist.barrier()
            ref.close()
            new.close()
            other.close()
        finally:
            dist.destroy_process_group()
        queue.put((rank, None))
    except BaseException:
        tb = traceback.format_exc()
        print(f"rank {rank}:\n{tb}", file=sys.stderr, flush=True)
        queue.put((rank, tb))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_noalloc_two_ranks_match_existing_entry_point():
    """One process per GPU over CUDA IPC, as PeerGather sets it up: two
    exchanges in a row through the library's state, bitwise the existing
    entry point's output."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    errs = []
    try:
        for _ in range(2):
            rank, err = queue.get(timeout=240)
            if err:
                errs.append(f"rank {rank}:\n{err}")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert not errs, "\n".join(errs)
