"""Multi-GPU partitioning of the hot path: one process per GPU, torch.distributed.

The reference runs on one device; a user of this package shards in two ways,
neither of which exchanges data on the compute path:

* **NF4 matmul by output rows.** Rank ``r`` holds rows ``[start, stop)`` of a
  weight (N, K) -- its slice of the codes, its slice of the block scales (or of
  the nested scale codes, with the whole second-level ``absmax2`` and the
  shard's first global block index) -- and computes ``y[:, start:stop]`` with
  the fused kernels. x is replicated. :func:`all_gather_rows` (NCCL all-gather,
  or any backend torch.distributed offers) assembles the full ``y`` only when
  the caller asks for it.
* **Quantize / dequantize by whole blocks.** Rank ``r`` holds elements
  ``[start, stop)`` of the flat tensor, a whole number of blocks (the partial
  last block on the last rank), and quantizes or decodes them alone. Double
  quantization needs the mean of all ranks' absmax: one all-reduce of a float64
  sum and a count (:func:`global_absmax_offset`).

The plans (:func:`row_partition`, :func:`block_partition`) and the collective
steps take CPU or CUDA tensors alike; only :func:`matmul_rows`,
:func:`quantize_shard` and :func:`dequantize_shard` launch the CUDA kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .array import _NESTED_BLOCKSIZE, QuantizedArray
from .kernels import create_dynamic_map, quantize_blockwise, quantize_nf4

__all__ = [
    "PeerGather",
    "RowShard",
    "all_gather_flat",
    "all_gather_rows",
    "block_partition",
    "dequantize_shard",
    "global_absmax_offset",
    "matmul_rows",
    "matmul_sharded",
    "quantize_shard",
    "row_partition",
    "shard_from_dict",
    "shard_rows",
]


# ------------------------------------------------------------------ row shards

def row_partition(n_rows: int, k: int, blocksize: int, world: int) -> list[tuple[int, int]]:
    """Balanced row ranges ``[(start, stop)] * world`` of an (n_rows, k) weight
    whose boundaries start whole blocks (``start * k % blocksize == 0``), so that
    every shard's codes and scales are contiguous slices. Trailing ranks may be
    empty when there are fewer row granules than ranks."""
    if world < 1 or n_rows < 0:
        raise ValueError(f"bad partition of {n_rows} rows over {world} ranks")
    granule = blocksize // math.gcd(k, blocksize)  # rows per whole number of blocks
    units = -(-n_rows // granule)
    bounds = [min(n_rows, granule * ((units * r) // world)) for r in range(world + 1)]
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


@dataclass
class RowShard:
    """Rows ``[start, stop)`` of an NF4 weight, in the form the fused kernels take.

    Attributes:
        data: packed codes of the rows, ``(stop - start) * k / 2`` bytes.
        absmax: float32 block scales of the rows, or (double-quantized) the
            uint8 codes of those scales.
        nested: ``(absmax2, code2, offset, blocksize2)`` of a double-quantized
            weight -- absmax2 whole, since it is indexed by global block -- else None.
        block0: global index of the shard's first block (the nested scale of
            local block ``b`` is ``absmax2[(block0 + b) // blocksize2]``).
        start, stop: the rows. n_rows_total, k: the full weight's shape.
    """

    data: torch.Tensor
    absmax: torch.Tensor
    nested: tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None
    blocksize: int
    block0: int
    start: int
    stop: int
    n_rows_total: int
    k: int

    @property
    def n_rows(self) -> int:
        return self.stop - self.start

    def to(self, device) -> RowShard:
        """Copy the shard's tensors to ``device`` (each rank moves only its own rows)."""
        nested = None
        if self.nested is not None:
            a2, c2, off, bs2 = self.nested
            nested = (a2.to(device), c2.to(device), off.to(device), bs2)
        return RowShard(self.data.to(device), self.absmax.to(device), nested, self.blocksize, self.block0,
                        self.start, self.stop, self.n_rows_total, self.k)


def shard_rows(w: QuantizedArray, start: int, stop: int) -> RowShard:
    """Rows ``[start, stop)`` of a 2-D NF4 weight as views of its tensors
    (use :func:`row_partition` for the ranges)."""
    if w.qtype != "nf4" or w.ndim != 2:
        raise ValueError(f"row shards are of 2-D NF4 weights, got {w.qtype} {w.shape}")
    n, k = w.shape
    bs = w.blocksize
    if not 0 <= start <= stop <= n or (start * k) % bs or ((stop * k) % bs and stop != n):
        raise ValueError(f"rows [{start}, {stop}) of a ({n}, {k}) weight do not start whole blocks of {bs}")
    b0, b1 = start * k // bs, -(-stop * k // bs)
    data = w.data.reshape(-1)[start * k // 2:stop * k // 2]
    absmax = w.absmax
    if isinstance(absmax, QuantizedArray):
        if absmax.offset is None or absmax.code is None or isinstance(absmax.absmax, QuantizedArray):
            raise ValueError("row shards support one level of centred 8-bit nested scales")
        nested = (absmax.absmax.reshape(-1), absmax.code.reshape(-1), absmax.offset.reshape(()),
                  absmax.blocksize)
        scales = absmax.data.reshape(-1)[b0:b1]
    else:
        nested = None
        scales = absmax.reshape(-1)[b0:b1]
    return RowShard(data, scales, nested, bs, b0, start, stop, n, k)


def shard_from_dict(weight: torch.Tensor, qs_dict: dict, rank: int, world: int,
                    device: torch.device | str | None = None) -> RowShard:
    """This rank's rows of a 4-bit weight saved by HuggingFace with
    bitsandbytes, loaded straight into ``device``: the arguments of
    :meth:`QuantizedArray.from_dict` (``weight`` and ``qs_dict`` may stay in
    host memory, e.g. from a safetensors file), the row range from
    :func:`row_partition` (whole nested blocks when double-quantized, so the
    scale codes split cleanly), and only that range's codes and scales --
    plus the small second-level arrays -- are copied to the device. The full
    weight never lands on any GPU."""
    w = QuantizedArray.from_dict(weight, qs_dict)
    if w.ndim != 2:
        raise ValueError(f"row shards are of 2-D weights, got shape {w.shape}")
    n, k = w.shape
    unit = w.blocksize
    if isinstance(w.absmax, QuantizedArray):
        unit *= w.absmax.blocksize
    start, stop = row_partition(n, k, unit, world)[rank]
    shard = shard_rows(w, start, stop)
    return shard if device is None else shard.to(device)


def matmul_rows(x: torch.Tensor, shard: RowShard, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ W[start:stop].T`` for an (M, K) bfloat16/float16 CUDA x: the fused
    GEMV (M <= 20) or tcgen05 GEMM, on this rank's rows only."""
    from .kernels.gemv import matmul_nf4
    if x.dim() != 2 or x.shape[1] != shard.k:
        raise ValueError(f"x {tuple(x.shape)} does not match a K={shard.k} weight")
    if shard.n_rows == 0:  # a trailing rank with no row granule
        return x.new_empty((x.shape[0], 0)) if out is None else out
    return matmul_nf4(x, shard.data, shard.absmax, shard.n_rows, shard.blocksize, nested=shard.nested,
                      absmax2_block0=shard.block0, out=out)


def all_gather_rows(y_local: torch.Tensor, ranges: list[tuple[int, int]], group=None) -> torch.Tensor:
    """Assemble ``y`` (M, N) from every rank's ``y[:, start:stop]``: one
    all-gather of equal-sized, zero-padded pieces (NCCL over NVLink on GPUs),
    then one copy into place."""
    world = dist.get_world_size(group)
    assert len(ranges) == world, (len(ranges), world)
    m = y_local.shape[0]
    width = max(b - a for a, b in ranges)
    piece = y_local.new_zeros((m, width))
    piece[:, :y_local.shape[1]] = y_local
    parts = _all_gather_bytes(piece, world, group)
    return torch.cat([p[:, :b - a] for p, (a, b) in zip(parts, ranges)], dim=1)


# CUDA IPC mappings opened in this process, by (device, handle): one handle can
# be opened only once per process, and small buffers of different owners'
# tensors often share one allocation (and so one handle).
_IPC_OPEN: dict[tuple[int, bytes], list[int]] = {}  # -> [base, references]


def _ipc_open(device: torch.device, handle: bytes) -> int:
    import ctypes as C
    from . import _lib
    key = (device.index, handle)
    if key not in _IPC_OPEN:
        base = C.c_void_p(0)
        hb = C.create_string_buffer(handle, 64)
        with torch.cuda.device(device):
            _lib.call("bnbq_ipc_open", C.cast(hb, C.c_void_p), C.addressof(base))
        _IPC_OPEN[key] = [base.value, 0]
    _IPC_OPEN[key][1] += 1
    return _IPC_OPEN[key][0]


def _ipc_close(device: torch.device, handle: bytes) -> None:
    from . import _lib
    key = (device.index, handle)
    entry = _IPC_OPEN[key]
    entry[1] -= 1
    if entry[1] == 0:
        with torch.cuda.device(device):
            _lib.call("bnbq_ipc_close", entry[0])
        del _IPC_OPEN[key]


class PeerGather:
    """All-gather of row-sharded outputs through NVLink peer memory.

    Every rank allocates an inbox of ``2 * max_rows * n_total`` 8-byte words
    (zeroed), shared with the other ranks through CUDA IPC (handles exchanged
    with ``all_gather_object``), a full output buffer that only it writes, and
    a small state word. :meth:`gather` then enqueues ONE kernel
    (``bnbq_peer_allgather_rows``): it stores this rank's slice into every
    peer's inbox as {value, epoch} words, copies it into the output, and fills
    the other columns from this rank's own inbox as the peers' words arrive
    (bounded waits) -- no NCCL call and no handshake on the data path.
    Construct it on every rank of ``group`` (a collective), and call
    :meth:`gather` on every rank in the same order. The returned tensor (a
    view of this rank's buffer, or ``out``) stays valid until this rank's
    next :meth:`gather` on the stream."""

    def __init__(self, max_rows: int, n_total: int, dtype: torch.dtype, device: torch.device, group=None):
        import ctypes as C
        from . import _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_total = n_total
        self.max_rows = max_rows
        self.dtype = dtype
        self.device = torch.device(device)
        self.y_full = torch.zeros((max_rows, n_total), dtype=dtype, device=device)
        self.inbox = torch.zeros(2 * max_rows * n_total, dtype=torch.int64, device=device)
        self.state = torch.zeros(2, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)

        def export(t):
            h = C.create_string_buffer(64)
            off = C.c_int64(0)
            with torch.cuda.device(self.device):
                _lib.call("bnbq_ipc_handle", t.data_ptr(), C.cast(h, C.c_void_p), C.addressof(off))
            return h.raw, off.value

        objs: list = [None] * self.world
        dist.all_gather_object(objs, export(self.inbox), group=group)
        self._opened: list[bytes] = []  # the peers' handles mapped here
        ptrs = []
        for r, (h, off) in enumerate(objs):
            if r == self.rank:
                ptrs.append(self.inbox.data_ptr())
                continue
            ptrs.append(_ipc_open(self.device, h) + off)
            self._opened.append(h)
        self.inbox_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the peers' inboxes (every rank, after its last gather has completed)."""
        torch.cuda.synchronize(self.device)
        for handle in self._opened:
            _ipc_close(self.device, handle)
        self._opened = []

    def _out(self, m: int, dtype, out):
        if m > self.max_rows or dtype != self.dtype:
            raise ValueError(f"{m} rows of {dtype} do not fit this gather ({self.max_rows} rows, {self.dtype})")
        if out is None:
            return self.y_full[:m]
        if out.shape != (m, self.n_total) or out.dtype != self.dtype or out.stride(1) != 1:
            raise ValueError(f"out {tuple(out.shape)} {out.dtype} is not an ({m}, {self.n_total}) {self.dtype} "
                             "matrix with unit column stride")
        return out

    def matmul(self, x: torch.Tensor, shard: RowShard, out: torch.Tensor | None = None) -> torch.Tensor:
        """``x @ W.T`` in full on every rank: this rank's rows of W (``shard``)
        and the exchange in one call (``bnbq_matmul_nf4_allgather``). For
        M <= 2 the matmul kernel itself stores its rows into the peers'
        inboxes and collects theirs (no separate exchange kernel). Bitwise
        :func:`matmul_rows` on every rank's rows, gathered."""
        from . import _lib
        if x.dim() != 2 or x.shape[1] != shard.k or shard.n_rows_total != self.n_total:
            raise ValueError(f"x {tuple(x.shape)} and a ({shard.n_rows_total}, {shard.k}) weight do not match "
                             f"this gather's {self.n_total} columns")
        if x.dtype not in (torch.bfloat16, torch.float16):
            raise NotImplementedError(f"matmul of {x.dtype} x is not implemented")
        m, k = x.shape
        out = self._out(m, x.dtype, out)
        if not x.is_contiguous() or x.data_ptr() % 16:
            x = _lib.aligned(x)
        dev = x.device
        plan = _shard_plan(shard, dev)
        stream = torch._C._cuda_getCurrentRawStream(dev.index)
        ws_ptr, ws_n = None, 0
        nb = plan.ws_bytes(m)
        if nb:
            ws = _lib.workspace(dev, stream, nb)
            ws_ptr, ws_n = ws.data_ptr(), ws.numel()
        w, a, aq, a2, c2, off = plan.ptrs
        args = (_lib.DTYPE_CODE[x.dtype], x.data_ptr(), m, k, w, shard.n_rows, shard.blocksize, a, aq, a2, c2, off,
                plan.bs2, shard.block0, out.data_ptr(), self.n_total, out.stride(0), shard.start,
                self.inbox_ptrs.data_ptr(), self.inbox.numel(), self.state.data_ptr(), self.world, self.rank,
                ws_ptr, ws_n, stream)
        if torch._C._cuda_getDevice() == dev.index:
            st = _lib.lib().bnbq_matmul_nf4_allgather(*args)
        else:
            with torch.cuda.device(dev):
                st = _lib.lib().bnbq_matmul_nf4_allgather(*args)
        if st:
            _lib.check(st, "bnbq_matmul_nf4_allgather")
        return out

    def gather(self, y_local: torch.Tensor, col0: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Columns [col0, col0 + y_local.shape[1]) from this rank, the rest
        from the peers: the full (m, n_total) output, in ``out`` if given (an
        (m, n_total) tensor of y's dtype with unit column stride)."""
        from . import _lib
        m, n_local = y_local.shape
        out = self._out(m, y_local.dtype, out)
        assert y_local.stride(1) == 1
        with torch.cuda.device(y_local.device):
            _lib.call("bnbq_peer_allgather_rows", _lib.DTYPE_CODE[y_local.dtype], y_local.data_ptr(), m, n_local,
                      y_local.stride(0), col0, out.data_ptr(), self.n_total, out.stride(0),
                      self.inbox_ptrs.data_ptr(), self.inbox.numel(), self.state.data_ptr(), self.world, self.rank,
                      _lib.stream_of(y_local))
        return out


class _ShardPlan:
    """A RowShard's C-ABI arguments, prepared once (aligned device tensors
    and their addresses) and cached on the shard."""

    __slots__ = ("data", "absmax", "device", "ptrs", "bs2", "keep", "k", "n", "_ws")

    def __init__(self, shard: RowShard, device):
        from . import _lib
        from .kernels.gemv import _CHUNK, _f32_on
        from .kernels.dequantize import _log2_blocksize
        self.data, self.absmax, self.device = shard.data, shard.absmax, device
        self.k, self.n = shard.k, shard.n_rows
        self._ws: dict[int, int] = {}
        if shard.k % _CHUNK:
            raise ValueError(f"K must be a multiple of {_CHUNK}, got {shard.k}")
        _log2_blocksize(shard.blocksize)
        if self.n == 0:
            self.ptrs, self.bs2, self.keep = (None,) * 6, 0, ()
            return
        _lib.require_cuda(shard.data, shard.absmax)
        w = _lib.aligned(shard.data.reshape(-1))
        if shard.nested is None:
            a = _lib.aligned(shard.absmax.reshape(-1), 4)
            self.keep = (w, a)
            self.ptrs = (w.data_ptr(), a.data_ptr(), None, None, None, None)
            self.bs2 = 0
        else:
            absmax2, code2, offset, bs2 = shard.nested
            _log2_blocksize(bs2)
            aq = _lib.aligned(shard.absmax.reshape(-1))
            a2 = _lib.aligned(_f32_on(absmax2, device).reshape(-1), 4)
            c2 = _lib.aligned(_f32_on(code2, device).reshape(-1), 4)
            off = _lib.aligned(_f32_on(offset, device).reshape(1), 4)
            self.keep = (w, aq, a2, c2, off)
            self.ptrs = (w.data_ptr(), None, aq.data_ptr(), a2.data_ptr(), c2.data_ptr(), off.data_ptr())
            self.bs2 = bs2

    def ws_bytes(self, m: int) -> int:
        from . import _lib
        from .kernels.gemv import GEMV_MAX_M
        nb = self._ws.get(m)
        if nb is None:
            nb = self._ws[m] = _lib.gemv_workspace_bytes(m, self.k, self.n) if self.n and m <= GEMV_MAX_M else 0
        return nb


def _shard_plan(shard: RowShard, device) -> _ShardPlan:
    plan = shard.__dict__.get("_bnbq_plan")
    if plan is None or plan.data is not shard.data or plan.absmax is not shard.absmax or plan.device != device:
        plan = _ShardPlan(shard, device)
        shard.__dict__["_bnbq_plan"] = plan
    return plan


def matmul_sharded(x: torch.Tensor, shard: RowShard, ranges: list[tuple[int, int]] | None = None,
                   group=None, gather: bool = True) -> torch.Tensor:
    """This rank's ``x @ W[start:stop].T``, all-gathered into the full (M, N)
    product when ``gather`` (``ranges`` as from :func:`row_partition`)."""
    y = matmul_rows(x, shard)
    if not gather:
        return y
    assert ranges is not None, "gathering needs every rank's row range"
    return all_gather_rows(y, ranges, group)


# ---------------------------------------------------------------- block shards

def block_partition(n: int, blocksize: int, world: int, align_blocks: int = 1) -> list[tuple[int, int]]:
    """Element ranges of a flat n-element tensor, each a whole number of
    ``blocksize * align_blocks`` elements except the last (which takes the
    partial tail). ``align_blocks = 256`` keeps every rank's absmax a whole
    number of nested blocks, as double quantization needs."""
    unit = blocksize * align_blocks
    units = -(-n // unit)
    bounds = [min(n, unit * ((units * r) // world)) for r in range(world + 1)]
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def global_absmax_offset(absmax_local: torch.Tensor, group=None) -> torch.Tensor:
    """The double-quantization offset -- mean of every rank's absmax -- from one
    all-reduce of a float64 (sum, count) pair; a float32 scalar on
    ``absmax_local``'s device. Without a process group: the local mean."""
    a = absmax_local.reshape(-1)
    acc = torch.stack([a.to(torch.float64).sum(), torch.tensor(float(a.numel()), dtype=torch.float64,
                                                                 device=a.device)])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=group)
    return (acc[0] / acc[1]).to(torch.float32)


def quantize_shard(x_local: torch.Tensor, qtype: str = "nf4", blocksize: int = 64, *,
                   code: torch.Tensor | None = None, double_quant: bool = False, group=None) -> QuantizedArray:
    """Quantize this rank's elements ``[start, stop)`` of a flat tensor (a range
    from :func:`block_partition`, ``align_blocks=256`` when ``double_quant``).
    The result equals the matching slice of quantizing the whole tensor: codes
    and absmax bitwise; with ``double_quant`` the offset is the all-reduced mean."""
    x = x_local.reshape(-1)
    if qtype == "nf4":
        data, absmax = quantize_nf4(x, blocksize=blocksize)
        code = None
    elif qtype == "8bit":
        code = (create_dynamic_map(device=x.device) if code is None
                else torch.as_tensor(code, dtype=torch.float32).reshape(-1).to(x.device))
        data, absmax = quantize_blockwise(x, code, blocksize=blocksize)
    else:
        raise NotImplementedError(f"quantization to {qtype!r} is not implemented")
    if double_quant:
        offset = global_absmax_offset(absmax, group).to(x.device)
        code2 = create_dynamic_map(device=x.device)
        q2, absmax2 = quantize_blockwise(absmax, code2, blocksize=_NESTED_BLOCKSIZE, offset=offset)
        absmax = QuantizedArray(q2, absmax2, code2, offset, "8bit", _NESTED_BLOCKSIZE, tuple(absmax.shape),
                                torch.float32)
    return QuantizedArray(data, absmax, code, None, qtype, blocksize, (x.numel(),), x.dtype)


def dequantize_shard(qa_local: QuantizedArray, dtype=None) -> torch.Tensor:
    """Decode this rank's block range (no collective)."""
    return qa_local.dequantize(dtype).reshape(-1)


def all_gather_flat(local: torch.Tensor, ranges: list[tuple[int, int]], group=None) -> torch.Tensor:
    """Concatenate every rank's flat piece ``[start, stop)`` into the whole tensor."""
    world = dist.get_world_size(group)
    assert len(ranges) == world, (len(ranges), world)
    width = max(b - a for a, b in ranges)
    piece = local.new_zeros(width)
    piece[:local.numel()] = local.reshape(-1)
    parts = _all_gather_bytes(piece, world, group)
    return torch.cat([p[:b - a] for p, (a, b) in zip(parts, ranges)])


def _all_gather_bytes(piece: torch.Tensor, world: int, group) -> list[torch.Tensor]:
    """all_gather of equal-shaped pieces moved as raw bytes (bit-exact for every
    dtype, and a type every backend carries)."""
    piece = piece.contiguous()
    raw = piece.view(torch.uint8)
    parts = [torch.empty_like(raw) for _ in range(world)]
    dist.all_gather(parts, raw, group=group)
    return [p.view(piece.dtype) for p in parts]
