"""Multi-GPU partitioning logic on CPU: gloo process groups of 2 ranks.

The per-rank compute is the host oracle here (the CUDA kernels have no CPU
path); the plans, the shard slicing, the block-index bookkeeping of nested
scales and the collectives are the library's own. Row shards of an NF4 weight
all-gathered reproduce the unsharded product bitwise; block shards quantize to
the unsharded codes, absmax and nested codes bitwise, with the double-quant
offset from one all-reduce."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from bnb_b200 import QuantizedArray
from bnb_b200.parallel import (all_gather_flat, all_gather_rows, block_partition, global_absmax_offset,
                               row_partition, shard_rows)
from dist_helpers import run_ranks
from oracle import oracle as O


def _nf4_weight(n, k, bs, seed, double_quant=True):
    """A double-quantized NF4 weight built by the oracle, as CPU tensors."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    q, am = O.quantize_nf4(w, O.F32, bs)
    if not double_quant:
        return QuantizedArray(torch.from_numpy(q), torch.from_numpy(am), None, None, "nf4", bs, (n, k),
                              torch.bfloat16), am
    code = O.create_dynamic_map()
    off = O.mean_f32(am)
    q2, am2 = O.quantize_8bit(am, O.F32, 256, code, offset=off)
    nested = QuantizedArray(torch.from_numpy(q2), torch.from_numpy(am2), torch.from_numpy(code),
                            torch.tensor(off, dtype=torch.float32), "8bit", 256, (am.size,), torch.float32)
    scales = O.nested_absmax(q2, am2, code, off, 256)
    return QuantizedArray(torch.from_numpy(q), nested, None, None, "nf4", bs, (n, k), torch.bfloat16), scales


def test_row_partition_whole_blocks():
    for n, k, bs, world in [(4096, 14336, 64, 8), (1000, 96, 64, 3), (7, 32, 256, 4), (1024, 4096, 4096, 8)]:
        ranges = row_partition(n, k, bs, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a <= b for a, b in ranges) and all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
        assert all((a * k) % bs == 0 for a, _ in ranges)
        sizes = [b - a for a, b in ranges]
        granule = bs // np.gcd(k, bs)
        assert max(sizes) - min(sizes) <= granule


def test_block_partition_aligned():
    n = 3 * 64 * 256 + 37
    ranges = block_partition(n, 64, 2, align_blocks=256)
    assert ranges == [(0, 2 * 64 * 256), (2 * 64 * 256, n)]
    ranges = block_partition(1000, 64, 4)
    assert ranges[-1][1] == 1000 and all(a % 64 == 0 for a, _ in ranges)


def test_shard_rows_rejects_split_blocks():
    w, _ = _nf4_weight(8, 96, 64, 0, double_quant=False)
    with pytest.raises(ValueError):
        shard_rows(w, 1, 8)  # row 1 starts at element 96: mid-block


def _rows_worker(rank, world, n, k, bs, m, double_quant):
    w, scales_full = _nf4_weight(n, k, bs, 7, double_quant)
    rng = np.random.default_rng(11)
    x = O.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32)).reshape(m, k)
    ranges = row_partition(n, k, bs, world)
    shard = shard_rows(w, *ranges[rank])
    if double_quant:
        a2, c2, off, bs2 = shard.nested
        scales = O.nested_absmax(shard.absmax.numpy(), a2.numpy(), c2.numpy(), float(off), bs2, shard.block0)
        assert np.array_equal(scales, scales_full[shard.block0:shard.block0 + scales.size])
    else:
        scales = shard.absmax.numpy()
    y_local = O.gemv_ref(x, O.BF16, shard.data.numpy(), shard.n_rows, bs, scales)
    y = all_gather_rows(torch.from_numpy(y_local.view(np.int16)), ranges)
    y_full = O.gemv_ref(x, O.BF16, w.data.numpy(), n, bs, scales_full)
    assert np.array_equal(y.numpy().view(np.uint16), y_full)


@pytest.mark.parametrize("n,k,bs,m,dq", [(256, 512, 64, 3, True), (250, 96, 64, 2, True), (130, 256, 128, 1, False)])
def test_row_shards_gather_to_full_product(n, k, bs, m, dq):
    run_ranks(_rows_worker, 2, n, k, bs, m, dq)


def _blocks_worker(rank, world, n, bs):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(n).astype(np.float32)
    x[rng.random(n) < 0.1] *= 8.0
    q_full, am_full = O.quantize_nf4(x, O.F32, bs)
    ranges = block_partition(n, bs, world, align_blocks=256)
    a, b = ranges[rank]
    q, am = O.quantize_nf4(x[a:b], O.F32, bs)  # this rank's blocks alone
    b0 = a // bs
    assert np.array_equal(am, am_full[b0:b0 + am.size])
    offset = global_absmax_offset(torch.from_numpy(am))
    assert offset.dtype == torch.float32 and float(offset) == float(O.mean_f32(am_full))
    code = O.create_dynamic_map()
    q2, am2 = O.quantize_8bit(am, O.F32, 256, code, offset=float(offset))
    q2_full, am2_full = O.quantize_8bit(am_full, O.F32, 256, code, offset=float(offset))
    assert np.array_equal(q2, q2_full[b0:b0 + q2.size])
    assert np.array_equal(am2, am2_full[b0 // 256:b0 // 256 + am2.size])
    codes = all_gather_flat(torch.from_numpy(q), [(s // 2, -(-e // 2)) for s, e in ranges])
    assert np.array_equal(codes.numpy(), q_full)


def test_block_shards_quantize_like_whole():
    run_ranks(_blocks_worker, 2, 3 * 64 * 256 + 37, 64)
