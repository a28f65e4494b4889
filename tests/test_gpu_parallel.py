"""Row-sharded NF4 matmul and block-sharded quantize over NCCL on 2 GPUs (one
process per GPU). Skipped on a box with fewer than two GPUs; the same logic is
covered on CPU with gloo in test_parallel.py."""
from __future__ import annotations

import pytest
import torch

from dist_helpers import _free_port

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, queue):
    import datetime
    import os
    import traceback
    try:
        import torch.distributed as dist
        import bnb_b200 as bnb
        from bnb_b200.parallel import (PeerGather, all_gather_flat, block_partition, matmul_rows, matmul_sharded,
                                       quantize_shard, row_partition, shard_rows)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        try:
            g = torch.Generator(dev).manual_seed(3)  # the same weight and x on every rank
            n, k = 1024, 2048
            w = bnb.quantize((torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16), "nf4", 64,
                             double_quant=True)
            ranges = row_partition(n, k, 64, world)
            shard = shard_rows(w, *ranges[rank])
            for m in (1, 7, 20, 33, 300):  # GEMV and GEMM routes
                x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
                y = matmul_sharded(x, shard, ranges)
                assert torch.equal(y, bnb.matmul(x, w)), m
            # the same exchange through NVLink peer memory, eager and from a CUDA graph
            pg = PeerGather(20, n, torch.bfloat16, dev)
            for m in (1, 7, 20, 3):
                x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
                y = pg.gather(matmul_rows(x, shard), ranges[rank][0]).clone()
                assert torch.equal(y, bnb.matmul(x, w)), ("peer", m)
            xg = torch.randn(8, k, device=dev, generator=g).to(torch.bfloat16)
            want = bnb.matmul(xg, w)
            out = torch.empty_like(want)
            stream = torch.cuda.Stream(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    for _ in range(2):
                        out.copy_(pg.gather(matmul_rows(xg, shard), ranges[rank][0]))
            for _ in range(3):
                out.zero_()
                graph.replay()
                torch.cuda.synchronize()
                assert torch.equal(out, want), "graph replay"
            del graph
            # back-to-back gathers with different inputs on one PeerGather, each
            # result read by a consumer kernel enqueued before the next gather;
            # rank 1 delays its consumers so rank 0 runs ahead into the next call
            # (whose stores must wait for rank 1's next gather to start)
            xs = [torch.randn(4, k, device=dev, generator=g).to(torch.bfloat16) for _ in range(6)]
            consumed = []
            for xi in xs:
                y = pg.gather(matmul_rows(xi, shard), ranges[rank][0])
                if rank == 1:
                    torch.cuda._sleep(2_000_000)
                consumed.append(y.float() * 1.0)
            torch.cuda.synchronize()
            for i, (xi, got) in enumerate(zip(xs, consumed)):
                assert torch.equal(got, bnb.matmul(xi, w).float()), ("back-to-back", i)
            # the matmul and the exchange in one call (the GEMV's own epilogue
            # exchanges for M <= 2), eagerly and from a CUDA graph; a wide
            # weight takes the table GEMV's route
            for m in (1, 2, 3, 7, 20):  # the same kernels on each rank's rows, gathered by NCCL
                x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
                assert torch.equal(pg.matmul(x, shard).clone(), matmul_sharded(x, shard, ranges)), ("fused", m)
            w2 = bnb.quantize((torch.randn(4096, 1024, device=dev, generator=g) * 0.02).to(torch.bfloat16), "nf4",
                              64, double_quant=True)
            r2 = row_partition(4096, 1024, 64, world)
            sh2 = shard_rows(w2, *r2[rank])
            pg2 = PeerGather(2, 4096, torch.bfloat16, dev)
            for m in (1, 2, 1):
                x = torch.randn(m, 1024, device=dev, generator=g).to(torch.bfloat16)
                want = matmul_sharded(x, sh2, r2)
                assert torch.equal(pg2.matmul(x, sh2).clone(), want), ("fused table", m)
                if world == 2:  # 2048-row shards take the table GEMV, as the whole weight does
                    assert torch.equal(want, bnb.matmul(x, w2)), ("table rows vs whole", m)
            xs2 = [torch.randn(1, 1024, device=dev, generator=g).to(torch.bfloat16) for _ in range(4)]
            wants = [matmul_sharded(xi, sh2, r2) for xi in xs2]
            outs = [torch.empty(1, 4096, dtype=torch.bfloat16, device=dev) for _ in xs2]
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    for xi, o in zip(xs2, outs):
                        pg2.matmul(xi, sh2, out=o)
            for _ in range(3):
                for o in outs:
                    o.zero_()
                graph.replay()
                torch.cuda.synchronize()
                for want, o in zip(wants, outs):
                    assert torch.equal(o, want), "fused graph replay"
            del graph
            torch.cuda.synchronize()
            dist.barrier()
            pg2.close()
            from bnb_b200 import _lib
            assert _lib.wait_timeouts() == 0
            # block-sharded quantize == the whole tensor's codes and absmax
            nel = 3 * 64 * 256 + 37
            xf = torch.randn(nel, device=dev, generator=g).to(torch.bfloat16)
            blocks = block_partition(nel, 64, world, align_blocks=256)
            a, b = blocks[rank]
            qa = quantize_shard(xf[a:b], "nf4", 64, double_quant=True)
            full = bnb.quantize(xf, "nf4", 64, double_quant=True)
            codes = all_gather_flat(qa.data, [(s // 2, -(-e // 2)) for s, e in blocks])
            assert torch.equal(codes, full.data)
            assert torch.equal(qa.absmax.offset, full.absmax.offset)
            b0 = a // 64
            assert torch.equal(qa.absmax.data, full.absmax.data[b0:b0 + qa.absmax.data.numel()])
            dq = all_gather_flat(qa.dequantize(torch.bfloat16).reshape(-1), blocks)
            assert torch.equal(dq, full.dequantize(torch.bfloat16).reshape(-1))
            torch.cuda.synchronize()
        finally:
            dist.destroy_process_group()
        queue.put((rank, None))
    except BaseException:
        import sys
        tb = traceback.format_exc()
        print(f"rank {rank}:\n{tb}", file=sys.stderr, flush=True)  # survives a crash during teardown
        queue.put((rank, tb))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_row_shards_and_block_shards():
    """Run on 2 GPUs, or on 4 when the box has them (the exchange then has
    three peers per rank)."""
    import multiprocessing as mp
    world = 4 if torch.cuda.device_count() >= 4 else 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    errs = []
    try:
        for _ in range(world):
            rank, err = queue.get(timeout=240)
            if err:
                errs.append(f"rank {rank}:\n{err}")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert not errs, "\n".join(errs)
