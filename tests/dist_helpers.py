"""Run a function on `world` CPU processes joined in a gloo process group
(127.0.0.1 rendezvous, spawned children, bounded waits)."""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import socket
import sys
import traceback


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(fn, rank, world, port, queue, args):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        try:
            fn(rank, world, *args)
        finally:
            dist.destroy_process_group()
        queue.put((rank, None))
    except BaseException:  # reported to the parent, which fails the test
        tb = traceback.format_exc()
        print(f"rank {rank}:\n{tb}", file=sys.stderr, flush=True)  # survives a crash during teardown
        queue.put((rank, tb))


def run_ranks(fn, world: int, *args, timeout: float = 180.0) -> None:
    """fn(rank, world, *args) on every rank; raise if any rank fails or hangs."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, queue, args)) for r in range(world)]
    for p in procs:
        p.start()
    errors = {}
    try:
        for _ in range(world):
            rank, err = queue.get(timeout=timeout)
            if err:
                errors[rank] = err
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    if errors:
        raise AssertionError("\n".join(f"rank {r}:\n{e}" for r, e in sorted(errors.items())))
