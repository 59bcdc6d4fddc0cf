"""Host side of the multi-rank path on CPU: group-id exchange and max-over-ranks timing
over a world-size-2 gloo group (no GPU, no NCCL communicator is created)."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    obj = [bytes(range(128)) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, obj[0], float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_id_exchange_and_max_reduce_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [g[1] for g in got] == [bytes(range(128))] * 2
    assert [g[2] for g in got] == [2.0, 2.0]


def test_unique_id_without_gpu():
    """Drawing a group id needs NCCL's bootstrap only, not a device."""
    from xvram_b200 import shard
    try:
        uid = shard.unique_id()
    except RuntimeError:
        return  # no NCCL library on this host: nothing else to check
    assert len(uid) == shard.ID_BYTES
