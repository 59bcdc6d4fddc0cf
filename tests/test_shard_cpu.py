"""The multi-GPU executor (xvram_b200_sgemm_sharded) on world-size 2 and 4 gloo ranks,
without a GPU.

Each rank is a spawned process that installs the host-memory fake device and creates its
shard group with collectives backed by torch.distributed over gloo
(xvram_b200_shard_group_create_custom).  The executor's own code then runs unchanged: the
plan exchange, the row groups, each rank's B slice copied and all-gathered, A arriving in
K panels, C's column blocks.  Each rank takes its rows from the library's partition
(xvram_b200_shard_rows) and checks

  * its rows of C against the CPU FP64 oracle, within the SGEMM tolerance (a wrong B slice
    on any rank corrupts every rank's result; a wrong row range corrupts its own);
  * that C's other rows, which belong to the other ranks, are untouched;
  * that every rank reports the same agreed plan (largest row count, smallest offered
    device memory, row groups, block width, slice sizes).

The cases cover ragged M with an empty rank, ragged last C blocks, every op(A) / op(B),
A arriving in several K panels, beta 0 and nonzero, and ranks offering different device
memory so that the smallest forces several row groups.
"""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest

TESTS = Path(__file__).resolve().parent
ROOT = TESTS.parent

# (op_a, op_b, m, n, k, alpha, beta, panel_k, block_n, budget per rank in KiB or None)
CASES = [
    (0, 0, 300, 200, 96, 1.0, 0.0, 0, 64, None),        # P=4: rank 0 empty; ragged block
    (1, 1, 600, 130, 200, 0.5, 1.5, 64, 64, None),      # K-major A in 4 panels; B sliced by k
    (1, 0, 700, 96, 160, -1.0, 0.25, 32, 32, (500, 300, 700, 900)),  # row groups
    (0, 1, 257, 70, 33, 2.0, -0.5, 0, 1024, None),      # one block; odd K
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _collectives(world):
    """all_reduce_max_u64 / all_gather_f32 over the default gloo group, on host memory."""
    import ctypes as C

    import numpy as np
    import torch
    import torch.distributed as dist

    def reduce_max(ptr, count, _stream):
        buf = np.ctypeslib.as_array((C.c_uint64 * count).from_address(ptr))
        vals = [None] * world
        dist.all_gather_object(vals, [int(v) for v in buf])
        buf[:] = np.array([max(col) for col in zip(*vals)], dtype=np.uint64)
        return 0

    def gather(send, recv, count, _stream):
        mine = torch.from_numpy(np.ctypeslib.as_array((C.c_float * count).from_address(send)).copy())
        parts = [torch.empty(count, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, mine)
        out = np.ctypeslib.as_array((C.c_float * (count * world)).from_address(recv))
        out[:] = torch.cat(parts).numpy()
        return 0

    return reduce_max, gather


def _rank_main(rank, world, port):
    sys.path[:0] = [str(ROOT), str(TESTS)]
    import numpy as np
    import torch.distributed as dist

    from fake_device import installed
    from oracle_lib import TOLERANCE, load_oracle, normalized_error
    from xvram_b200 import shard

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    orc = load_oracle()
    reduce_max, gather = _collectives(world)
    headroom = 1 << 30  # the executor leaves this much device memory free
    for ci, (op_a, op_b, m, n, k, alpha, beta, panel_k, block_n, budget) in enumerate(CASES):
        offer = (budget[rank % len(budget)] << 10) if budget else (256 << 20)
        os.environ["XVRAM_B200_SHARD_BLOCK_N"] = str(block_n)
        with installed(free_bytes=headroom + offer):
            group = shard.ShardGroup.custom(rank, world, reduce_max, gather)
            a = orc.uniform(m * k, 10 + ci).reshape((m, k) if op_a else (k, m))  # (cols, rows)
            b = orc.uniform(k * n, 20 + ci).reshape((k, n) if op_b else (n, k))
            c = orc.uniform(m * n, 30 + ci).reshape(n, m)
            lda, ldb = (k if op_a else m), (n if op_b else k)
            r0, mr = shard.rows(m, world, rank)
            out = c.copy()
            # this rank's rows: views into the full matrices, leading dimensions unchanged
            a_off = r0 * lda if op_a else r0
            a_ptr = a.ctypes.data + 4 * a_off
            c_ptr = out.ctypes.data + 4 * r0
            st = group.sgemm(op_a, op_b, mr, n, k, alpha, a_ptr, lda, b, ldb, beta, c_ptr, m,
                             panel_k=panel_k)
            assert st == 0, (ci, rank, st)
            plan = group.last_plan()
            group.close()
        ref = orc.gemm(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, m)
        rows = slice(r0, r0 + mr)
        if mr:
            err = normalized_error(out[:, rows], ref[:, rows], k, float(np.abs(a).max()),
                                   float(np.abs(b).max()))
            assert err <= TOLERANCE, (ci, rank, err)
        others = np.ones(m, dtype=bool)
        others[rows] = False
        assert np.array_equal(out[:, others], c[:, others]), (ci, rank, "wrote other rows")
        # the agreed plan is the same on every rank, and it is the one the numbers give
        plans = [None] * world
        shared = {key: v for key, v in plan.items()
                  if key not in ("rank", "h2d_bytes", "d2h_bytes")}
        dist.all_gather_object(plans, shared)
        assert all(p == plans[0] for p in plans), (ci, plans)
        want_m_max = max(shard.rows(m, world, q)[1] for q in range(world))
        assert plan["m_max"] == want_m_max
        offers = [((budget[q % len(budget)] << 10) if budget else (256 << 20))
                  for q in range(world)]
        assert plan["avail_min"] == min(offers)
        assert plan["device_bytes"] <= plan["avail_min"]
        assert plan["group_rows"] % 128 == 0
        assert plan["row_groups"] == -(-want_m_max // plan["group_rows"])
        assert plan["block_n"] == min(n, -(-block_n // 32) * 32)
        if op_b == 0:
            assert plan["b_slice_cols"] == -(-plan["block_n"] // world) and plan["b_slice_k"] == 0
        else:
            assert plan["b_slice_k"] == -(-k // world) and plan["b_slice_cols"] == 0
        blocks = -(-n // plan["block_n"])
        assert plan["gathers"] == blocks * plan["row_groups"]
        if budget:
            assert plan["row_groups"] > 1  # the smallest offer forced several groups
    dist.barrier()
    dist.destroy_process_group()


def _run(world: int) -> None:
    import torch.multiprocessing as tmp
    env_lib = os.environ.get("XVRAM_B200_LIBRARY")
    if not env_lib:
        pytest.skip("needs the test link of the library (tests/conftest.py)")
    tmp.start_processes(_rank_main, args=(world, _free_port()), nprocs=world, join=True,
                        start_method="spawn")


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_sharded_executor_over_gloo_ranks_matches_the_oracle(world):
    _run(world)


def test_row_partition_covers_every_row_once():
    from xvram_b200 import shard
    for m in (0, 1, 127, 128, 129, 300, 1000, 131072, 262144 + 5):
        for world in (1, 2, 3, 4, 8):
            parts = [shard.rows(m, world, r) for r in range(world)]
            assert parts[0][0] == 0
            for (b0, n0), (b1, _) in zip(parts, parts[1:]):
                assert b0 + n0 == b1
            assert sum(n for _, n in parts) == m
            full = [n for _, n in parts if n]
            # whole 128-row tiles except the last rank with rows; tile counts differ by <= 1
            assert all(b % 128 == 0 for b, n in parts if n)
            tiles = [-(-n // 128) for _, n in parts]
            assert max(tiles) - min(tiles) <= 1 or m == 0
            assert len(full) == min(world, -(-m // 128))


def test_unique_id_without_gpu():
    """Drawing a group id needs NCCL's bootstrap only, not a device."""
    from xvram_b200 import shard
    try:
        uid = shard.unique_id()
    except RuntimeError:
        return  # no NCCL library on this host: nothing else to check
    assert len(uid) == shard.ID_BYTES


def test_row_partition_rejects_bad_arguments():
    import ctypes as C
    from xvram_b200._native import lib
    b0, n = C.c_int64(0), C.c_int64(0)
    for m, world, rank in ((-1, 2, 0), (10, 0, 0), (10, 2, 2), (10, 2, -1)):
        assert lib.xvram_b200_shard_rows(m, world, rank, C.byref(b0), C.byref(n)) == 1
    assert lib.xvram_b200_shard_rows(10, 2, 0, None, C.byref(n)) == 1


def test_custom_group_rejects_incomplete_collectives():
    import ctypes as C
    from xvram_b200._native import ShardCollectives, lib
    ops = ShardCollectives()
    ops.struct_size = C.sizeof(ShardCollectives)
    out = C.c_uint64(0)
    # no functions
    assert lib.xvram_b200_shard_group_create_custom(C.byref(ops), 0, 1, C.byref(out)) == 1
    ops.all_reduce_max_u64 = ShardCollectives.ALL_REDUCE(lambda *a: 0)
    ops.all_gather_f32 = ShardCollectives.ALL_GATHER(lambda *a: 0)
    ops.struct_size = 8   # older/smaller than v1
    assert lib.xvram_b200_shard_group_create_custom(C.byref(ops), 0, 1, C.byref(out)) == 1
    ops.struct_size = C.sizeof(ShardCollectives)
    assert lib.xvram_b200_shard_group_create_custom(C.byref(ops), 1, 1, C.byref(out)) == 1
    assert lib.xvram_b200_shard_group_create_custom(None, 0, 1, C.byref(out)) == 1


def test_failing_collective_fails_the_call_and_poisons_the_group():
    """A collective that raises (or returns an error) fails the sharded call and leaves the
    group POISONED; nothing hangs (one rank, fake device)."""
    import numpy as np
    from fake_device import installed
    from xvram_b200 import shard

    def bad_reduce(ptr, count, stream):
        raise RuntimeError("peer lost")

    with installed():
        g = shard.ShardGroup.custom(0, 2, bad_reduce, lambda *a: 0)
        a = np.ones((64, 128), np.float32)
        b = np.ones((64, 128), np.float32)
        c = np.zeros((64, 128), np.float32)
        st = g.sgemm(0, 0, 128, 64, 64, 1.0, a, 128, b, 64, 0.0, c, 128)
        assert st == 13                                   # CUDA_ERROR from the collective
        assert g.sgemm(0, 0, 128, 64, 64, 1.0, a, 128, b, 64, 0.0, c, 128) == 15  # POISONED
        g.close()
