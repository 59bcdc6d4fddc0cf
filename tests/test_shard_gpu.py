"""Multi-GPU partitioned SGEMM: C rows per rank, B panels all-gathered over NVLink."""
from __future__ import annotations

import multiprocessing as mp

import numpy as np
import pytest

from oracle_lib import TOLERANCE, load_oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)


def operands(orc, op_a, op_b, m, n, k, seed):
    a = orc.uniform(m * k, seed).reshape((m, k) if op_a else (k, m))   # stored k x m or m x k
    b = orc.uniform(k * n, seed + 1).reshape((k, n) if op_b else (n, k))
    c = orc.uniform(m * n, seed + 2).reshape(n, m)
    return a, b, c


def rank_rows(m, world, rank, split="even"):
    if split == "first":  # every row on rank 0, none on the others
        return (0, m) if rank == 0 else (m, 0)
    per = (m + world - 1) // world
    r0 = min(m, rank * per)
    return r0, min(m, r0 + per) - r0


def run_rank(rank, world, uid, op_a, op_b, m, n, k, panel_k, q, split="even", env=None,
             beta=1.5):
    """Computes this rank's rows and returns them (runs in the test process or a child)."""
    import os
    for key, val in (env or {}).items():
        os.environ[key] = val
    import torch
    torch.cuda.set_device(rank)
    from xvram_b200.shard import ShardGroup
    orc = load_oracle()
    a, b, c = operands(orc, op_a, op_b, m, n, k, 90)
    r0, mr = rank_rows(m, world, rank, split)
    # this rank's rows of op(A): op N -> rows r0.. of the m x k matrix; op T -> columns
    if op_a == 0:
        a_loc = np.ascontiguousarray(a[:, r0:r0 + mr])       # (k, mr): m-rows slice, ld mr
        lda = mr
    else:
        a_loc = np.ascontiguousarray(a[r0:r0 + mr, :])       # (mr, k): ld k
        lda = k
    c_loc = np.ascontiguousarray(c[:, r0:r0 + mr])
    a_t = torch.from_numpy(a_loc).pin_memory()
    b_t = torch.from_numpy(b).pin_memory()
    c_t = torch.from_numpy(c_loc).pin_memory()
    with ShardGroup(uid, rank, world) as g:
        st = g.sgemm(op_a, op_b, mr, n, k, 0.5, a_t, max(lda, 1), b_t, b.shape[1], beta, c_t,
                     max(mr, 1), panel_k=panel_k)
        # a second call on the same group reuses its buffers and must give the same rows
        if st == 0 and mr > 0 and beta == 0.0:
            first = c_t.numpy().copy()
            st = g.sgemm(op_a, op_b, mr, n, k, 0.5, a_t, lda, b_t, b.shape[1], beta, c_t, mr,
                         panel_k=panel_k)
            if st == 0 and not np.array_equal(first, c_t.numpy()):
                st = -1
    for key in (env or {}):
        os.environ.pop(key, None)
    out = (st, r0, c_t.numpy().copy())
    if q is not None:
        q.put(out)
    return out


def check_rows(orc, op_a, op_b, m, n, k, results, beta=1.5):
    a, b, c = operands(orc, op_a, op_b, m, n, k, 90)
    ref = orc.gemm(op_a, op_b, m, n, k, 0.5, a, a.shape[1], b, b.shape[1], beta, c, m, threads=16)
    for st, r0, rows in results:
        assert st == 0
        mr = rows.shape[1]
        if mr == 0:
            continue
        err = float(np.max(np.abs(rows.astype(np.float64) - ref[:, r0:r0 + mr]))) / k
        assert err <= TOLERANCE, err


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_single_rank_group_matches_oracle(op_a, op_b):
    from xvram_b200.shard import unique_id
    m, n, k = 600, 500, 700
    res = run_rank(0, 1, unique_id(), op_a, op_b, m, n, k, 256, None)
    check_rows(load_oracle(), op_a, op_b, m, n, k, [res])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("op_a,op_b", [(1, 0), (0, 1)])
def test_two_ranks_share_b_over_nvlink(op_a, op_b):
    from xvram_b200.shard import unique_id
    m, n, k = 1000, 777, 900
    uid = unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=run_rank, args=(r, 2, uid, op_a, op_b, m, n, k, 256, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    check_rows(load_oracle(), op_a, op_b, m, n, k, results)


# Small C blocks (ragged last block) and a device budget that forces row groups: the
# plan then runs several groups of A rows, each re-gathering B block by block.
# (6 MB: 2 to 5 row groups of 128-320 rows for three of the four op pairs at 600 x 500 x
# 700; 5 MB: 2 groups of 256 rows per rank in the two-rank case.)
BLOCKS_AND_GROUPS = {"XVRAM_B200_SHARD_BLOCK_N": "256", "XVRAM_B200_SHARD_BUDGET_BYTES": "6000000"}
BLOCKS_AND_GROUPS_2 = {"XVRAM_B200_SHARD_BLOCK_N": "256",
                       "XVRAM_B200_SHARD_BUDGET_BYTES": "5000000"}


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_single_rank_blocks_and_row_groups(op_a, op_b):
    from xvram_b200.shard import unique_id
    m, n, k = 600, 500, 700
    res = run_rank(0, 1, unique_id(), op_a, op_b, m, n, k, 256, None, env=BLOCKS_AND_GROUPS)
    check_rows(load_oracle(), op_a, op_b, m, n, k, [res])


def test_single_rank_beta_zero_repeatable():
    """beta = 0 never reads C; a second call on the same group gives identical rows."""
    from xvram_b200.shard import unique_id
    m, n, k = 333, 1100, 257
    res = run_rank(0, 1, unique_id(), 1, 0, m, n, k, 128, None, beta=0.0,
                   env={"XVRAM_B200_SHARD_BLOCK_N": "512"})
    check_rows(load_oracle(), 1, 0, m, n, k, [res], beta=0.0)


def _two_ranks(op_a, op_b, m, n, k, panel_k, split="even", env=None):
    from xvram_b200.shard import unique_id
    uid = unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=run_rank, args=(r, 2, uid, op_a, op_b, m, n, k, panel_k, q),
                         kwargs={"split": split, "env": env})
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    check_rows(load_oracle(), op_a, op_b, m, n, k, results)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_one_without_rows():
    """A rank with no rows still takes part in every all-gather."""
    _two_ranks(0, 0, 700, 600, 500, 256, split="first", env={"XVRAM_B200_SHARD_BLOCK_N": "256"})


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_blocks_and_row_groups():
    _two_ranks(1, 1, 900, 700, 600, 256, env=BLOCKS_AND_GROUPS_2)
