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


def rank_rows(m, world, rank):
    per = (m + world - 1) // world
    r0 = min(m, rank * per)
    return r0, min(m, r0 + per) - r0


def run_rank(rank, world, uid, op_a, op_b, m, n, k, panel_k, q):
    """Computes this rank's rows and returns them (runs in the test process or a child)."""
    import torch
    torch.cuda.set_device(rank)
    from xvram_b200.shard import ShardGroup
    orc = load_oracle()
    a, b, c = operands(orc, op_a, op_b, m, n, k, 90)
    r0, mr = rank_rows(m, world, rank)
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
        st = g.sgemm(op_a, op_b, mr, n, k, 0.5, a_t, lda, b_t, b.shape[1], 1.5, c_t, mr,
                     panel_k=panel_k)
    out = (st, r0, c_t.numpy().copy())
    if q is not None:
        q.put(out)
    return out


def check_rows(orc, op_a, op_b, m, n, k, results):
    a, b, c = operands(orc, op_a, op_b, m, n, k, 90)
    ref = orc.gemm(op_a, op_b, m, n, k, 0.5, a, a.shape[1], b, b.shape[1], 1.5, c, m, threads=16)
    for st, r0, rows in results:
        assert st == 0
        mr = rows.shape[1]
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
