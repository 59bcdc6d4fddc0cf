"""The MLP split by output features over the ranks of a ShardGroup
(xvram_b200.mlp.ShardedMLP, the multi-GPU form of C5): each rank streams its rows of
every weight through its own small device budget, and the activation row blocks are
all-gathered over NVLink between layers.  One rank on one GPU (the exchange reduces to
the staging copies), two ranks on two GPUs; both against an FP64 forward."""
from __future__ import annotations

import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

MiB = 1 << 20
F, BATCH, LAYERS = 1024, 64, 5


def problem():
    rng = np.random.default_rng(17)
    W = [(rng.standard_normal((F, F)) / np.sqrt(F)).astype(np.float32) for _ in range(LAYERS)]
    bias = rng.uniform(-1 / 32, 1 / 32, (LAYERS, F)).astype(np.float32)
    x = rng.uniform(-1, 1, (BATCH, F)).astype(np.float32)
    return W, bias, x


def reference(W, bias, x):
    ref = x.astype(np.float64)
    for i in range(LAYERS):
        ref = np.maximum(ref @ W[i].astype(np.float64).T + bias[i], 0.0)
    return ref


def run_rank(rank, world, uid, budget_mib, q):
    import torch
    torch.cuda.set_device(rank)
    from xvram_b200 import sdk
    from xvram_b200.mlp import ShardedMLP
    from xvram_b200.shard import ShardGroup
    W, bias, x = problem()
    Fr = F // world
    rows = slice(rank * Fr, (rank + 1) * Fr)
    cfg = sdk.session_config(device_ordinal=rank, chunk_size_bytes=2 * MiB,
                             cache_target_bytes=budget_mib * MiB)
    out = np.empty((BATCH, F), dtype=np.float32)
    with ShardGroup(uid, rank, world) as g, sdk.Sdk(cfg) as s:
        net = ShardedMLP(s, g, F, BATCH, LAYERS)
        for i, w in enumerate(W):
            # this rank's rows of W (out x in), column-major Fr x F: C-order bytes of w_r.T
            net.load_weight(i, np.ascontiguousarray(w[rows, :].T))
        net.load_biases(np.ascontiguousarray(bias[:, rows]))
        for _ in range(2):
            net.forward(x, out)
        tel = s.telemetry()
        statuses = list(net.statuses)
        net.close()
    res = (rank, out, statuses, int(tel.handle_reuses), int(tel.bytes_h2d))
    if q is not None:
        q.put(res)
    return res


def check(results):
    W, bias, x = problem()
    ref = reference(W, bias, x)
    for rank, out, statuses, _, _ in results:
        assert statuses and all(st == 0 for st in statuses), (rank, statuses)
        err = float(np.max(np.abs(out - ref)))
        assert err <= 1e-5 * np.sqrt(F) * LAYERS, (rank, err)


def test_one_rank():
    from xvram_b200.shard import unique_id
    res = run_rank(0, 1, unique_id(), 16, None)
    check([res])
    assert res[3] > 0  # 20 MiB of weights through 16 MiB: frames reused


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_exchange_activations_over_nvlink():
    from xvram_b200.shard import unique_id
    uid = unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=run_rank, args=(r, 2, uid, 8, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    check(results)
    # each rank streamed its half of the weights through its budget: frames were reused
    assert all(reuses > 0 for _, _, _, reuses, _ in results)
