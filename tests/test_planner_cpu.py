"""Panel planner: coverage, slot-cache replay, budget and accounting invariants."""
from __future__ import annotations

import itertools

import pytest

from xvram_b200 import device

MiB = 1 << 20
GiB = 1 << 30


def ceil_div(a, b):
    return (a + b - 1) // b


def replay(steps, info, m, n, k, mb, nb, kb):
    """Replays the plan's slot assignments: every step must find its panels in the
    slots it names, loads happen only on misses, and the slot count is respected."""
    slots = {}
    loads = 0
    bm_n = ceil_div(m, mb)
    for (bm, bn, bk, sa, sb) in steps:
        for key, slot in ((("A", bm, bk), sa), (("B", bn, bk), sb)):
            assert 0 <= slot < info["panel_slots"]
            if slots.get(slot) != key:
                slots[slot] = key
                loads += 1
        assert sa != sb
    assert loads == info["panel_loads"]
    del bm_n
    return loads


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("shape", [(1000, 700, 3000), (4096, 4096, 4096), (130, 129, 33)])
def test_every_block_and_panel_covered_once(op_a, op_b, shape):
    m, n, k = shape
    budget = 256 * MiB
    st, steps = device.plan_steps(op_a, op_b, m, n, k, True, budget, 2 * MiB,
                                  force=(512, 512, 256))
    assert st == 0
    info = device.plan_panels(op_a, op_b, m, n, k, True, budget, 2 * MiB, force=(512, 512, 256))
    seen = set()
    for (bm, bn, bk, _, _) in steps:
        assert (bm, bn, bk) not in seen
        seen.add((bm, bn, bk))
    want = set(itertools.product(range(ceil_div(m, 512)), range(ceil_div(n, 512)),
                                 range(ceil_div(k, 256))))
    assert seen == want
    # the K panels of one C block are consecutive
    blocks = [(bm, bn) for (bm, bn, _, _, _) in steps]
    runs = [key for key, _ in itertools.groupby(blocks)]
    assert len(runs) == len(set(runs))
    replay(steps, info, m, n, k, 512, 512, 256)


def test_budget_respected_and_accounting():
    m = n = k = 16384
    budget = 2 * GiB
    q = 64 * MiB
    info = device.plan_panels(0, 1, m, n, k, True, budget, q)
    assert info["return_status"] == 0
    used = info["panel_slots"] * info["slot_bytes"] + info["c_slots"] * info["c_slot_bytes"]
    assert used <= budget
    assert info["slot_bytes"] % q == 0 and info["c_slot_bytes"] % q == 0
    assert info["block_m"] % 128 == 0 and info["block_n"] % 128 == 0 and info["panel_k"] % 32 == 0
    # C is read once (beta != 0) and written once; panels at least once each
    c_bytes = m * n * 4
    ab = (m * k + k * n) * 4
    assert info["d2h_bytes"] == c_bytes
    assert info["h2d_bytes"] >= c_bytes + ab
    assert info["panel_loads"] + info["panel_hits"] == 2 * info["steps"]


def test_everything_fits_loads_each_panel_once():
    m, n, k = 3000, 2000, 5000
    info = device.plan_panels(1, 0, m, n, k, False, 8 * GiB, 2 * MiB, force=(1024, 1024, 1024))
    bm, bn, bk = ceil_div(m, 1024), ceil_div(n, 1024), ceil_div(k, 1024)
    assert info["panel_loads"] == (bm + bn) * bk
    assert info["panel_evictions"] == 0
    assert info["h2d_bytes"] == (m * k + k * n) * 4  # beta == 0: C is not read
    assert info["d2h_bytes"] == m * n * 4


def test_tight_budget_evicts_and_reuses_slots():
    m = n = k = 8192
    info = device.plan_panels(0, 0, m, n, k, True, 512 * MiB, 2 * MiB, force=(2048, 2048, 1024))
    assert info["return_status"] == 0
    assert info["panel_evictions"] > 0
    st, steps = device.plan_steps(0, 0, m, n, k, True, 512 * MiB, 2 * MiB,
                                  force=(2048, 2048, 1024))
    assert st == 0
    replay(steps, info, m, n, k, 2048, 2048, 1024)


def test_belady_never_worse_than_lru_replay():
    """The plan's loads are no more than an LRU cache of the same size would need."""
    m = n = k = 6144
    force = (1024, 1024, 1024)
    budget = 160 * MiB
    info = device.plan_panels(0, 0, m, n, k, False, budget, 2 * MiB, force=force)
    st, steps = device.plan_steps(0, 0, m, n, k, False, budget, 2 * MiB, force=force)
    slots = info["panel_slots"]
    from collections import OrderedDict
    lru, lru_loads = OrderedDict(), 0
    for (bm, bn, bk, _, _) in steps:
        for key in (("A", bm, bk), ("B", bn, bk)):
            if key in lru:
                lru.move_to_end(key)
            else:
                lru_loads += 1
                if len(lru) >= slots:
                    lru.popitem(last=False)
                lru[key] = True
    assert info["panel_loads"] <= lru_loads


def test_budget_too_small_is_reported():
    info = device.plan_panels(0, 0, 65536, 65536, 65536, True, 64 * MiB, 64 * MiB)
    assert info["return_status"] != 0 and info["status"] == 2


def test_invalid_geometry_rejected():
    info = device.plan_panels(0, 0, 100, 100, 100, True, GiB, 2 * MiB, force=(100, 128, 32))
    assert info["status"] == 1


def test_out_of_core_c3_shape_is_compute_bound():
    """131072^3 NT with a 40 GiB budget: the chosen plan moves far
    less than the reference's chunk-granular schedule and predicts compute-bound time."""
    n = 131072
    info = device.plan_panels(0, 1, n, n, n, True, 40 * GiB, 64 * MiB, flops_per_s=70e12,
                              h2d=50e9, d2h=50e9)
    assert info["return_status"] == 0
    flops = 2.0 * n ** 3
    compute_s = flops / 70e12
    assert info["h2d_bytes"] / 50e9 < compute_s          # link time hides under compute
    assert info["est_seconds"] < compute_s * 1.15
    assert info["panel_evictions"] > 0                    # real eviction and slot reuse
