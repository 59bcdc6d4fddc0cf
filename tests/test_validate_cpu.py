"""Problem validation has the reference's error taxonomy (gemm::validate_problem)."""
from __future__ import annotations

from xvram_b200 import device


def test_validation_matches_reference_golden_table(golden):
    names = golden["problem_error_names"]
    for c in golden["validation"]:
        err, op = device.validate(c["m"], c["n"], c["k"], c["op_a"], c["op_b"], c["ids"],
                                  c["bytes"], c["offsets"], c["rows"], c["cols"], c["lds"])
        assert (names[err], op) == (names[c["error"]], c["operand"]), c["name"]


def test_validation_matches_live_reference(ref_lib):
    import ctypes as C
    import itertools
    import random
    rnd = random.Random(11)
    arr = lambda xs: (C.c_uint64 * 3)(*xs)
    for _ in range(3000):
        m, n, k = (rnd.choice([0, 1, 5, 37, 100]) for _ in range(3))
        oa, ob = rnd.randint(0, 1), rnd.randint(0, 1)
        rows = [m if oa == 0 else k, k if ob == 0 else n, m]
        cols = [k if oa == 0 else m, n if ob == 0 else k, n]
        rows = [r + rnd.choice([0, 0, 0, 1, -1]) for r in rows]
        rows = [max(r, 0) for r in rows]
        lds = [max(r, 1) + rnd.choice([0, 0, 3, -1]) for r in rows]
        ids = [rnd.choice([0, 1, 2, 3]) for _ in range(3)]
        nbytes = [rnd.choice([1 << 12, 1 << 16, 1 << 20, 0]) for _ in range(3)]
        offs = [rnd.choice([0, 0, 64, 4096, 1 << 19]) for _ in range(3)]
        op = C.create_string_buffer(1)
        want = ref_lib.xr_validate_problem(m, n, k, oa, ob, arr(ids), arr(nbytes), arr(offs),
                                           arr(rows), arr(cols), arr(lds), op)
        got, gop = device.validate(m, n, k, oa, ob, ids, nbytes, offs, rows, cols, lds)
        assert (got, gop) == (want, op.value.decode() if op.value else ""), (m, n, k, oa, ob, rows, cols, lds, ids, nbytes, offs)
    del itertools
