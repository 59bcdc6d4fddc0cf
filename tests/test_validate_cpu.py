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


def test_typed_validation_matches_reference_golden_table(golden):
    """Element types and compute modes: every type triple under every mode, byte-exact
    bounds per element size, invalid enumerators (reference planner.cpp:785-859)."""
    names = golden["problem_error_names"]
    for c in golden["validation_typed"]:
        err, op = device.validate_typed(c["m"], c["n"], c["k"], c["op_a"], c["op_b"], c["ids"],
                                        c["bytes"], c["offsets"], c["rows"], c["cols"],
                                        c["lds"], c["types"], c["compute"])
        assert (names[err], op) == (names[c["error"]], c["operand"]), c["name"]


def test_typed_validation_matches_live_reference(ref_lib):
    import ctypes as C
    import random
    if not hasattr(ref_lib, "xr_validate_problem_typed"):
        import pytest
        pytest.skip("reference shim predates the typed entry point")
    ref_lib.xr_validate_problem_typed.argtypes = [C.c_uint64] * 3 + [C.c_int] * 2 + \
        [C.POINTER(C.c_uint64)] * 6 + [C.POINTER(C.c_uint32), C.c_int, C.c_char_p]
    rnd = random.Random(23)
    arr = lambda xs: (C.c_uint64 * 3)(*xs)
    for _ in range(3000):
        m, n, k = (rnd.choice([1, 5, 37]) for _ in range(3))
        oa, ob = rnd.randint(0, 1), rnd.randint(0, 1)
        rows = [m if oa == 0 else k, k if ob == 0 else n, m]
        cols = [k if oa == 0 else m, n if ob == 0 else k, n]
        lds = [r + rnd.choice([0, 0, 3]) for r in rows]
        types = [rnd.choice([0, 1, 2, 3, 2, 2]) for _ in range(3)]
        if rnd.random() < 0.5:
            types[1] = types[0]
        compute = rnd.choice([0, 1, 2])
        esz = [{0: 2, 1: 2, 2: 4, 3: 8}[t] for t in types]
        nbytes = [e * (ld * (c - 1) + r) + rnd.choice([0, 0, -1, 8])
                  for e, ld, c, r in zip(esz, lds, cols, rows)]
        ids = [1, 2, 3]
        offs = [0, 0, 0]
        op = C.create_string_buffer(1)
        want = ref_lib.xr_validate_problem_typed(m, n, k, oa, ob, arr(ids), arr(nbytes),
                                                 arr(offs), arr(rows), arr(cols), arr(lds),
                                                 (C.c_uint32 * 3)(*types), compute, op)
        got, gop = device.validate_typed(m, n, k, oa, ob, ids, nbytes, offs, rows, cols, lds,
                                         types, compute)
        assert (got, gop) == (want, op.value.decode() if op.value else ""), \
            (m, n, k, oa, ob, rows, cols, lds, nbytes, types, compute)
