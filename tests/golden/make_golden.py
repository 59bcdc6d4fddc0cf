#!/usr/bin/env python3
"""Generate tests/golden/reference_vectors.json from the reference's own CPU code.

Run in a container that has the reference sources:

    make -C oracle ref && python tests/golden/make_golden.py

The values come from oracle/_ref/libxvram_ref.so, which oracle/Makefile compiles
from the reference's src/compat_bench/pattern.cpp, src/gemm_bench/pattern.cpp,
src/gemm/planner.cpp and src/residency/core.cpp (read in place, never copied).
The committed JSON lets the CPU tests pin the C oracle on machines without the
reference tree.  Floats are stored as IEEE-754 bit patterns (hex) so the check
is bit-exact.
"""
from __future__ import annotations

import ctypes as C
import json
import struct
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
REF = ROOT / "oracle" / "_ref" / "libxvram_ref.so"
OUT = Path(__file__).resolve().parent / "reference_vectors.json"

u64 = C.c_uint64


def f32hex(x: float) -> str:
    return struct.pack("<f", x).hex()


def f64hex(x: float) -> str:
    return struct.pack("<d", x).hex()


def load():
    lib = C.CDLL(str(REF))
    lib.xr_cb_pattern_a.argtypes = [u64, u64, u64]
    lib.xr_cb_pattern_a.restype = C.c_float
    lib.xr_cb_pattern_b.argtypes = [u64, u64, u64]
    lib.xr_cb_pattern_b.restype = C.c_float
    lib.xr_cb_pattern_c.argtypes = [u64, u64]
    lib.xr_cb_pattern_c.restype = C.c_float
    lib.xr_cb_reference_dot.argtypes = [u64, u64, u64, u64, C.c_int]
    lib.xr_cb_reference_dot.restype = C.c_double
    lib.xr_cb_reference_result.argtypes = [u64, u64, u64, u64, u64, u64, C.c_float, C.c_float,
                                           C.c_uint32, C.c_int]
    lib.xr_cb_reference_result.restype = C.c_double
    lib.xr_cb_fill_pattern.argtypes = [C.POINTER(C.c_float), u64, u64, u64, u64, u64, u64, u64,
                                       C.c_int, C.c_int, C.c_int, u64]
    lib.xr_cb_fill_pattern.restype = C.c_int
    lib.xr_cb_padding_value.restype = C.c_float
    lib.xr_gb_a.argtypes = [u64, u64]
    lib.xr_gb_a.restype = u64
    lib.xr_gb_b.argtypes = [u64, u64]
    lib.xr_gb_b.restype = u64
    lib.xr_gb_expected.argtypes = [u64, u64, u64, C.POINTER(u64)]
    lib.xr_gb_expected.restype = C.c_int
    lib.xr_validate_problem.argtypes = [u64, u64, u64, C.c_int, C.c_int] + [C.POINTER(u64)] * 6 + [
        C.c_char_p]
    lib.xr_validate_problem.restype = C.c_int
    lib.xr_validate_problem_typed.argtypes = [u64, u64, u64, C.c_int, C.c_int] + \
        [C.POINTER(u64)] * 6 + [C.POINTER(C.c_uint32), C.c_int, C.c_char_p]
    lib.xr_validate_problem_typed.restype = C.c_int
    return lib


# Padded suite of the reference's hardware gate: 37x19x67, padding 5, offset 11,
# NN/NT/TN/TT (src/compat_bench/executor.cpp:208-213).
PADDED = dict(m=37, n=19, k=67, padding=5, offset=11)
SEEDS = [0, 1, 2, 0x1234, 0x300, 0xFFFFFFFFFFFF]


def storage_elements(m, n, k, padding, offset, ta, tb, operand):
    if operand == 0:
        rows, cols = (k, m) if ta else (m, k)
    elif operand == 1:
        rows, cols = (n, k) if tb else (k, n)
    else:
        rows, cols = m, n
    ld = rows + padding
    return ld * cols + offset + offset, ld


def validation_cases():
    """(name, m, n, k, op_a, op_b, ids, bytes, offsets, rows, cols, lds)."""
    cases = []
    big = 1 << 40

    def case(name, m, n, k, oa, ob, ids, nbytes, offs, rows, cols, lds):
        cases.append(dict(name=name, m=m, n=n, k=k, op_a=oa, op_b=ob, ids=ids, bytes=nbytes,
                          offsets=offs, rows=rows, cols=cols, lds=lds))

    sz = lambda r, c, ld: 4 * (ld * (c - 1) + r)
    m, n, k = 37, 19, 67
    ok_b = [sz(m, k, m), sz(k, n, k), sz(m, n, m)]
    case("ok_nn", m, n, k, 0, 0, [1, 2, 3], ok_b, [0, 0, 0], [m, k, m], [k, n, n], [m, k, m])
    case("ok_tt", m, n, k, 1, 1, [1, 2, 3], [sz(k, m, k), sz(n, k, n), sz(m, n, m)], [0, 0, 0],
         [k, n, m], [m, k, n], [k, n, m])
    case("zero_m", 0, n, k, 0, 0, [1, 2, 3], ok_b, [0, 0, 0], [0, k, 0], [k, n, n], [1, k, 1])
    case("zero_k", m, n, 0, 0, 0, [1, 2, 3], ok_b, [0, 0, 0], [m, 0, m], [0, n, n], [m, 1, m])
    case("no_alloc_a", m, n, k, 0, 0, [0, 2, 3], ok_b, [0, 0, 0], [m, k, m], [k, n, n], [m, k, m])
    case("ld_small_a", m, n, k, 0, 0, [1, 2, 3], ok_b, [0, 0, 0], [m, k, m], [k, n, n],
         [m - 1, k, m])
    case("ld_small_c", m, n, k, 0, 0, [1, 2, 3], ok_b, [0, 0, 0], [m, k, m], [k, n, n],
         [m, k, m - 1])
    case("ld_int_limit", m, n, k, 0, 0, [1, 2, 3], [big, big, big], [0, 0, 0], [m, k, m],
         [k, n, n], [1 << 31, k, m])
    case("oob_b", m, n, k, 0, 0, [1, 2, 3], [ok_b[0], ok_b[1] - 4, ok_b[2]], [0, 0, 0],
         [m, k, m], [k, n, n], [m, k, m])
    case("offset_oob", m, n, k, 0, 0, [1, 2, 3], ok_b, [0, 0, ok_b[2]], [m, k, m], [k, n, n],
         [m, k, m])
    case("mismatch", m, n, k, 0, 0, [1, 2, 3], ok_b, [0, 0, 0], [m, k + 1, m], [k, n, n],
         [m, k + 1, m])
    case("mismatch_op", m, n, k, 1, 0, [1, 2, 3], ok_b, [0, 0, 0], [m, k, m], [k, n, n],
         [m, k, m])
    case("alias_c_a", m, n, k, 0, 0, [1, 2, 1], [1 << 20] * 3, [0, 0, 4096], [m, k, m],
         [k, n, n], [m, k, m])
    case("disjoint_same_alloc", m, n, k, 0, 0, [1, 1, 1], [1 << 20] * 3,
         [0, 65536, 262144], [m, k, m], [k, n, n], [m, k, m])
    case("same_id_diff_bytes", m, n, k, 0, 0, [1, 1, 3], [1 << 20, 1 << 21, ok_b[2]],
         [0, 65536, 0], [m, k, m], [k, n, n], [m, k, m])
    case("overflow", m, n, k, 0, 0, [1, 2, 3], [big, big, big], [0, 0, 0], [m, k, m],
         [k, (1 << 62), n], [m, k, m])
    return cases


def typed_validation_cases():
    """Element-type and compute-mode cases: every (A, B, C) type triple over the four types
    under every compute mode on a valid 37 x 19 x 67 NN shape sized for 8-byte elements,
    plus byte-exact bounds per element size and invalid enumerators."""
    cases = []
    m, n, k = 37, 19, 67
    sz = lambda r, c, ld, e: e * (ld * (c - 1) + r)
    big = [sz(m, k, m, 8), sz(k, n, k, 8), sz(m, n, m, 8)]
    base = dict(m=m, n=n, k=k, op_a=0, op_b=0, ids=[1, 2, 3], offsets=[0, 0, 0],
                rows=[m, k, m], cols=[k, n, n], lds=[m, k, m])
    for ta in range(4):
        for tb in range(4):
            for tc in range(4):
                for comp in range(3):
                    cases.append(dict(base, name=f"t{ta}{tb}{tc}_c{comp}", bytes=big,
                                      types=[ta, tb, tc], compute=comp))
    esz = {0: 2, 1: 2, 2: 4, 3: 8}
    for t, comp in ((0, 0), (1, 0), (2, 0), (2, 1), (3, 2)):
        e = esz[t]
        exact = [sz(m, k, m, e), sz(k, n, k, e), sz(m, n, m, e)]
        cases.append(dict(base, name=f"exact_t{t}_c{comp}", bytes=exact, types=[t, t, t], compute=comp))
        short = [exact[0], exact[1] - 1, exact[2]]
        cases.append(dict(base, name=f"short_b_t{t}_c{comp}", bytes=short, types=[t, t, t],
                          compute=comp))
    cases.append(dict(base, name="half_in_f32_out", bytes=big, types=[0, 0, 2], compute=0))
    cases.append(dict(base, name="bf16_in_f32_out", bytes=big, types=[1, 1, 2], compute=0))
    cases.append(dict(base, name="bad_type_a", bytes=big, types=[4, 2, 2], compute=0))
    cases.append(dict(base, name="bad_type_c", bytes=big, types=[2, 2, 7], compute=0))
    cases.append(dict(base, name="bad_compute", bytes=big, types=[2, 2, 2], compute=3))
    cases.append(dict(base, name="mismatch_then_types", bytes=big, types=[0, 2, 2], compute=0,
                      rows=[m, k + 1, m], lds=[m, k + 1, m]))
    return cases


def main() -> None:
    lib = load()
    out: dict = {"source": "oracle/_ref/libxvram_ref.so (reference CPU sources compiled in place)"}

    pat = []
    for seed in SEEDS:
        for row in (0, 1, 2, 3, 5, 17, 1 << 20, (1 << 40) + 7):
            for k in (0, 1, 2, 3, 4, 7, 1 << 33):
                pat.append([seed, row, k, f32hex(lib.xr_cb_pattern_a(row, k, seed)),
                            f32hex(lib.xr_cb_pattern_b(k, row, seed)),
                            f32hex(lib.xr_cb_pattern_c(row, k))])
    out["cb_patterns"] = pat

    dots = []
    for seed in (0, 1, 0x1234, 0x300):
        for row, col in ((0, 0), (1, 2), (5, 3), (36, 18)):
            for k in (1, 2, 3, 4, 5, 67, 1024, 4099):
                dots.append([seed, row, col, k, f64hex(lib.xr_cb_reference_dot(row, col, k, seed, 1)),
                             f64hex(lib.xr_cb_reference_dot(row, col, k, seed, 0))])
    out["cb_dots"] = dots

    res = []
    for seed in (0, 0x1234):
        for alpha, beta in ((1.0, 0.0), (0.5, 1.5), (-2.0, 0.25)):
            for passes in (1, 2):
                for row, col in ((0, 0), (3, 7)):
                    res.append([seed, 37, 19, 67, row, col, alpha, beta, passes,
                                f64hex(lib.xr_cb_reference_result(37, 19, 67, row, col, seed,
                                                                  alpha, beta, passes, 1))])
    out["cb_results"] = res

    fills = []
    for ta in (0, 1):
        for tb in (0, 1):
            for operand in (0, 1, 2):
                count, ld = storage_elements(**PADDED, ta=ta, tb=tb, operand=operand)
                buf = (C.c_float * count)()
                rc = lib.xr_cb_fill_pattern(buf, count, 0, PADDED["m"], PADDED["n"], PADDED["k"],
                                            PADDED["padding"], PADDED["offset"], ta, tb, operand, 0)
                assert rc == 0
                fills.append(dict(ta=ta, tb=tb, operand=operand, ld=ld, count=count,
                                  bits=b"".join(struct.pack("<f", v) for v in buf).hex()))
    out["cb_padded_fills"] = dict(shape=PADDED, padding_value=f32hex(lib.xr_cb_padding_value()),
                                  seed=0, fills=fills)

    gbv = []
    for row in (0, 1, 2, 3, 4, 10, 99):
        for col in (0, 1, 4, 5, 13):
            for k in (1, 2, 3, 5, 6, 7, 64, 4096, 131072, 262147):
                e = u64(0)
                rc = lib.xr_gb_expected(row, col, k, C.byref(e))
                gbv.append([row, col, k, lib.xr_gb_a(row, k), lib.xr_gb_b(k, col),
                            e.value if rc == 0 else None])
    out["gb_expected"] = gbv

    vals = []
    for c in validation_cases():
        arr = lambda xs: (u64 * 3)(*xs)
        op = C.create_string_buffer(1)
        err = lib.xr_validate_problem(c["m"], c["n"], c["k"], c["op_a"], c["op_b"], arr(c["ids"]),
                                      arr(c["bytes"]), arr(c["offsets"]), arr(c["rows"]),
                                      arr(c["cols"]), arr(c["lds"]), op)
        c["error"] = err
        c["operand"] = op.value.decode() if op.value else ""
        vals.append(c)
    out["validation"] = vals

    tvals = []
    for c in typed_validation_cases():
        arr = lambda xs: (u64 * 3)(*xs)
        op = C.create_string_buffer(1)
        err = lib.xr_validate_problem_typed(c["m"], c["n"], c["k"], c["op_a"], c["op_b"],
                                            arr(c["ids"]), arr(c["bytes"]), arr(c["offsets"]),
                                            arr(c["rows"]), arr(c["cols"]), arr(c["lds"]),
                                            (C.c_uint32 * 3)(*c["types"]), c["compute"], op)
        c["error"] = err
        c["operand"] = op.value.decode() if op.value else ""
        tvals.append(c)
    out["validation_typed"] = tvals
    out["problem_error_names"] = [
        "none", "zero_dimension", "invalid_allocation", "invalid_layout", "invalid_operation",
        "invalid_element_type", "invalid_compute_mode", "dimension_mismatch",
        "leading_dimension_too_small", "storage_overflow", "storage_out_of_bounds",
        "unsupported_type_combination", "output_aliases_input", "integer_limit_exceeded"]

    OUT.write_text(json.dumps(out, indent=0, sort_keys=True) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
