"""Times the SGEMM kernel on device-resident operands (CUDA events, one stream).

    python -m xvram_b200.profile_sgemm --m 8192 --n 6144 --k 4096 --op TN --iters 5
    python -m xvram_b200.profile_sgemm --dtype f64                  # FP64 tensor-core kernel
    python -m xvram_b200.profile_sgemm --dtype f16 --c-dtype f16    # FP16 inputs, FP16 C

Operands come from the library's seeded generator and stay in HBM; each launch is
C = alpha op(A) op(B) + beta C through xvram_b200_sgemm_device (FP32) or
xvram_b200_gemm_device_typed (the other element types, strict FP32 arithmetic for FP16 /
BF16, FP64 for FP64; the launch includes the widening / canonicalising passes).  Prints
one JSON line with the mean launch time and TFLOP/s.  Used for kernel tuning and as the command
under ncu for the summaries in profiles/.
"""
from __future__ import annotations

import argparse
import json


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=6144)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--op", default="TN", choices=["NN", "NT", "TN", "TT"])
    ap.add_argument("--alpha", type=float, default=0.5)
    ap.add_argument("--beta", type=float, default=1.5)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--path", type=int, default=0, help="0 auto, 1 TMA, 2 generic")
    ap.add_argument("--dtype", default="f32", choices=["f32", "f16", "bf16", "f64"])
    ap.add_argument("--c-dtype", default=None, choices=["f32", "f16", "bf16", "f64"],
                    help="C's type (default: f64 for f64 inputs, else f32)")
    a = ap.parse_args()

    import torch

    from xvram_b200 import device as xd

    op_a, op_b = int(a.op[0] == "T"), int(a.op[1] == "T")
    m, n, k = a.m, a.n, a.k
    ra, ca = (k, m) if op_a else (m, k)
    rb, cb = (n, k) if op_b else (k, n)
    host = []
    for seed, (rows, cols) in enumerate(((ra, ca), (rb, cb), (m, n))):
        t = torch.empty((cols, rows), dtype=torch.float32)
        xd.fill_uniform(t, 10 + seed)
        host.append(t)
    types = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16,
             "f64": torch.float64}
    c_dtype = a.c_dtype or ("f64" if a.dtype == "f64" else "f32")
    A, B = (t.to(types[a.dtype]).cuda() for t in host[:2])
    Cd = host[2].to(types[c_dtype]).cuda()
    stream = torch.cuda.Stream()

    def launch():
        if a.dtype == "f32" and c_dtype == "f32":
            st = xd.sgemm(op_a, op_b, m, n, k, a.alpha, A, ra, B, rb, a.beta, Cd, m,
                          stream=stream, path=a.path)
        else:
            st = xd.gemm_typed(op_a, op_b, m, n, k, a.alpha, A, ra, B, rb, a.beta, Cd, m,
                               stream=stream)
        assert st == 0, st

    for _ in range(a.warmup):
        launch()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(a.iters):
            launch()
        e1.record(stream)
    e1.synchronize()
    assert xd.kernel_status(stream) == 0
    ms = e0.elapsed_time(e1) / a.iters
    flop = 2.0 * m * n * k
    print(json.dumps({"m": m, "n": n, "k": k, "op": a.op, "path": a.path, "dtype": a.dtype,
                      "c_dtype": c_dtype, "iters": a.iters, "ms": ms,
                      "tflops": flop / ms / 1e9}))


if __name__ == "__main__":
    main()
