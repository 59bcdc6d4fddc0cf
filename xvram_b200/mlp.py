"""Static-shape FP32 MLP inference through the SDK (include/xvram.h): Linear + bias + ReLU
layers whose weights live in host memory and stream through the session's device budget.

Each layer is one GEMM plan (strict FP32 on the sm_100a kernel) plus one transaction whose
callback runs the library's bias + ReLU kernel on the resident output; the next layer's
weight is prefetched before the current GEMM is submitted, so its upload overlaps the
current layer's compute.  The reference's tiled GEMM takes no bias and its torch route
rejects biased linear layers (reference python/xvram/torch_native.py:1913-1921): this is
the SDK-level composition its transaction API (reference include/xvram/xvram.h:217-252)
allows.

Layouts: activations are column-major features x batch (the same bytes as row-major
batch x features); weights are column-major out x in, so the GEMM is op(A) = N.
"""
from __future__ import annotations

import ctypes as C

from . import sdk


class StreamedMLP:
    def __init__(self, session: "sdk.Sdk", features: int, batch: int, layers: int):
        self.s, self.F, self.B, self.L = session, features, batch, layers
        self.wbytes = features * features * 4
        self.abytes = features * batch * 4
        self.W = [session.alloc(self.wbytes) for _ in range(layers)]
        self.bias = session.alloc(layers * features * 4)
        self.H = [session.alloc(self.abytes), session.alloc(self.abytes)]
        self.statuses: list[int] = []
        F, Bt = features, batch
        self.plans = []
        for i in range(layers):
            src, dst = self.H[i % 2], self.H[(i + 1) % 2]
            d = session.gemm_desc(sdk.matrix(self.W[i], F, F, F), sdk.matrix(src, F, Bt, F),
                                  sdk.matrix(dst, F, Bt, F), sdk.OP_N, sdk.OP_N,
                                  mode=sdk.COMPUTE_FP32_STRICT)
            self.plans.append(session.plan(d))
        self.txns = [session.transaction_desc(
            [(self.H[(i + 1) % 2], 0, self.abytes, sdk.READ_WRITE),
             (self.bias, i * F * 4, F * 4, sdk.READ)], self._body()) for i in range(layers)]
        self.prefetches = [session.prefetch_desc([(w, 0, self.wbytes, sdk.READ)]) for w in self.W]

    def _body(self):
        F, Bt = self.F, self.B

        def body(ctx):
            y, b = ctx.ranges[0], ctx.ranges[1]
            st = sdk.bias_activation(y.device_address, F, F, Bt, b.device_address, True,
                                     ctx.native_stream)
            self.statuses.append(st)
            return st
        return body

    def load_weight(self, i: int, host_col_major) -> None:
        """Weight i as F x F column-major FP32 (out x in) from host memory."""
        self.W[i].write(host_col_major)

    def load_biases(self, host) -> None:
        """All biases, layer after layer (layers x F floats)."""
        self.bias.write(host)

    def forward(self, x_host, out_host) -> None:
        """x_host, out_host: batch x F row-major FP32 host buffers (pinned for speed)."""
        s = self.s
        self.H[0].write(x_host)
        ops = []

        def submit(fn, *args):
            op = C.c_void_p()
            s.check(fn, getattr(s.t, fn)(*args, C.byref(op)))
            ops.append(op.value)
        submit("prefetch_submit", s.session, C.byref(self.prefetches[0]))
        for i in range(self.L):
            if i + 1 < self.L:
                submit("prefetch_submit", s.session, C.byref(self.prefetches[i + 1]))
            submit("gemm_submit", self.plans[i])
            submit("transaction_submit", s.session, C.byref(self.txns[i]))
        failure = None
        for op in ops:
            info = s.wait(op)
            if info.result != sdk.SUCCESS and failure is None:
                failure = sdk.SdkError("MLP layer operation", info.result, s.op_error(op))
            s.t.operation_release(op)
        if failure is not None:
            raise failure
        self.H[self.L % 2].read(out_host)

    def close(self) -> None:
        for p in self.plans:
            self.s.t.gemm_plan_release(p)
        self.plans = []


class ShardedMLP:
    """The same MLP over the ranks of a ShardGroup (one process per GPU), each layer split
    by output features: rank r holds rows [r F/P, (r + 1) F/P) of every weight (and its
    bias slice) in host memory and streams only those through its own session, computes
    its rows of Y = W X, applies bias + ReLU, and the row blocks are all-gathered over
    NVLink into every rank's next activation (xvram_b200_shard_allgather_rows).  Host
    traffic per rank per forward is 1/P of the weights; the exchange is F x B floats per
    layer.  Collective: every rank calls forward with the same input."""

    def __init__(self, session: "sdk.Sdk", group, features: int, batch: int, layers: int):
        P, r = group.world, group.rank
        if features % P:
            raise ValueError("features must divide evenly over the ranks")
        self.s, self.g, self.F, self.B, self.L = session, group, features, batch, layers
        self.Fr = features // P
        self.wbytes = self.Fr * features * 4
        self.abytes = features * batch * 4
        self.ybytes = self.Fr * batch * 4
        self.W = [session.alloc(self.wbytes) for _ in range(layers)]
        self.bias = session.alloc(layers * self.Fr * 4)
        self.H = [session.alloc(self.abytes), session.alloc(self.abytes)]
        self.Y = session.alloc(self.ybytes)
        self.statuses: list[int] = []
        F, Fr, Bt = features, self.Fr, batch
        self.plans = []
        for i in range(layers):
            d = session.gemm_desc(sdk.matrix(self.W[i], Fr, F, Fr),
                                  sdk.matrix(self.H[i % 2], F, Bt, F),
                                  sdk.matrix(self.Y, Fr, Bt, Fr), sdk.OP_N, sdk.OP_N,
                                  mode=sdk.COMPUTE_FP32_STRICT)
            self.plans.append(session.plan(d))
        self.txns = [session.transaction_desc(
            [(self.Y, 0, self.ybytes, sdk.READ_WRITE),
             (self.bias, i * Fr * 4, Fr * 4, sdk.READ),
             (self.H[(i + 1) % 2], 0, self.abytes, sdk.WRITE_ONLY)],
            self._body(), workspace_bytes=self.abytes) for i in range(layers)]
        self.prefetches = [session.prefetch_desc([(w, 0, self.wbytes, sdk.READ)]) for w in self.W]

    def _body(self):
        F, Fr, Bt, g = self.F, self.Fr, self.B, self.g

        def body(ctx):
            y, b, h = ctx.ranges[0], ctx.ranges[1], ctx.ranges[2]
            st = sdk.bias_activation(y.device_address, Fr, Fr, Bt, b.device_address, True,
                                     ctx.native_stream)
            if st == sdk.SUCCESS:
                st = g.allgather_rows(y.device_address, Fr, Bt, Fr, h.device_address, F,
                                      ctx.workspace_device_address, ctx.workspace_bytes,
                                      ctx.native_stream)
            self.statuses.append(st)
            return st
        return body

    def load_weight(self, i: int, host_rows) -> None:
        """This rank's rows of weight i: an (F / P) x F column-major FP32 block (out x in)."""
        self.W[i].write(host_rows)

    def load_biases(self, host) -> None:
        """This rank's bias slices, layer after layer (layers x F / P floats)."""
        self.bias.write(host)

    def forward(self, x_host, out_host) -> None:
        """x_host, out_host: batch x F row-major FP32 host buffers (the whole activation on
        every rank)."""
        s = self.s
        self.H[0].write(x_host)
        ops = []

        def submit(fn, *args):
            op = C.c_void_p()
            s.check(fn, getattr(s.t, fn)(*args, C.byref(op)))
            ops.append(op.value)
        submit("prefetch_submit", s.session, C.byref(self.prefetches[0]))
        for i in range(self.L):
            if i + 1 < self.L:
                submit("prefetch_submit", s.session, C.byref(self.prefetches[i + 1]))
            submit("gemm_submit", self.plans[i])
            submit("transaction_submit", s.session, C.byref(self.txns[i]))
        failure = None
        for op in ops:
            info = s.wait(op)
            if info.result != sdk.SUCCESS and failure is None:
                failure = sdk.SdkError("sharded MLP layer operation", info.result,
                                       s.op_error(op))
            s.t.operation_release(op)
        if failure is not None:
            raise failure
        self.H[self.L % 2].read(out_host)

    def close(self) -> None:
        for p in self.plans:
            self.s.t.gemm_plan_release(p)
        self.plans = []
