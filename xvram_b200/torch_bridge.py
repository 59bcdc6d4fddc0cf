"""PyTorch tiled-GEMM bridge: `mm` and `linear` on this library's kernels.

The reference routes bias-free `mm` / `linear` of torch graphs whose working set exceeds
the device budget through its native tiled GEMM (reference
python/xvram/torch_native.py:1876-1935, `_submit_tiled_gemm` / `_make_gemm_problem`).
This bridge serves the same two operations, B200-side:

* CUDA tensors run in HBM through `xvram_b200_sgemm_device` (float32) or
  `xvram_b200_gemm_device_typed` (the other types) on torch's current stream.
  Row-major (C-contiguous) and column-major (transposed) views are passed as the matching
  column-major operand and operation, so no copy is made for either.
* Host tensors run out of core through an SDK session (`xvram_get_api`): the operands
  live in page-locked host memory and stream through the session's device budget, as in
  the reference's oversized path.
* `linear` takes a bias and a ReLU (the reference's route refuses biased linear layers,
  torch_native.py:1913-1921); on the GPU they are one pass of `xvram_b200_bias_activation`
  over the output.

Element types are the reference route's (python/xvram/torch_native.py:95-100): float32,
and float16 / bfloat16 / float64 matrices of one type, with the result in that type --
FP16 / BF16 under strict FP32 arithmetic (the products are exact in FP32, the result is
rounded to the type once), FP64 in FP64.  `tensor_cores=True` selects the three-term TF32
kernel for float32 (FP32-accurate within max|err| / (K max|a| max|b|) <= 1e-6); the
default is strict FP32 FFMA.  Bias and ReLU are float32 only (the reference route takes
neither).  There is no CPU fallback: without a GPU every call raises.
"""
from __future__ import annotations

import ctypes
import atexit
import threading

import torch

from . import device as xd
from . import sdk

_TF32X3 = 3
_TYPES = {torch.float16: sdk.FP16, torch.bfloat16: sdk.BF16, torch.float32: sdk.FP32,
          torch.float64: sdk.FP64}


def _dtype_of(a: torch.Tensor, b: torch.Tensor) -> torch.dtype:
    if a.dtype != b.dtype or a.dtype not in _TYPES:
        raise TypeError("mm supports float16, bfloat16, float32 and float64 matrices of one "
                        f"type (got {a.dtype} and {b.dtype})")
    return a.dtype


def _colmajor(x: torch.Tensor):
    """(storage is op(S) of a column-major S, ld, op): a row-major (r, c) tensor is the
    column-major (c, r) matrix transposed."""
    if x.dim() != 2:
        raise ValueError("expected a 2-D tensor")
    r, c = x.shape
    s0, s1 = x.stride()
    if s1 == 1 and s0 >= max(c, 1):
        return x, s0, 1          # row-major: column-major X^T, ld = row stride, op T
    if s0 == 1 and s1 >= max(r, 1):
        return x, s1, 0          # column-major: X itself, op N
    x = x.contiguous()
    return x, max(c, 1), 1


def _check(st: int, what: str) -> None:
    if st != 0:
        raise RuntimeError(f"{what} failed with xvram_status {st}")


def mm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
       tensor_cores: bool = False) -> torch.Tensor:
    """a @ b for (m x k) @ (k x n) matrices of one floating type, on the device the
    tensors are on; the result has that type."""
    dtype = _dtype_of(a, b)
    if tensor_cores and dtype != torch.float32:
        raise TypeError("tensor_cores applies to float32 matrices")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"shapes {tuple(a.shape)} and {tuple(b.shape)} do not multiply")
    if a.device != b.device:
        raise ValueError("a and b must be on the same device")
    if a.device.type != "cuda":
        return _host_session().mm(a, b, out, tensor_cores)
    m, k = a.shape
    n = b.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=dtype, device=a.device)
    elif out.shape != (m, n) or not out.is_contiguous() or out.dtype != dtype:
        raise ValueError(f"out must be a contiguous {dtype} (m, n) tensor")
    if m == 0 or n == 0:
        return out
    if k == 0:
        return out.zero_()
    # Row-major C (m x n) is column-major C^T (n x m) = op(B)^T op(A)^T.
    bs, ldb, ob = _colmajor(b)       # b as op_b(S_b): b = S_b^T when ob == 1
    as_, lda, oa = _colmajor(a)
    # C^T = b^T a^T: the first operand is b^T = op(S_b) with the operation flipped, etc.
    if dtype == torch.float32:
        st = xd.sgemm(1 - ob, 1 - oa, n, m, k, 1.0, bs, ldb, as_, lda, 0.0, out, n,
                      path=_TF32X3 if tensor_cores else 0)
        _check(st, "xvram_b200_sgemm_device")
    else:
        st = xd.gemm_typed(1 - ob, 1 - oa, n, m, k, 1.0, bs, ldb, as_, lda, 0.0, out, n)
        _check(st, "xvram_b200_gemm_device_typed")
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           relu: bool = False, tensor_cores: bool = False) -> torch.Tensor:
    """x @ weight^T (+ bias) (then ReLU), x: (batch, in), weight: (out, in)."""
    if (bias is not None or relu) and x.dtype != torch.float32:
        raise TypeError("bias and ReLU apply to float32 matrices")
    if x.device.type != "cuda":
        return _host_session().linear(x, weight, bias, relu, tensor_cores)
    y = mm(x, weight.t(), tensor_cores=tensor_cores)
    if bias is not None or relu:
        if bias is not None and (bias.dtype != torch.float32 or bias.numel() != y.shape[1]):
            raise ValueError("bias must be float32 with one value per output feature")
        b = bias.contiguous() if bias is not None else None
        # y is row-major (batch, out) = column-major (out, batch): bias runs along rows.
        st = xd.bias_activation(y, y.shape[1], y.shape[1], y.shape[0], b, relu)
        _check(st, "xvram_b200_bias_activation")
    return y


class HostGemm:
    """Out-of-core mm / linear for host tensors through one SDK session.

    Every call uploads its operands into session allocations (page-locked host backing
    when they do not fit the budget), runs one GEMM plan (and, for linear, one bias/ReLU
    transaction) and reads the result back.  `budget_bytes` caps the session's device
    memory (0 = free memory minus headroom)."""

    def __init__(self, budget_bytes: int = 0, device_ordinal: int | None = None):
        ordinal = torch.cuda.current_device() if device_ordinal is None else device_ordinal
        # Budgets below a few GiB get 2 MiB frames (the VMM granularity) so they still
        # hold enough frames for a panel schedule; larger ones keep 64 MiB frames.
        chunk = (2 << 20) if 0 < budget_bytes < (4 << 30) else (64 << 20)
        self.s = sdk.Sdk(sdk.session_config(cache_target_bytes=budget_bytes,
                                            device_ordinal=ordinal, chunk_size_bytes=chunk))
        self.lock = threading.Lock()

    def close(self) -> None:
        self.s.close()

    def _upload(self, t: torch.Tensor):
        t = t.contiguous()
        alloc = self.s.alloc(max(t.numel() * t.element_size(), 4))
        if t.numel():
            alloc.write(t)
        return alloc

    def mm(self, a, b, out=None, tensor_cores=False, b_transposed=False, bias=None,
           relu=False):
        """Row-major a (m x k) @ b (k x n), or a @ b^T for b (n x k) when b_transposed."""
        dtype = _dtype_of(a, b)
        if (tensor_cores or bias is not None or relu) and dtype != torch.float32:
            raise TypeError("tensor_cores, bias and ReLU apply to float32 matrices")
        dt = _TYPES[dtype]
        m, k = a.shape
        n = b.shape[0] if b_transposed else b.shape[1]
        if (b.shape[1] if b_transposed else b.shape[0]) != k:
            raise ValueError(f"shapes {tuple(a.shape)} and {tuple(b.shape)} do not multiply")
        if out is None:
            out = torch.empty((m, n), dtype=dtype)
        if m == 0 or n == 0:
            return out
        if k == 0:
            raise ValueError("the out-of-core path needs k > 0 (no host-side arithmetic)")
        with self.lock:
            A, B = self._upload(a), self._upload(b)
            C = self.s.alloc(max(m * n * a.element_size(), 4))
            allocs = [A, B, C]
            try:
                mode = (sdk.COMPUTE_FP64 if dt == sdk.FP64 else
                        sdk.COMPUTE_FP32_TF32 if tensor_cores else sdk.COMPUTE_FP32_STRICT)
                if b_transposed:  # b is (n x k) row-major; op(B) = T
                    bdesc = sdk.matrix(B, n, k, k, sdk.ROW_MAJOR, data_type=dt)
                else:
                    bdesc = sdk.matrix(B, k, n, n, sdk.ROW_MAJOR, data_type=dt)
                desc = self.s.gemm_desc(sdk.matrix(A, m, k, k, sdk.ROW_MAJOR, data_type=dt),
                                        bdesc, sdk.matrix(C, m, n, n, sdk.ROW_MAJOR, data_type=dt),
                                        sdk.OP_N, sdk.OP_T if b_transposed else sdk.OP_N,
                                        mode=mode)
                plan = self.s.plan(desc)
                try:
                    self.s.check("gemm_execute", self.s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
                finally:
                    self.s.t.gemm_plan_release(plan)
                if bias is not None or relu:
                    Bias = self._upload(bias.to(torch.float32)) if bias is not None else None
                    if Bias is not None:
                        allocs.append(Bias)
                    spec = [(C, 0, m * n * 4, sdk.READ_WRITE)]
                    if Bias is not None:
                        spec.append((Bias, 0, n * 4, sdk.READ))

                    def body(ctx):
                        y = ctx.ranges[0].device_address
                        bptr = ctx.ranges[1].device_address if Bias is not None else 0
                        # row-major (m, n) = column-major (n, m): n features x m rows
                        return sdk.bias_activation(y, n, n, m, bptr, relu, ctx.native_stream)
                    d = self.s.transaction_desc(spec, body)
                    self.s.check("transaction_execute",
                                 self.s.t.transaction_execute(self.s.session, ctypes.byref(d),
                                                              sdk.TIMEOUT_INFINITE))
                C.read(out)
                return out
            finally:
                for x in allocs:
                    x.release()

    def linear(self, x, weight, bias=None, relu=False, tensor_cores=False):
        return self.mm(x, weight, tensor_cores=tensor_cores, b_transposed=True, bias=bias,
                       relu=relu)


_host = None
_host_lock = threading.Lock()


def _close_host_session() -> None:
    """Closes the host-tensor session at interpreter exit, before the CUDA runtime's own
    teardown (its worker and budget sampler must not outlive the device)."""
    global _host
    with _host_lock:
        if _host is not None:
            _host.close()
            _host = None


atexit.register(_close_host_session)


def _host_session() -> HostGemm:
    global _host
    if not torch.cuda.is_available():
        raise RuntimeError("xvram_b200.torch_bridge needs a CUDA device (there is no CPU path)")
    with _host_lock:
        if _host is None:
            _host = HostGemm()
        return _host


def set_host_budget(budget_bytes: int) -> None:
    """Re-open the host-tensor session with a device budget (bytes; 0 = automatic)."""
    global _host
    with _host_lock:
        if _host is not None:
            _host.close()
        _host = HostGemm(budget_bytes)
