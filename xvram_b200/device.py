"""Native entry points of include/xvram_b200.h for Python callers.

Column-major convention: an ``rows x cols`` column-major matrix with leading
dimension ``ld`` is held in a torch tensor of shape ``(cols, ld)`` (row j of the
tensor is column j of the matrix).  ``colmajor(t)`` / ``from_colmajor`` convert.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

from ._native import PlanInfo, lib

u32, u64 = C.c_uint32, C.c_uint64

PATH_AUTO, PATH_TMA, PATH_GENERIC = 0, 1, 2


def _stream_handle(stream) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def sgemm(op_a: int, op_b: int, m: int, n: int, k: int, alpha: float, a, lda: int, b, ldb: int,
          beta: float, c, ldc: int, stream=None, path: int = PATH_AUTO) -> int:
    """C = alpha op(A) op(B) + beta C on CUDA tensors (or raw device pointers); returns
    the xvram_status.  Enqueued on `stream` (default: torch's current stream)."""
    ptr = lambda x: x if isinstance(x, int) else x.data_ptr()
    return lib.xvram_b200_sgemm_device(op_a, op_b, m, n, k, alpha, ptr(a), lda, ptr(b), ldb, beta,
                                       ptr(c), ldc, _stream_handle(stream), path)


def workspace_bytes(op_a: int, op_b: int, m: int, n: int, k: int) -> int:
    """Scratch the K-major canonicalisation needs (0 for op(A)=N, op(B)=T)."""
    return lib.xvram_b200_sgemm_workspace_bytes(op_a, op_b, m, n, k)


def tile_shape(m: int, n: int) -> tuple[int, int]:
    """The C tile (rows, columns) the TMA kernel uses for an M-/N-major m x n problem on the
    current device: (192, 192), (128, 256) or (128, 128)."""
    import ctypes as C
    tm, tn = C.c_int32(0), C.c_int32(0)
    st = lib.xvram_b200_sgemm_tile_shape(m, n, C.byref(tm), C.byref(tn))
    if st != 0:
        raise ValueError(f"xvram_b200_sgemm_tile_shape failed with status {st}")
    return tm.value, tn.value


def sgemm_ws(op_a: int, op_b: int, m: int, n: int, k: int, alpha: float, a, lda: int, b,
             ldb: int, beta: float, c, ldc: int, workspace, workspace_bytes: int, stream=None,
             path: int = PATH_AUTO) -> int:
    """sgemm with caller-provided device workspace (no allocation inside)."""
    ptr = lambda x: x if isinstance(x, int) else x.data_ptr()
    return lib.xvram_b200_sgemm_device_ws(op_a, op_b, m, n, k, alpha, ptr(a), lda, ptr(b), ldb,
                                          beta, ptr(c), ldc, ptr(workspace), workspace_bytes,
                                          _stream_handle(stream), path)


def bias_activation(y, ldy: int, rows: int, cols: int, bias=None, relu: bool = False,
                    stream=None) -> int:
    """Y = act(Y + bias) on a column-major rows x cols device block (bias: rows floats or
    None); returns the xvram_status.  Enqueued on `stream` (default: torch's current)."""
    ptr = lambda x: 0 if x is None else (x if isinstance(x, int) else x.data_ptr())
    return lib.xvram_b200_bias_activation(ptr(y), ldy, rows, cols, ptr(bias), 1 if relu else 0,
                                          _stream_handle(stream))


def kernel_status(stream=None) -> int:
    """Synchronises the stream and returns (and clears) the kernel error word."""
    w = u32(0)
    st = lib.xvram_b200_kernel_status(_stream_handle(stream), C.byref(w))
    if st != 0:
        raise RuntimeError(f"xvram_b200_kernel_status failed with status {st}")
    return w.value


def fill_uniform(t, seed: int, first_index: int = 0, threads: int = 0) -> None:
    """Fills a contiguous float32 CPU tensor (or numpy array) with the seeded stream."""
    if hasattr(t, "data_ptr"):
        assert t.is_contiguous() and t.dtype.itemsize == 4 and not t.is_cuda
        ptr, count = t.data_ptr(), t.numel()
    else:
        assert t.flags["C_CONTIGUOUS"] and t.dtype.itemsize == 4
        ptr, count = t.ctypes.data, t.size
    lib.xvram_b200_fill_uniform(ptr, count, seed, first_index, threads)


def plan_panels(op_a: int, op_b: int, m: int, n: int, k: int, beta_nonzero: bool, budget: int,
                quantum: int, flops_per_s: float = 0.0, h2d: float = 0.0, d2h: float = 0.0,
                force=(0, 0, 0)) -> dict:
    info = PlanInfo()
    info.struct_size = C.sizeof(PlanInfo)
    st = lib.xvram_b200_plan_panels(op_a, op_b, m, n, k, int(beta_nonzero), budget, quantum,
                                    flops_per_s, h2d, d2h, force[0], force[1], force[2],
                                    C.byref(info))
    out = {name: getattr(info, name) for name, _ in PlanInfo._fields_}
    out["return_status"] = st
    return out


def plan_steps(op_a: int, op_b: int, m: int, n: int, k: int, beta_nonzero: bool, budget: int,
               quantum: int, force=(0, 0, 0), capacity: Optional[int] = None):
    """Step list of the plan as a list of (bm, bn, bk, slot_a, slot_b)."""
    info = plan_panels(op_a, op_b, m, n, k, beta_nonzero, budget, quantum, force=force)
    if info["return_status"] != 0:
        return info["return_status"], []
    cap = info["steps"] if capacity is None else capacity
    buf = (C.c_int32 * (5 * max(cap, 1)))()
    st = lib.xvram_b200_plan_steps(op_a, op_b, m, n, k, int(beta_nonzero), budget, quantum,
                                   force[0], force[1], force[2], buf, cap)
    if st != 0:
        return st, []
    return 0, [tuple(buf[5 * i:5 * i + 5]) for i in range(cap)]


def validate(m, n, k, op_a, op_b, ids, nbytes, offsets, rows, cols, lds) -> tuple[int, str]:
    arr = lambda xs: (u64 * 3)(*xs)
    op = C.create_string_buffer(1)
    err = lib.xvram_b200_validate_gemm(m, n, k, op_a, op_b, arr(ids), arr(nbytes), arr(offsets),
                                       arr(rows), arr(cols), arr(lds), op)
    return err, (op.value.decode() if op.value else "")


def validate_typed(m, n, k, op_a, op_b, ids, nbytes, offsets, rows, cols, lds, types,
                   compute) -> tuple[int, str]:
    arr = lambda xs: (u64 * 3)(*xs)
    op = C.create_string_buffer(1)
    err = lib.xvram_b200_validate_gemm_typed(m, n, k, op_a, op_b, arr(ids), arr(nbytes),
                                             arr(offsets), arr(rows), arr(cols), arr(lds),
                                             (C.c_uint32 * 3)(*types), compute, op)
    return err, (op.value.decode() if op.value else "")


# Element types (XVRAM_DATA_*) and arithmetic (the reference's gemm::ComputeMode order).
FP16, BF16, FP32, FP64 = range(4)
STRICT_FP32, TF32, COMPUTE_FP64 = range(3)
_TORCH_TYPES = {"float16": FP16, "bfloat16": BF16, "float32": FP32, "float64": FP64}


def gemm_typed(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, Cm, ldc, compute=None,
               stream=None) -> int:
    """C = alpha op(A) op(B) + beta C on CUDA tensors of the reference's type combinations
    (types read from the tensors; compute defaults to strict FP32, FP64 for FP64), with a
    workspace allocated here."""
    import torch
    ab = _TORCH_TYPES[str(A.dtype).split(".")[-1]]
    ct = _TORCH_TYPES[str(Cm.dtype).split(".")[-1]]
    if compute is None:
        compute = COMPUTE_FP64 if ab == FP64 else STRICT_FP32
    need = lib.xvram_b200_gemm_typed_workspace_bytes(ab, ct, compute, op_a, op_b, m, n, k)
    ws = torch.empty(need + 256, dtype=torch.uint8, device=A.device) if need else None
    if ws is not None and isinstance(stream, torch.cuda.Stream):
        ws.record_stream(stream)  # freed here, but not reused before the stream's work ends
    wp = ((ws.data_ptr() + 255) // 256 * 256) if ws is not None else 0
    return lib.xvram_b200_gemm_device_typed(ab, ct, compute, op_a, op_b, m, n, k, alpha,
                                            A.data_ptr(), lda, B.data_ptr(), ldb, beta,
                                            Cm.data_ptr(), ldc, wp, need, _stream_handle(stream))


def ffma_probe(blocks: int, iterations: int, sink, stream=None, packed: bool = False) -> int:
    fn = lib.xvram_b200_ffma2_probe if packed else lib.xvram_b200_ffma_probe
    return fn(blocks, iterations, sink.data_ptr(), _stream_handle(stream))
