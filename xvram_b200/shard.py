"""Multi-GPU partitioned SGEMM (include/xvram_b200.h: xvram_b200_shard_*).

One process per GPU.  Rank 0 draws a 128-byte group id, every rank receives it (through
``exchange_unique_id`` over an existing torch.distributed process group, or any other
channel), then each rank creates its ShardGroup with its GPU current and calls
``sgemm`` collectively on its own rows of A and C (``rows`` says which).

``ShardGroup.custom`` makes a group whose collectives are Python callables instead of
NCCL (``xvram_b200_shard_group_create_custom``), e.g. torch.distributed ones.
"""
from __future__ import annotations

import ctypes as C

from ._native import ShardCollectives, ShardPlan, lib


def rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of an m-row C that `rank` owns (xvram_b200_shard_rows)."""
    b0, n = C.c_int64(0), C.c_int64(0)
    st = lib.xvram_b200_shard_rows(m, world, rank, C.byref(b0), C.byref(n))
    if st != 0:
        raise ValueError(f"xvram_b200_shard_rows failed with status {st}")
    return b0.value, n.value


ID_BYTES = 128


def unique_id() -> bytes:
    buf = C.create_string_buffer(ID_BYTES)
    st = lib.xvram_b200_shard_unique_id(buf, ID_BYTES)
    if st != 0:
        raise RuntimeError(f"xvram_b200_shard_unique_id failed with status {st}")
    return buf.raw


def exchange_unique_id(rank: int) -> bytes:
    """Rank 0's id, delivered to every rank of the default torch.distributed group."""
    import torch.distributed as dist
    obj = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def _ptr(x) -> int:
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return x.ctypes.data


class ShardGroup:
    def __init__(self, uid: bytes | None, rank: int, world: int, _ops=None):
        out = C.c_uint64(0)
        self._ops = _ops  # keeps the callbacks alive while the group exists
        if _ops is not None:
            st = lib.xvram_b200_shard_group_create_custom(C.byref(_ops), rank, world,
                                                          C.byref(out))
            what = "xvram_b200_shard_group_create_custom"
        else:
            if uid is None or len(uid) != ID_BYTES:
                raise ValueError("group id must be 128 bytes")
            st = lib.xvram_b200_shard_group_create(uid, ID_BYTES, rank, world, C.byref(out))
            what = "xvram_b200_shard_group_create"
        if st != 0:
            raise RuntimeError(f"{what} failed with status {st}")
        self.handle, self.rank, self.world = out.value, rank, world

    @classmethod
    def custom(cls, rank: int, world: int, all_reduce_max_u64, all_gather_f32) -> "ShardGroup":
        """A group over the caller's collectives.  all_reduce_max_u64(ptr, count, stream)
        and all_gather_f32(send_ptr, recv_ptr, count, stream) receive device addresses
        (host addresses on a host test device) as ints and return 0 on success."""
        # A Python exception cannot cross the C boundary: it becomes a failed collective
        # (XVRAM_STATUS_CUDA_ERROR), which fails the call and poisons the group.
        def _reduce(_ctx, buf, count, stream):
            try:
                return int(all_reduce_max_u64(C.cast(buf, C.c_void_p).value, count, stream) or 0)
            except Exception:  # noqa: BLE001
                return 13

        def _gather(_ctx, send, recv, count, stream):
            try:
                return int(all_gather_f32(C.cast(send, C.c_void_p).value,
                                          C.cast(recv, C.c_void_p).value, count, stream) or 0)
            except Exception:  # noqa: BLE001
                return 13
        ops = ShardCollectives()
        ops.struct_size = C.sizeof(ShardCollectives)
        ops.all_reduce_max_u64 = ShardCollectives.ALL_REDUCE(_reduce)
        ops.all_gather_f32 = ShardCollectives.ALL_GATHER(_gather)
        return cls(None, rank, world, _ops=ops)

    def last_plan(self) -> dict:
        """The agreed plan of the last sgemm call and this rank's copy volumes."""
        info = ShardPlan()
        info.struct_size = C.sizeof(ShardPlan)
        st = lib.xvram_b200_shard_last_plan(self.handle, C.byref(info))
        if st != 0:
            raise RuntimeError(f"xvram_b200_shard_last_plan failed with status {st}")
        return {name: getattr(info, name) for name, _ in ShardPlan._fields_
                if name not in ("struct_size", "reserved0")}

    def sgemm(self, op_a: int, op_b: int, m_local: int, n: int, k: int, alpha: float, a, lda: int,
              b, ldb: int, beta: float, c, ldc: int, panel_k: int = 0) -> int:
        return lib.xvram_b200_sgemm_sharded(self.handle, op_a, op_b, m_local, n, k, alpha, _ptr(a),
                                            lda, _ptr(b), ldb, beta, _ptr(c), ldc, panel_k)

    def allgather_rows(self, block: int, rows: int, cols: int, ld_block: int, dst: int,
                       ld_dst: int, staging: int, staging_bytes: int, stream: int) -> int:
        """xvram_b200_shard_allgather_rows on raw device addresses and a native stream."""
        return lib.xvram_b200_shard_allgather_rows(self.handle, block, rows, cols, ld_block, dst,
                                                   ld_dst, staging, staging_bytes, stream)

    def close(self) -> None:
        if self.handle:
            lib.xvram_b200_shard_group_destroy(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
