"""Multi-GPU partitioned SGEMM (include/xvram_b200.h: xvram_b200_shard_*).

One process per GPU.  Rank 0 draws a 128-byte group id, every rank receives it (through
``exchange_unique_id`` over an existing torch.distributed process group, or any other
channel), then each rank creates its ShardGroup with its GPU current and calls
``sgemm`` collectively on its own rows of A and C.
"""
from __future__ import annotations

import ctypes as C

from ._native import lib

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
    def __init__(self, uid: bytes, rank: int, world: int):
        if len(uid) != ID_BYTES:
            raise ValueError("group id must be 128 bytes")
        out = C.c_uint64(0)
        st = lib.xvram_b200_shard_group_create(uid, ID_BYTES, rank, world, C.byref(out))
        if st != 0:
            raise RuntimeError(f"xvram_b200_shard_group_create failed with status {st}")
        self.handle, self.rank, self.world = out.value, rank, world

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
