"""Multi-GPU sharding of strided-batched and very large GEMMs.

One process per GPU (``torch.distributed``, NCCL over NVLink/NVSwitch on B200
boxes, gloo for CPU tests).  The reference has no multi-GPU code; this follows
the plan its hot path admits:

* strided-batched GEMM: rank r computes the contiguous batch range
  ``vkblas_shard_range(batch, r, world)``; its A/B/C shards are resident on
  its own GPU, so the data path has no collective;
* a very large GEMM: rank r computes a contiguous block of C's columns
  (hipBLAS column-major C, so the block is contiguous in memory) from the
  replicated op(A) and its own columns of op(B);
* replicated C is optional: one ``all_gather_into_tensor`` of the C shards,
  issued on the compute stream right after the local GEMM.

The local GEMM is the C-ABI engine (``vkblas_b200.gemm`` on device pointers) by
default; ``gemm_fn`` lets CPU tests substitute a host implementation.
"""
from __future__ import annotations

from typing import Callable, Optional

import vkblas_b200 as vk


def batch_shard(batch: int, rank: int, world: int):
    """(begin, count) of this rank's batch entries."""
    return vk.shard_range(batch, rank, world, 1)


def column_shard(n: int, rank: int, world: int, block: int = 256):
    """(begin, count) of this rank's columns of C, in whole blocks of ``block`` columns."""
    return vk.shard_range(n, rank, world, block)


def _all_gather_flat(out, shard, world, group=None):
    """out[r*len(shard):(r+1)*len(shard)] = rank r's shard (NCCL: one fused all-gather)."""
    import torch.distributed as dist
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, shard, group=group)
    else:
        parts = list(out.chunk(world))
        dist.all_gather(parts, shard, group=group)


def _engine_gemm(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch, sa, sb, sc):
    import torch
    vk.set_stream(torch.cuda.current_stream())
    st = vk.gemm(dtype, op_a, op_b, M, N, K, alpha, A.data_ptr(), lda, B.data_ptr(), ldb, beta,
                 C.data_ptr(), ldc, batch, sa, sb, sc)
    if st != vk.VKBLAS_OK:
        raise vk.VkblasError(f"vkblas gemm status {st}")


def sharded_batched_gemm(dtype: int, op_a: int, op_b: int, M: int, N: int, K: int, alpha: float,
                         A_local, lda: int, sa: int, B_local, ldb: int, sb: int, beta: float,
                         C_local, ldc: int, sc: int, batch: int, *, rank: int, world: int,
                         group=None, C_full=None, gemm_fn: Optional[Callable] = None):
    """Strided-batched GEMM (engine row-major contract) sharded by batch.

    ``A_local``/``B_local``/``C_local`` are flat tensors holding exactly this
    rank's batch entries (``batch_shard(batch, rank, world)``) with strides
    sa/sb/sc (0 = broadcast operand, passed whole to every rank).  When
    ``C_full`` is given, every rank receives all of C: the shards are gathered
    with one all-gather (shards padded to the largest count, sc * count each).
    Returns (begin, count)."""
    import torch
    begin, count = batch_shard(batch, rank, world)
    fn = gemm_fn or _engine_gemm
    if count:
        fn(dtype, op_a, op_b, M, N, K, alpha, A_local, lda, B_local, ldb, beta, C_local, ldc,
           count, sa, sb, sc)
    if C_full is not None:
        if sc < M * ldc:
            raise ValueError("replicated C needs non-overlapping C batches (sc >= M*ldc)")
        per = max(batch_shard(batch, r, world)[1] for r in range(world))
        if batch % world == 0:
            # Equal shards: gather straight into C_full (in place when C_local is
            # this rank's slice of C_full, as NCCL's in-place all-gather expects).
            _all_gather_flat(C_full[: batch * sc], C_local[: count * sc], world, group)
            return begin, count
        shard = torch.zeros(per * sc, dtype=C_local.dtype, device=C_local.device)
        if count:
            shard[: count * sc].copy_(C_local[: count * sc])
        out = torch.empty(world * per * sc, dtype=C_local.dtype, device=C_local.device)
        _all_gather_flat(out, shard, world, group)
        for r in range(world):
            b0, n = batch_shard(batch, r, world)
            if n:
                C_full[b0 * sc: (b0 + n) * sc].copy_(out[r * per * sc: r * per * sc + n * sc])
    return begin, count


def sharded_column_gemm_hip(dtype: int, transA: int, transB: int, m: int, n: int, k: int,
                            alpha: float, A, lda: int, B_cols, ldb: int, beta: float, C_cols,
                            ldc: int, *, rank: int, world: int, group=None, C_full=None,
                            block: int = 256, gemm_fn: Optional[Callable] = None):
    """hipBLAS-convention GEMM C(m x n) = op(A) op(B) split by column blocks of C.

    ``A`` is replicated; ``B_cols`` holds this rank's columns of op(B) (for
    transB == N: columns begin..begin+count of B, i.e. ``count * ldb``
    elements; for transB == T: rows of B, i.e. B + begin with ldb unchanged --
    pass the full B then) and ``C_cols`` this rank's ``count * ldc`` elements
    of C.  Engine call: op_a <- transB, op_b <- transA, M <- count, N <- m
    (src/vkblas_hipblas.c:234-239).  Returns (begin, count)."""
    import torch
    begin, count = column_shard(n, rank, world, block)
    fn = gemm_fn or _engine_gemm
    if count:
        Bv = B_cols if transB == 0 else B_cols[begin:]
        fn(dtype, transB, transA, count, m, k, alpha, Bv, ldb, A, lda, beta, C_cols, ldc, 1, 0, 0, 0)
    if C_full is not None:
        per = max(column_shard(n, r, world, block)[1] for r in range(world))
        shard = torch.zeros(per * ldc, dtype=C_cols.dtype, device=C_cols.device)
        if count:
            shard[: count * ldc].copy_(C_cols[: count * ldc])
        out = torch.empty(world * per * ldc, dtype=C_cols.dtype, device=C_cols.device)
        _all_gather_flat(out, shard, world, group)
        for r in range(world):
            c0, c = column_shard(n, r, world, block)
            if c:
                C_full[c0 * ldc: (c0 + c) * ldc].copy_(out[r * per * ldc: r * per * ldc + c * ldc])
    return begin, count
