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
  issued on the compute stream right after the local GEMM, or (``chunks`` > 1)
  point-to-point gathers of pieces of the shards, each issued on a side stream
  as soon as its piece is computed, so that NVLink traffic overlaps the GEMM.

The local GEMM is the C-ABI engine (``vkblas_b200.gemm`` on device pointers) by
default; ``gemm_fn`` lets CPU tests substitute a host implementation.

Failure handling: when C is replicated, a rank whose local GEMM fails must not
leave its peers waiting in the all-gather.  With ``status_group`` (a gloo group
over the same ranks, host tensors only) every rank first learns, on the host,
whether any rank's local GEMM failed; then either all ranks gather or all raise
``VkblasError``, before any data collective is issued.
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


def _all_ranks_ok(ok: bool, status_group) -> bool:
    """Host-side agreement (MAX of a failure flag over ``status_group``)."""
    import torch
    import torch.distributed as dist
    flag = torch.tensor([0 if ok else 1], dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=status_group)
    return int(flag.item()) == 0


def _local_then_agree(run_local, gathering: bool, status_group):
    """Run this rank's GEMM; when C will be gathered and a status group is
    given, raise on every rank if any rank's GEMM failed."""
    err = None
    try:
        run_local()
    except Exception as exc:         # reported to the peers, then re-raised
        err = exc
    if gathering and status_group is not None and not _all_ranks_ok(err is None, status_group):
        if err is not None:
            raise err
        raise vk.VkblasError("the local GEMM failed on another rank; C was not gathered")
    if err is not None:
        raise err


def _pieces(count: int, n: int):
    """[0, count) cut into n contiguous, nearly equal pieces (some empty when count < n)."""
    return [(count * i // n, count * (i + 1) // n) for i in range(n)]


def _peer(r: int, group):
    import torch.distributed as dist
    return r if group is None else dist.get_global_rank(group, r)


def _gather_piece(C_full, spans, unit: int, rank: int, world: int, group):
    """Point-to-point gather of one piece per rank: spans[r] = (lo, hi) units of
    C_full (``unit`` elements each) that rank r computed; this rank sends its
    span to every other rank and receives theirs in place.  Returns the works."""
    import torch.distributed as dist
    ops = []
    lo, hi = spans[rank]
    if hi > lo:
        mine = C_full[lo * unit: hi * unit]
        ops += [dist.P2POp(dist.isend, mine, _peer(r, group), group)
                for r in range(world) if r != rank]
    for r in range(world):
        l, h = spans[r]
        if r != rank and h > l:
            ops.append(dist.P2POp(dist.irecv, C_full[l * unit: h * unit], _peer(r, group), group))
    return dist.batch_isend_irecv(ops) if ops else []


_side_streams = {}


def _pipelined(run_chunk, starts, counts, chunks: int, C_full, unit: int, rank: int, world: int,
               group, status_group):
    """Replicated C with the gather overlapped: this rank's range is cut into
    ``chunks`` pieces; every piece's GEMM is enqueued on the current stream
    (``run_chunk(lo, hi)``, offsets relative to this rank's start), the ranks
    agree on the host that all GEMMs were enqueued (``status_group``), then the
    gather of piece c is issued on a side stream as soon as an event says piece
    c's GEMM is done, so it crosses NVLink while the next pieces compute.  The
    current stream finally waits for every gather."""
    import torch
    on_gpu = C_full.is_cuda
    mine = _pieces(counts[rank], chunks)
    events = []
    _local_then_agree(lambda: _enqueue_pieces(run_chunk, mine, events, on_gpu), True,
                      status_group)
    works = []
    side = None
    if on_gpu:
        dev = C_full.device
        side = _side_streams.get(dev)
        if side is None:
            side = _side_streams[dev] = torch.cuda.Stream(device=dev)
    for c in range(chunks):
        spans = []
        for r in range(world):
            lo, hi = _pieces(counts[r], chunks)[c]
            spans.append((starts[r] + lo, starts[r] + hi))
        if on_gpu:
            with torch.cuda.stream(side):
                side.wait_event(events[c])
                works += _gather_piece(C_full, spans, unit, rank, world, group)
        else:
            works += _gather_piece(C_full, spans, unit, rank, world, group)
    for w in works:
        w.wait()


def _enqueue_pieces(run_chunk, mine, events, on_gpu):
    import torch
    for lo, hi in mine:
        if hi > lo:
            run_chunk(lo, hi)
        if on_gpu:
            ev = torch.cuda.Event()
            ev.record()
            events.append(ev)


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
                         group=None, C_full=None, gemm_fn: Optional[Callable] = None,
                         status_group=None, chunks: int = 1):
    """Strided-batched GEMM (engine row-major contract) sharded by batch.

    ``A_local``/``B_local``/``C_local`` are flat tensors holding exactly this
    rank's batch entries (``batch_shard(batch, rank, world)``) with strides
    sa/sb/sc (0 = broadcast operand, passed whole to every rank).  When
    ``C_full`` is given, every rank receives all of C: the shards are gathered
    with one all-gather (shards padded to the largest count, sc * count each).
    ``status_group``: see the module docstring.  ``chunks`` > 1 overlaps the
    gather with the GEMM (``_pipelined``): the GEMM writes this rank's region
    of C_full in place (copied to C_local afterwards when that is another
    buffer).  Every rank must pass the same ``chunks``.  Returns (begin, count)."""
    import torch
    begin, count = batch_shard(batch, rank, world)
    fn = gemm_fn or _engine_gemm
    if C_full is not None and chunks > 1:
        if sc < M * ldc:
            raise ValueError("replicated C needs non-overlapping C batches (sc >= M*ldc)")
        plan = [batch_shard(batch, r, world) for r in range(world)]
        region = C_full[begin * sc: (begin + count) * sc]
        aliased = count == 0 or C_local.data_ptr() == region.data_ptr()
        if not aliased and beta != 0.0:
            region.copy_(C_local[: count * sc])

        def run_chunk(lo, hi):
            fn(dtype, op_a, op_b, M, N, K, alpha, A_local[lo * sa:] if sa else A_local, lda,
               B_local[lo * sb:] if sb else B_local, ldb, beta, region[lo * sc:], ldc, hi - lo,
               sa, sb, sc)
        _pipelined(run_chunk, [b for b, _ in plan], [n for _, n in plan], chunks, C_full, sc,
                   rank, world, group, status_group)
        if not aliased:
            C_local[: count * sc].copy_(region)
        return begin, count

    def local():
        if count:
            fn(dtype, op_a, op_b, M, N, K, alpha, A_local, lda, B_local, ldb, beta, C_local, ldc,
               count, sa, sb, sc)
    _local_then_agree(local, C_full is not None, status_group)
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
                            block: int = 256, gemm_fn: Optional[Callable] = None,
                            status_group=None, chunks: int = 1):
    """hipBLAS-convention GEMM C(m x n) = op(A) op(B) split by column blocks of C.

    ``A`` is replicated; ``B_cols`` holds this rank's columns of op(B) (for
    transB == N: columns begin..begin+count of B, i.e. ``count * ldb``
    elements; for transB == T: rows of B, i.e. B + begin with ldb unchanged --
    pass the full B then) and ``C_cols`` this rank's ``count * ldc`` elements
    of C.  ``chunks`` > 1 overlaps the gather with the GEMM, as for
    sharded_batched_gemm.  Engine call: op_a <- transB, op_b <- transA, M <- count, N <- m
    (src/vkblas_hipblas.c:234-239).  Returns (begin, count)."""
    import torch
    begin, count = column_shard(n, rank, world, block)
    fn = gemm_fn or _engine_gemm
    if C_full is not None and chunks > 1:
        plan = [column_shard(n, r, world, block) for r in range(world)]
        region = C_full[begin * ldc: (begin + count) * ldc]
        aliased = count == 0 or C_cols.data_ptr() == region.data_ptr()
        if not aliased and beta != 0.0:
            region.copy_(C_cols[: count * ldc])

        def run_chunk(lo, hi):
            Bv = B_cols[lo * ldb:] if transB == 0 else B_cols[begin + lo:]
            fn(dtype, transB, transA, hi - lo, m, k, alpha, Bv, ldb, A, lda, beta,
               region[lo * ldc:], ldc, 1, 0, 0, 0)
        _pipelined(run_chunk, [c for c, _ in plan], [c for _, c in plan], chunks, C_full, ldc,
                   rank, world, group, status_group)
        if not aliased:
            C_cols[: count * ldc].copy_(region)
        return begin, count

    def local():
        if count:
            Bv = B_cols if transB == 0 else B_cols[begin:]
            fn(dtype, transB, transA, count, m, k, alpha, Bv, ldb, A, lda, beta, C_cols, ldc, 1, 0,
               0, 0)
    _local_then_agree(local, C_full is not None, status_group)
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
