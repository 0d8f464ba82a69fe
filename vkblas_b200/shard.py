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
  issued on the compute stream right after the local GEMM
  (``replicate="gather"``), or the fused form (``replicate="p2p"``): the
  tcgen05 GEMM's epilogue stores each finished tile into this rank's C and,
  over NVLink, into every peer's C (``vkblas_b200_gemm_replicated``, buffers
  mapped with CUDA IPC by ``PeerMap``), so the exchange overlaps the math
  tile by tile and the only collective is a one-element all-reduce that
  serves as the rendezvous.

The local GEMM is the C-ABI engine (``vkblas_b200.gemm`` on device pointers) by
default; ``gemm_fn`` lets CPU tests substitute a host implementation.

Failure handling: when C is replicated, a rank whose local GEMM fails must not
leave its peers waiting in the all-gather or the rendezvous.  With ``status_group`` (a gloo group
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


def _all_ranks_ok(ok: bool, status_group, device=None) -> bool:
    """Agreement (MAX of a failure flag over ``status_group``): a host tensor,
    or one on ``device`` when the group is NCCL's."""
    import torch
    import torch.distributed as dist
    flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=device)
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


def _engine_gemm(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch, sa, sb, sc):
    import torch
    vk.set_stream(torch.cuda.current_stream())
    st = vk.gemm(dtype, op_a, op_b, M, N, K, alpha, A.data_ptr(), lda, B.data_ptr(), ldb, beta,
                 C.data_ptr(), ldc, batch, sa, sb, sc)
    if st != vk.VKBLAS_OK:
        raise vk.VkblasError(f"vkblas gemm status {st}")


def _engine_gemm_replicated(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                            batch, sa, sb, sc, peers):
    """vkblas_b200_gemm_replicated on the current stream; returns VKBLAS_OK or
    VKBLAS_ERR_FALLBACK (nothing launched), raises on any other status."""
    import torch
    st = vk.gemm_replicated(dtype, op_a, op_b, M, N, K, alpha, A.data_ptr(), lda, B.data_ptr(),
                            ldb, beta, C.data_ptr(), ldc, peers, batch, sa, sb, sc,
                            stream=torch.cuda.current_stream())
    if st not in (vk.VKBLAS_OK, vk.VKBLAS_ERR_FALLBACK):
        raise vk.VkblasError(f"vkblas replicated gemm status {st}")
    return st


class PeerMap:
    """Every rank's replicated C buffer, mapped into this process (CUDA IPC).

    Built collectively (every rank constructs it for its own ``C_full``, same
    size on all ranks); ``peers[r]`` is the address of rank r's buffer here
    (this rank's own pointer at ``peers[rank]``).  The handles travel as host
    objects over ``exchange_group`` (None: the default group).  A map belongs
    to the buffer it was built for: close it (``close()``, after a barrier so
    that no peer still writes into this rank's buffer) before that buffer is
    freed, since the allocator may hand the same address to another tensor.
    Raises ``VkblasError`` on every rank when any rank could not export or
    open a handle."""

    def __init__(self, C_full, rank: int, world: int, exchange_group=None):
        import torch
        import torch.distributed as dist
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt
        self.rank, self.world = rank, world
        self.c_ptr = C_full.data_ptr()
        self.c_bytes = C_full.numel() * C_full.element_size()
        self.peers = [0] * world
        self._opened = []
        self._rt = rt
        torch.cuda.set_device(C_full.device)
        rt.cudaSetDevice(C_full.device.index)
        mine, err = None, None
        e, base, _ = drv.cuMemGetAddressRange(self.c_ptr)
        if e != drv.CUresult.CUDA_SUCCESS:
            err = f"cuMemGetAddressRange: {e}"
        else:
            e, h = rt.cudaIpcGetMemHandle(int(base))
            if e != rt.cudaError_t.cudaSuccess:
                err = f"cudaIpcGetMemHandle: {e}"
            else:
                mine = (bytes(h.reserved), self.c_ptr - int(base), self.c_bytes)
        objs = [None] * world
        dist.all_gather_object(objs, (mine, err), group=exchange_group)
        bad = [f"rank {r}: {o[1]}" for r, o in enumerate(objs) if o[1] is not None]
        if not bad and any(o[0][2] != self.c_bytes for o in objs):
            bad.append("the replicated C buffers differ in size")
        if bad:
            raise vk.VkblasError("PeerMap: " + "; ".join(bad))
        ok = True
        for r, (obj, _) in enumerate(objs):
            if r == rank:
                self.peers[r] = self.c_ptr
                continue
            hh = rt.cudaIpcMemHandle_t()
            hh.reserved = obj[0]
            e, ptr = rt.cudaIpcOpenMemHandle(hh, rt.cudaIpcMemLazyEnablePeerAccess)
            if e != rt.cudaError_t.cudaSuccess:
                ok = False
                err = f"cudaIpcOpenMemHandle of rank {r}: {e}"
                break
            self._opened.append(int(ptr))
            self.peers[r] = int(ptr) + obj[1]
        on_nccl = dist.get_backend(exchange_group) == "nccl"
        if not _all_ranks_ok(ok, exchange_group, device=C_full.device if on_nccl else None):
            self.close()
            raise vk.VkblasError(f"PeerMap: {err or 'another rank could not open a handle'}")

    def others(self, byte_offset: int = 0):
        """Addresses, in rank order without this rank, of byte ``byte_offset``
        of every other rank's buffer."""
        return [p + byte_offset for r, p in enumerate(self.peers) if r != self.rank]

    def close(self) -> None:
        for ptr in self._opened:
            self._rt.cudaIpcCloseMemHandle(ptr)
        self._opened = []
        self.peers = [0] * self.world


def _replicated(C_full, region, C_local, beta, run_rep, run_plain, gather, peer_map, rank, world,
                group, status_group):
    """Replicated C through the fused P2P epilogue.

    ``region`` is this rank's slice of ``C_full``; run_rep(region, peers) runs
    the replicated GEMM into it (returning VKBLAS_OK or VKBLAS_ERR_FALLBACK),
    run_plain(region) the plain GEMM, gather() the all-gather of every rank's
    region.  The ranks agree on one outcome (MAX of 0 = replicated, 1 = a rank
    fell back, 2 = a rank failed): on 0 a one-element all-reduce on the data
    group is the rendezvous after which every rank's stores have landed; on 1
    the ranks that fell back compute plainly and all gather; on 2 all raise."""
    import torch
    import torch.distributed as dist
    pm = peer_map
    if pm is None or pm.world != world or pm.rank != rank:
        raise ValueError("replicate='p2p' needs the PeerMap of C_full for this rank and world")
    if pm.c_ptr != C_full.data_ptr() or pm.c_bytes != C_full.numel() * C_full.element_size():
        raise ValueError("peer_map was built for another buffer than C_full")
    aliased = region.numel() == 0 or C_local.data_ptr() == region.data_ptr()
    code, err = 0, None
    try:
        if region.numel():
            if not aliased and beta != 0.0:
                region.copy_(C_local[: region.numel()])
            off = region.data_ptr() - C_full.data_ptr()
            if run_rep(region, pm.others(off)) != vk.VKBLAS_OK:
                code = 1
                run_plain(region)
    except Exception as exc:        # reported to the peers, then re-raised
        code, err = 2, exc
    if status_group is not None:
        flag = torch.tensor([code], dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=status_group)
        agreed = int(flag.item())
        if agreed == 0:
            dist.all_reduce(torch.zeros(1, dtype=torch.int32, device=C_full.device), group=group)
    else:
        # Without a host group the agreement travels on the data group: the
        # same all-reduce is the rendezvous (it completes after every rank's
        # GEMM); the host reads it, which waits for the GEMMs.
        flag = torch.tensor([code], dtype=torch.int32, device=C_full.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
        agreed = int(flag.item())
    if agreed == 2:
        if err is not None:
            raise err
        raise vk.VkblasError("the local GEMM failed on another rank; C was not replicated")
    if agreed == 1:
        gather()
    if not aliased:
        C_local[: region.numel()].copy_(region)


def _gather_batched(C_full, C_local, count, sc, batch, rank, world, group):
    import torch
    per = max(batch_shard(batch, r, world)[1] for r in range(world))
    if batch % world == 0:
        # Equal shards: gather straight into C_full (in place when C_local is
        # this rank's slice of C_full, as NCCL's in-place all-gather expects).
        _all_gather_flat(C_full[: batch * sc], C_local[: count * sc], world, group)
        return
    shard = torch.zeros(per * sc, dtype=C_local.dtype, device=C_local.device)
    if count:
        shard[: count * sc].copy_(C_local[: count * sc])
    out = torch.empty(world * per * sc, dtype=C_local.dtype, device=C_local.device)
    _all_gather_flat(out, shard, world, group)
    for r in range(world):
        b0, n = batch_shard(batch, r, world)
        if n:
            C_full[b0 * sc: (b0 + n) * sc].copy_(out[r * per * sc: r * per * sc + n * sc])


def _gather_columns(C_full, C_cols, count, ldc, n, block, rank, world, group):
    import torch
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


def _check_replicate(replicate: str) -> None:
    if replicate not in ("gather", "p2p"):
        raise ValueError(f"replicate must be 'gather' or 'p2p', not {replicate!r}")


def sharded_batched_gemm(dtype: int, op_a: int, op_b: int, M: int, N: int, K: int, alpha: float,
                         A_local, lda: int, sa: int, B_local, ldb: int, sb: int, beta: float,
                         C_local, ldc: int, sc: int, batch: int, *, rank: int, world: int,
                         group=None, C_full=None, gemm_fn: Optional[Callable] = None,
                         status_group=None, replicate: str = "gather", peer_map=None,
                         rep_fn: Optional[Callable] = None):
    """Strided-batched GEMM (engine row-major contract) sharded by batch.

    ``A_local``/``B_local``/``C_local`` are flat tensors holding exactly this
    rank's batch entries (``batch_shard(batch, rank, world)``) with strides
    sa/sb/sc (0 = broadcast operand, passed whole to every rank).  When
    ``C_full`` is given, every rank receives all of C:

    * ``replicate="gather"``: the shards are gathered with one all-gather
      (shards padded to the largest count, sc * count each);
    * ``replicate="p2p"``: the GEMM runs into this rank's region of C_full and
      its epilogue also stores every tile into the other ranks' C_full over
      NVLink (``peer_map``: the ``PeerMap`` of C_full); one one-element
      all-reduce is the rendezvous.  Ranks whose call cannot take that kernel
      compute plainly and then all ranks gather.  C_local receives this
      rank's entries afterwards unless it is the region itself.

    ``status_group``: see the module docstring.  ``gemm_fn`` / ``rep_fn``
    replace the engine's plain / replicated GEMM (CPU tests).  Every rank must
    pass the same ``replicate``.  Returns (begin, count)."""
    _check_replicate(replicate)
    begin, count = batch_shard(batch, rank, world)
    fn = gemm_fn or _engine_gemm
    if C_full is not None and sc < M * ldc:
        raise ValueError("replicated C needs non-overlapping C batches (sc >= M*ldc)")

    def local(Cdst):
        if count:
            fn(dtype, op_a, op_b, M, N, K, alpha, A_local, lda, B_local, ldb, beta, Cdst, ldc,
               count, sa, sb, sc)

    if C_full is not None and replicate == "p2p":
        rfn = rep_fn or _engine_gemm_replicated
        region = C_full[begin * sc: (begin + count) * sc]
        _replicated(C_full, region, C_local, beta,
                    lambda R, peers: rfn(dtype, op_a, op_b, M, N, K, alpha, A_local, lda, B_local,
                                         ldb, beta, R, ldc, count, sa, sb, sc, peers),
                    local,
                    lambda: _gather_batched(C_full, region, count, sc, batch, rank, world, group),
                    peer_map, rank, world, group, status_group)
        return begin, count
    _local_then_agree(lambda: local(C_local), C_full is not None, status_group)
    if C_full is not None:
        _gather_batched(C_full, C_local, count, sc, batch, rank, world, group)
    return begin, count


def sharded_column_gemm_hip(dtype: int, transA: int, transB: int, m: int, n: int, k: int,
                            alpha: float, A, lda: int, B_cols, ldb: int, beta: float, C_cols,
                            ldc: int, *, rank: int, world: int, group=None, C_full=None,
                            block: int = 256, gemm_fn: Optional[Callable] = None,
                            status_group=None, replicate: str = "gather", peer_map=None,
                            rep_fn: Optional[Callable] = None):
    """hipBLAS-convention GEMM C(m x n) = op(A) op(B) split by column blocks of C.

    ``A`` is replicated; ``B_cols`` holds this rank's columns of op(B) (for
    transB == N: columns begin..begin+count of B, i.e. ``count * ldb``
    elements; for transB == T: rows of B, i.e. B + begin with ldb unchanged --
    pass the full B then) and ``C_cols`` this rank's ``count * ldc`` elements
    of C.  ``C_full``, ``replicate`` and ``peer_map`` as for
    sharded_batched_gemm (a rank's columns are one contiguous region of
    column-major C).  Engine call: op_a <- transB, op_b <- transA, M <- count,
    N <- m (src/vkblas_hipblas.c:234-239).  Returns (begin, count)."""
    _check_replicate(replicate)
    begin, count = column_shard(n, rank, world, block)
    fn = gemm_fn or _engine_gemm
    Bv = B_cols if transB == 0 else B_cols[begin:]

    def local(Cdst):
        if count:
            fn(dtype, transB, transA, count, m, k, alpha, Bv, ldb, A, lda, beta, Cdst, ldc, 1, 0,
               0, 0)

    if C_full is not None and replicate == "p2p":
        rfn = rep_fn or _engine_gemm_replicated
        region = C_full[begin * ldc: (begin + count) * ldc]
        _replicated(C_full, region, C_cols, beta,
                    lambda R, peers: rfn(dtype, transB, transA, count, m, k, alpha, Bv, ldb, A,
                                         lda, beta, R, ldc, 1, 0, 0, 0, peers),
                    local,
                    lambda: _gather_columns(C_full, region, count, ldc, n, block, rank, world,
                                            group),
                    peer_map, rank, world, group, status_group)
        return begin, count
    _local_then_agree(lambda: local(C_cols), C_full is not None, status_group)
    if C_full is not None:
        _gather_columns(C_full, C_cols, count, ldc, n, block, rank, world, group)
    return begin, count
