"""Multi-GPU shard driver, exercised as 2 gloo ranks on CPU (no GPU).

The local GEMM is the oracle's sequential-fmaf GEMM, so the gathered result
must equal the single-process oracle bit for bit: this checks the shard plan
(every batch entry / column block exactly once), the operand offsets and the
all-gather of C."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc


def _cpu_gemm(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch, sa, sb, sc):
    c = C.numpy()
    orc.gemm_rowmajor_f32seq(op_a, op_b, M, N, K, alpha, np.ascontiguousarray(A.numpy()), lda,
                             np.ascontiguousarray(B.numpy()), ldb, beta, c, ldc, batch, sa, sb, sc)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, kind):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from vkblas_b200 import shard
    rng = np.random.default_rng(99)
    try:
        if kind == "batch":
            M, N, K = 24, 20, 16
            # batch 7: uneven shards (padded gather); batch 8: equal shards, C
            # computed in place in this rank's slice of the replicated C
            for batch, bcast in ((7, None), (7, "a"), (8, None)):
                sa = 0 if bcast == "a" else M * K
                sb, sc = K * N, M * N
                A = rng.uniform(-1, 1, (sa * (batch - 1) if sa else 0) + M * K).astype(np.float32)
                B = rng.uniform(-1, 1, sb * batch).astype(np.float32)
                C0 = rng.uniform(-1, 1, sc * batch).astype(np.float32)
                want = C0.copy()
                orc.gemm_rowmajor_f32seq(0, 0, M, N, K, 1.5, A, K, B, N, 0.5, want, N, batch, sa, sb, sc)
                b0, n = shard.batch_shard(batch, rank, world)
                Al = torch.from_numpy(A[b0 * sa: (b0 + n) * sa] if sa else A).clone()
                Bl = torch.from_numpy(B[b0 * sb: (b0 + n) * sb]).clone()
                full = torch.zeros(sc * batch)
                if batch % world == 0:
                    Cl = full[b0 * sc: (b0 + n) * sc]
                    Cl.copy_(torch.from_numpy(C0[b0 * sc: (b0 + n) * sc]))
                else:
                    Cl = torch.from_numpy(C0[b0 * sc: (b0 + n) * sc]).clone()
                shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.5, Al, K, sa, Bl, N, sb, 0.5, Cl, N, sc,
                                           batch, rank=rank, world=world, C_full=full,
                                           gemm_fn=_cpu_gemm)
                assert np.array_equal(full.numpy(), want), f"rank {rank} batch shard mismatch"
        else:
            m, n, k = 40, 1000, 24            # hipBLAS column-major C(m x n)
            for transB in (0, 1):
                A = rng.uniform(-1, 1, m * k).astype(np.float32)           # N: m x k, lda = m
                B = rng.uniform(-1, 1, k * n).astype(np.float32)
                ldb = k if transB == 0 else n
                C0 = rng.uniform(-1, 1, m * n).astype(np.float32)
                want = C0.copy()
                orc.gemm_rowmajor_f32seq(transB, 0, n, m, k, 1.0, B, ldb, A, m, 0.25, want, m)
                c0, cnt = shard.column_shard(n, rank, world, block=64)
                Bc = torch.from_numpy(B[c0 * ldb: (c0 + cnt) * ldb] if transB == 0 else B).clone()
                Cc = torch.from_numpy(C0[c0 * m: (c0 + cnt) * m]).clone()
                full = torch.zeros(m * n)
                shard.sharded_column_gemm_hip(0, 0, transB, m, n, k, 1.0, torch.from_numpy(A), m, Bc,
                                              ldb, 0.25, Cc, m, rank=rank, world=world, C_full=full,
                                              block=64, gemm_fn=_cpu_gemm)
                assert np.array_equal(full.numpy(), want), f"rank {rank} column shard mismatch"
    finally:
        dist.destroy_process_group()


def _worker_pipelined(rank, world, port):
    """chunks > 1: the shards are cut into pieces whose gathers are point-to-point
    sends and receives issued piece by piece (overlapped with the GEMM on a GPU);
    uneven shards, pieces that are empty on some ranks, C_local aliased to
    C_full or a separate buffer."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from vkblas_b200 import shard
    rng = np.random.default_rng(5)
    try:
        M, N, K = 12, 10, 8
        for batch, chunks, aliased in ((7, 3, True), (8, 4, False), (5, 4, True), (3, 4, False)):
            sa, sb, sc = M * K, K * N, M * N
            A = rng.uniform(-1, 1, sa * batch).astype(np.float32)
            B = rng.uniform(-1, 1, sb * batch).astype(np.float32)
            C0 = rng.uniform(-1, 1, sc * batch).astype(np.float32)
            want = C0.copy()
            orc.gemm_rowmajor_f32seq(0, 0, M, N, K, 1.25, A, K, B, N, -0.5, want, N, batch, sa, sb, sc)
            b0, n = shard.batch_shard(batch, rank, world)
            full = torch.zeros(sc * batch)
            mine = torch.from_numpy(C0[b0 * sc: (b0 + n) * sc]).clone()
            if aliased:
                Cl = full[b0 * sc: (b0 + n) * sc]
                Cl.copy_(mine)
            else:
                Cl = mine
            shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.25,
                                       torch.from_numpy(A[b0 * sa: (b0 + n) * sa]).clone(), K, sa,
                                       torch.from_numpy(B[b0 * sb: (b0 + n) * sb]).clone(), N, sb,
                                       -0.5, Cl, N, sc, batch, rank=rank, world=world,
                                       C_full=full, gemm_fn=_cpu_gemm, chunks=chunks,
                                       status_group=dist.group.WORLD)
            assert np.array_equal(full.numpy(), want), f"rank {rank} batch {batch} chunks {chunks}"
            assert np.array_equal(Cl.numpy(), want[b0 * sc: (b0 + n) * sc])
        m, n, k = 20, 300, 16                 # hipBLAS column-major C(m x n), blocks of 64
        for transB in (0, 1):
            A = rng.uniform(-1, 1, m * k).astype(np.float32)
            B = rng.uniform(-1, 1, k * n).astype(np.float32)
            ldb = k if transB == 0 else n
            want = np.zeros(m * n, np.float32)
            orc.gemm_rowmajor_f32seq(transB, 0, n, m, k, 1.0, B, ldb, A, m, 0.0, want, m)
            c0, cnt = shard.column_shard(n, rank, world, block=64)
            full = torch.zeros(m * n)
            Bc = torch.from_numpy(B[c0 * ldb: (c0 + cnt) * ldb] if transB == 0 else B).clone()
            shard.sharded_column_gemm_hip(0, 0, transB, m, n, k, 1.0, torch.from_numpy(A), m, Bc,
                                          ldb, 0.0, full[c0 * m: (c0 + cnt) * m], m, rank=rank,
                                          world=world, C_full=full, block=64, gemm_fn=_cpu_gemm,
                                          chunks=3)
            assert np.array_equal(full.numpy(), want), f"rank {rank} column pieces"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["batch", "columns"])
def test_sharded_gemm_two_gloo_ranks(kind):
    mp.spawn(_worker, args=(2, _free_port(), kind), nprocs=2, join=True)


def test_pipelined_gather_two_gloo_ranks():
    mp.spawn(_worker_pipelined, args=(2, _free_port()), nprocs=2, join=True)
