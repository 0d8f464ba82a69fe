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


# replicate="p2p" on CPU: every rank's C_full is a shared-memory tensor, the
# "peer addresses" are fake (rank << 40 | byte offset) and the fake replicated
# GEMM decodes them to store into the other ranks' shared tensors, as the
# kernel's epilogue stores into the peers' buffers over NVLink.
_FAKE = 1 << 40


class _FakePeerMap:
    def __init__(self, C_full, rank, world):
        self.rank, self.world = rank, world
        self.c_ptr = C_full.data_ptr()
        self.c_bytes = C_full.numel() * C_full.element_size()

    def others(self, off=0):
        return [r * _FAKE + off for r in range(self.world) if r != self.rank]


def _fake_rep(shared, fallback_ranks, rank):
    def rep(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch, sa, sb, sc,
            peers):
        if rank in fallback_ranks:
            return 1                   # VKBLAS_ERR_FALLBACK: nothing computed
        _cpu_gemm(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch, sa, sb,
                  sc)
        for addr in peers:
            r, off = addr // _FAKE, (addr % _FAKE) // 4
            shared[r][off: off + C.numel()].copy_(C)
        return 0
    return rep


def _worker_p2p(rank, world, port, shared):
    """replicate="p2p" host logic: region offsets, the agreement when a rank
    falls back (all gather) or fails (all raise), C_local aliased to C_full
    or separate, with and without a host status group."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import vkblas_b200 as vk
    from vkblas_b200 import shard
    rng = np.random.default_rng(5)
    try:
        M, N, K = 12, 10, 8
        cases = [(7, True, (), None), (8, False, (), dist.group.WORLD), (5, True, (1,), None),
                 (6, False, (0,), dist.group.WORLD), (3, False, (0, 1), None)]
        for batch, aliased, fallback, sg in cases:
            sa, sb, sc = M * K, K * N, M * N
            assert sc * batch <= shared[rank].numel()
            A = rng.uniform(-1, 1, sa * batch).astype(np.float32)
            B = rng.uniform(-1, 1, sb * batch).astype(np.float32)
            C0 = rng.uniform(-1, 1, sc * batch).astype(np.float32)
            want = C0.copy()
            orc.gemm_rowmajor_f32seq(0, 0, M, N, K, 1.25, A, K, B, N, -0.5, want, N, batch, sa, sb,
                                     sc)
            b0, n = shard.batch_shard(batch, rank, world)
            full = shared[rank][: sc * batch]
            full.fill_(float("nan"))
            dist.barrier()
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
                                       C_full=full, gemm_fn=_cpu_gemm, replicate="p2p",
                                       peer_map=_FakePeerMap(full, rank, world),
                                       rep_fn=_fake_rep(shared, fallback, rank), status_group=sg)
            dist.barrier()
            assert np.array_equal(full.numpy(), want), f"rank {rank} batch {batch} {fallback}"
            assert np.array_equal(Cl.numpy(), want[b0 * sc: (b0 + n) * sc])
        m, n, k = 20, 300, 16                 # hipBLAS column-major C(m x n), blocks of 64
        for transB, fallback in ((0, ()), (1, (1,))):
            A = rng.uniform(-1, 1, m * k).astype(np.float32)
            B = rng.uniform(-1, 1, k * n).astype(np.float32)
            ldb = k if transB == 0 else n
            want = np.zeros(m * n, np.float32)
            orc.gemm_rowmajor_f32seq(transB, 0, n, m, k, 1.0, B, ldb, A, m, 0.0, want, m)
            c0, cnt = shard.column_shard(n, rank, world, block=64)
            assert m * n <= shared[rank].numel()
            full = shared[rank][: m * n]
            full.fill_(float("nan"))
            dist.barrier()
            Bc = torch.from_numpy(B[c0 * ldb: (c0 + cnt) * ldb] if transB == 0 else B).clone()
            shard.sharded_column_gemm_hip(0, 0, transB, m, n, k, 1.0, torch.from_numpy(A), m, Bc,
                                          ldb, 0.0, full[c0 * m: (c0 + cnt) * m], m, rank=rank,
                                          world=world, C_full=full, block=64, gemm_fn=_cpu_gemm,
                                          replicate="p2p", peer_map=_FakePeerMap(full, rank, world),
                                          rep_fn=_fake_rep(shared, fallback, rank))
            dist.barrier()
            assert np.array_equal(full.numpy(), want), f"rank {rank} columns transB {transB}"
        # a failing rank: every rank raises, none waits in the rendezvous
        full = shared[rank][: M * N * 2]

        def boom(*args):
            raise vk.VkblasError("injected")
        with pytest.raises(vk.VkblasError):
            shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.0, torch.ones(M * K), K, M * K,
                                       torch.ones(K * N), N, K * N, 0.0,
                                       full[rank * M * N: (rank + 1) * M * N], N, M * N, 2,
                                       rank=rank, world=world, C_full=full, gemm_fn=_cpu_gemm,
                                       replicate="p2p", peer_map=_FakePeerMap(full, rank, world),
                                       rep_fn=boom if rank == 1 else _fake_rep(shared, (), rank))
        # a map built for another buffer is refused before anything runs
        with pytest.raises(ValueError):
            shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.0, torch.ones(M * K), K, M * K,
                                       torch.ones(K * N), N, K * N, 0.0,
                                       full[rank * M * N: (rank + 1) * M * N], N, M * N, 2,
                                       rank=rank, world=world, C_full=full, replicate="p2p",
                                       peer_map=_FakePeerMap(full[1:], rank, world))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["batch", "columns"])
def test_sharded_gemm_two_gloo_ranks(kind):
    mp.spawn(_worker, args=(2, _free_port(), kind), nprocs=2, join=True)


def test_p2p_replication_host_logic_two_gloo_ranks():
    shared = [torch.zeros(8192).share_memory_() for _ in range(2)]
    mp.spawn(_worker_p2p, args=(2, _free_port(), shared), nprocs=2, join=True)
