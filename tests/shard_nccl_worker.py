"""Worker of tests/test_shard_nccl_gpu.py: one rank per GPU over NCCL.

Run under torchrun (2+ GPUs).  Each rank computes its shard with the library
on its own GPU, the shards are gathered with NCCL, and every rank checks the
whole replicated C against the CPU oracle (double precision for the tensor-core
paths, bit for bit for the exact SIMT path):

* batch shards of a strided-batched fp16 GEMM, equal shards (C computed in
  place in this rank's slice of the replicated C, one in-place all-gather)
  and uneven shards (padded gather), plus a broadcast A operand;
* batch shards of an fp32 GEMM on the exact SIMT kernel;
* column blocks of a hipBLAS-convention fp16 GEMM, transB = N and T;
* the pipelined gather (chunks > 1: point-to-point gathers of pieces of the
  shards, issued on a side stream as each piece's GEMM finishes), with the
  ranks' host-side status exchange over a gloo group.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import vkblas_b200 as vk  # noqa: E402
from vkblas_b200 import shard  # noqa: E402
from oracle import oracle as orc  # noqa: E402

STATUS = None        # gloo group for the host-side status exchange (set in main)


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _dev16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.float16)


def check_batch(rank, world, rng):
    M, N, K = 192, 160, 136
    for batch, bcast, chunks in ((4 * world, False, 1), (4 * world + 1, False, 1),
                                 (2 * world, True, 1), (4 * world + 1, False, 3),
                                 (8 * world, True, 4)):
        sa = 0 if bcast else M * K
        sb, sc = K * N, M * N
        A = orc.f2h(rng.uniform(-1, 1, (sa * (batch - 1) if sa else 0) + M * K).astype(np.float32))
        B = orc.f2h(rng.uniform(-1, 1, sb * batch).astype(np.float32))
        want = orc.hgemm_rowmajor_f64(0, 0, 0, M, N, K, 1.0, A, K, B, N, 0.0, None, N, batch, sa,
                                      sb, sc)
        b0, n = shard.batch_shard(batch, rank, world)
        Al = _dev16(A[b0 * sa: (b0 + n) * sa] if sa else A)
        Bl = _dev16(B[b0 * sb: (b0 + n) * sb])
        full = torch.zeros(sc * batch, dtype=torch.float16, device="cuda")
        Cl = (full[b0 * sc: (b0 + n) * sc] if batch % world == 0
              else torch.zeros(n * sc, dtype=torch.float16, device="cuda"))
        shard.sharded_batched_gemm(vk.DT_F16, 0, 0, M, N, K, 1.0, Al, K, sa, Bl, N, sb, 0.0, Cl, N,
                                   sc, batch, rank=rank, world=world, C_full=full, chunks=chunks,
                                   status_group=STATUS)
        torch.cuda.synchronize()
        got = orc.h2f(_u16(full)).reshape(batch, M, N)
        err = orc.rel_frobenius(got, want)
        assert err <= 2e-3, (f"rank {rank}: fp16 batch shard (batch {batch}, chunks {chunks}) "
                             f"relative error {err}")
    # fp32 on the exact SIMT kernel: bit for bit
    M, N, K, batch = 64, 48, 40, 2 * world + 1
    A = rng.uniform(-1, 1, M * K * batch).astype(np.float32)
    B = rng.uniform(-1, 1, K * N * batch).astype(np.float32)
    want = np.zeros(M * N * batch, np.float32)
    orc.gemm_rowmajor_f32seq(0, 0, M, N, K, 1.0, A, K, B, N, 0.0, want, N, batch, M * K, K * N,
                             M * N)
    b0, n = shard.batch_shard(batch, rank, world)
    Al = torch.from_numpy(A[b0 * M * K: (b0 + n) * M * K]).cuda()
    Bl = torch.from_numpy(B[b0 * K * N: (b0 + n) * K * N]).cuda()
    Cl = torch.zeros(n * M * N, device="cuda")
    full = torch.zeros(M * N * batch, device="cuda")
    vk.set_path(vk.PATH_SIMT)
    try:
        shard.sharded_batched_gemm(vk.DT_F32, 0, 0, M, N, K, 1.0, Al, K, M * K, Bl, N, K * N, 0.0,
                                   Cl, N, M * N, batch, rank=rank, world=world, C_full=full)
        torch.cuda.synchronize()
    finally:
        vk.set_path(vk.PATH_AUTO)
    assert np.array_equal(full.cpu().numpy().view(np.uint32), want.view(np.uint32)), \
        f"rank {rank}: fp32 SIMT batch shard not bit-exact"


def check_columns(rank, world, rng):
    m, n, k = 256, 1024 + 96, 192          # hipBLAS column-major C(m x n); ragged last block
    for transB, chunks in ((0, 1), (1, 1), (0, 3)):
        A = orc.f2h(rng.uniform(-1, 1, m * k).astype(np.float32))          # transA = N, lda = m
        B = orc.f2h(rng.uniform(-1, 1, k * n).astype(np.float32))
        ldb = k if transB == 0 else n
        # column-major C = A op(B): the engine call (op_a = transB, op_b = N, M = n, N = m)
        want = orc.hgemm_rowmajor_f64(0, transB, 0, n, m, k, 1.0, B, ldb, A, m, 0.0, None, m)[0]
        c0, cnt = shard.column_shard(n, rank, world, block=128)
        Bc = _dev16(B[c0 * ldb: (c0 + cnt) * ldb] if transB == 0 else B)
        Cc = torch.zeros(max(cnt, 1) * m, dtype=torch.float16, device="cuda")
        full = torch.zeros(m * n, dtype=torch.float16, device="cuda")
        shard.sharded_column_gemm_hip(vk.DT_F16, 0, transB, m, n, k, 1.0, _dev16(A), m, Bc, ldb, 0.0,
                                      Cc, m, rank=rank, world=world, C_full=full, block=128,
                                      chunks=chunks, status_group=STATUS)
        torch.cuda.synchronize()
        got = orc.h2f(_u16(full)).reshape(n, m)
        err = orc.rel_frobenius(got, want)
        assert err <= 2e-3, f"rank {rank}: column shard (transB {transB}) relative error {err}"


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    global STATUS
    STATUS = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(2024)     # same inputs on every rank
    try:
        check_batch(rank, world, rng)
        check_columns(rank, world, rng)
        assert vk.device_status(True) == 0
        dist.barrier()
        print(f"OK rank {rank} of {world} ({dist.get_backend()})", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
