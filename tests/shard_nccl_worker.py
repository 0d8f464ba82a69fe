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
* the fused replication (replicate="p2p": the tcgen05 epilogue stores each
  tile into every rank's C over NVLink through a CUDA IPC PeerMap, then a
  one-element all-reduce), for batch and column shards, a rank with an empty
  shard, and problems the replicated kernel declines (all ranks gather);
  every rank's replicated C must be bit for bit the same.  The host-side
  status exchange runs over a gloo group.
"""
import hashlib
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


def _same_on_every_rank(full, what):
    h = hashlib.sha1(full.view(torch.uint8).cpu().numpy().tobytes()).hexdigest()
    hs = [None] * dist.get_world_size()
    dist.all_gather_object(hs, h, group=STATUS)
    assert len(set(hs)) == 1, f"{what}: the replicas differ"


def _run(mode, full, fn):
    """Run fn(peer_map) with a PeerMap of `full` for mode "p2p" (closed after
    a barrier, so no rank still stores into this rank's buffer)."""
    pm = shard.PeerMap(full, dist.get_rank(), dist.get_world_size(), STATUS) if mode == "p2p" else None
    try:
        fn(pm)
        torch.cuda.synchronize()
    finally:
        if pm is not None:
            dist.barrier(group=STATUS)
            pm.close()


def check_batch(rank, world, rng):
    M, N, K = 192, 160, 136
    for batch, bcast, mode in ((4 * world, False, "gather"), (4 * world + 1, False, "gather"),
                               (2 * world, True, "gather"), (4 * world + 1, False, "p2p"),
                               (8 * world, True, "p2p"), (1, False, "p2p")):
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
        _run(mode, full, lambda pm: shard.sharded_batched_gemm(
            vk.DT_F16, 0, 0, M, N, K, 1.0, Al, K, sa, Bl, N, sb, 0.0, Cl, N, sc, batch, rank=rank,
            world=world, C_full=full, status_group=STATUS, replicate=mode, peer_map=pm))
        got = orc.h2f(_u16(full)).reshape(batch, M, N)
        err = orc.rel_frobenius(got, want)
        assert err <= 2e-3, (f"rank {rank}: fp16 batch shard (batch {batch}, {mode}) "
                             f"relative error {err}")
        if n:
            assert np.array_equal(_u16(Cl)[: n * sc], _u16(full)[b0 * sc: (b0 + n) * sc])
        _same_on_every_rank(full, f"batch {batch} {mode}")
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
    for transB, mode in ((0, "gather"), (1, "gather"), (0, "p2p"), (1, "p2p")):
        A = orc.f2h(rng.uniform(-1, 1, m * k).astype(np.float32))          # transA = N, lda = m
        B = orc.f2h(rng.uniform(-1, 1, k * n).astype(np.float32))
        ldb = k if transB == 0 else n
        # column-major C = A op(B): the engine call (op_a = transB, op_b = N, M = n, N = m)
        want = orc.hgemm_rowmajor_f64(0, transB, 0, n, m, k, 1.0, B, ldb, A, m, 0.0, None, m)[0]
        c0, cnt = shard.column_shard(n, rank, world, block=128)
        Bc = _dev16(B[c0 * ldb: (c0 + cnt) * ldb] if transB == 0 else B)
        Cc = torch.zeros(max(cnt, 1) * m, dtype=torch.float16, device="cuda")
        full = torch.zeros(m * n, dtype=torch.float16, device="cuda")
        dA = _dev16(A)
        _run(mode, full, lambda pm: shard.sharded_column_gemm_hip(
            vk.DT_F16, 0, transB, m, n, k, 1.0, dA, m, Bc, ldb, 0.0, Cc, m, rank=rank, world=world,
            C_full=full, block=128, status_group=STATUS, replicate=mode, peer_map=pm))
        got = orc.h2f(_u16(full)).reshape(n, m)
        err = orc.rel_frobenius(got, want)
        assert err <= 2e-3, f"rank {rank}: column shard (transB {transB}, {mode}) relative error {err}"
        _same_on_every_rank(full, f"columns transB {transB} {mode}")


def check_p2p_fallback(rank, world, rng):
    """fp16 with M <= 64 and N >= 128 runs transposed, which the replicated
    kernel declines: every rank computes plainly and all gather; the result
    is the same as with replicate="gather", without and with a status group."""
    M, N, K, batch = 32, 256, 64, 2 * world
    A = orc.f2h(rng.uniform(-1, 1, M * K * batch).astype(np.float32))
    B = orc.f2h(rng.uniform(-1, 1, K * N * batch).astype(np.float32))
    want = orc.hgemm_rowmajor_f64(0, 0, 0, M, N, K, 1.0, A, K, B, N, 0.0, None, N, batch, M * K,
                                  K * N, M * N)
    b0, n = shard.batch_shard(batch, rank, world)
    Al = _dev16(A[b0 * M * K: (b0 + n) * M * K])
    Bl = _dev16(B[b0 * K * N: (b0 + n) * K * N])
    for sg in (STATUS, None):
        full = torch.zeros(M * N * batch, dtype=torch.float16, device="cuda")
        Cl = full[b0 * M * N: (b0 + n) * M * N]
        _run("p2p", full, lambda pm: shard.sharded_batched_gemm(
            vk.DT_F16, 0, 0, M, N, K, 1.0, Al, K, M * K, Bl, N, K * N, 0.0, Cl, N, M * N, batch,
            rank=rank, world=world, C_full=full, status_group=sg, replicate="p2p", peer_map=pm))
        got = orc.h2f(_u16(full)).reshape(batch, M, N)
        assert orc.rel_frobenius(got, want) <= 2e-3, f"rank {rank}: p2p fallback"
        _same_on_every_rank(full, "p2p fallback")


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
        check_p2p_fallback(rank, world, rng)
        assert vk.device_status(True) == 0
        dist.barrier()
        print(f"OK rank {rank} of {world} ({dist.get_backend()})", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
