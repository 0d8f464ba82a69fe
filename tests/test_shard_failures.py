"""Failures of a multi-rank sharded GEMM surface as exceptions, not hangs.

Simulated on the host as gloo ranks on CPU (no GPU is faulted, stalled or
left waiting): a rank whose local GEMM raises, a rank that never joins the
process group, and a rank that dies between steps.  Every surviving rank must
raise within a few seconds -- far below the process-group timeout, so a hang
would show as the timeout instead.
"""
import os
import socket
import time

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import vkblas_b200 as vk
from oracle import oracle as orc

PG_TIMEOUT_S = 60


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_gemm(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch, sa, sb, sc):
    c = C.numpy()
    orc.gemm_rowmajor_f32seq(op_a, op_b, M, N, K, alpha, np.ascontiguousarray(A.numpy()), lda,
                             np.ascontiguousarray(B.numpy()), ldb, beta, c, ldc, batch, sa, sb, sc)


def _failing_gemm(*args):
    raise vk.VkblasError("injected: local GEMM failed")


def _init(rank, world, port, timeout_s=PG_TIMEOUT_S):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_gemm_fails(rank, world, port, q):
    from vkblas_b200 import shard
    _init(rank, world, port)
    M, N, K, batch = 16, 12, 8, 4
    b0, n = shard.batch_shard(batch, rank, world)
    A = torch.ones(n * M * K)
    B = torch.ones(n * K * N)
    full = torch.zeros(batch * M * N)
    C = full[b0 * M * N: (b0 + n) * M * N]
    t0 = time.monotonic()
    try:
        shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.0, A, K, M * K, B, N, K * N, 0.0, C, N,
                                   M * N, batch, rank=rank, world=world, C_full=full,
                                   gemm_fn=_failing_gemm if rank == 1 else _cpu_gemm,
                                   status_group=dist.group.WORLD)
        q.put((rank, "no error", time.monotonic() - t0))
    except vk.VkblasError as exc:
        q.put((rank, str(exc), time.monotonic() - t0))
    finally:
        dist.destroy_process_group()


def test_local_gemm_failure_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.spawn(_worker_gemm_fails, args=(2, _free_port(), q), nprocs=2, join=True)
    got = {}
    while not q.empty():
        r, msg, dt = q.get()
        got[r] = (msg, dt)
    assert got[1][0] == "injected: local GEMM failed"
    assert "another rank" in got[0][0], got
    assert max(dt for _, dt in got.values()) < 10, got


def _worker_never_joins(rank, world, port, q):
    if rank == 1:
        return                               # this rank exits before joining
    t0 = time.monotonic()
    try:
        _init(rank, world, port, timeout_s=3)
        q.put((rank, "joined", time.monotonic() - t0))
        dist.destroy_process_group()
    except Exception as exc:                 # DistStoreError / RuntimeError from the rendezvous
        q.put((rank, type(exc).__name__, time.monotonic() - t0))


def test_rank_that_never_joins_ends_init_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.spawn(_worker_never_joins, args=(2, _free_port(), q), nprocs=2, join=True)
    r, what, dt = q.get()
    assert r == 0 and what != "joined", what
    assert dt < 30, dt


def _worker_dies_between_steps(rank, world, port, q):
    from vkblas_b200 import shard
    _init(rank, world, port, timeout_s=10)
    M, N, K, batch = 8, 8, 8, 2
    b0, n = shard.batch_shard(batch, rank, world)
    A, B = torch.ones(n * M * K), torch.ones(n * K * N)
    full = torch.zeros(batch * M * N)
    C = full[b0 * M * N: (b0 + n) * M * N]
    step = dict(rank=rank, world=world, C_full=full, gemm_fn=_cpu_gemm,
                status_group=dist.group.WORLD)
    shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.0, A, K, M * K, B, N, K * N, 0.0, C, N, M * N,
                               batch, **step)
    if rank == 1:
        os._exit(0)                          # leaves between steps, nothing in flight
    t0 = time.monotonic()
    try:
        shard.sharded_batched_gemm(0, 0, 0, M, N, K, 1.0, A, K, M * K, B, N, K * N, 0.0, C, N,
                                   M * N, batch, **step)
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception as exc:
        q.put((rank, type(exc).__name__, time.monotonic() - t0))


def test_rank_that_dies_between_steps_ends_the_next_step_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_dies_between_steps, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    r, what, dt = q.get()
    assert r == 0 and what != "no error", what
    assert dt < 30, dt
