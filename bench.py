"""Benchmark of the B200 BLAS core (one JSON line on rank 0).

Headline workload: fp32 SGEMM 4096 x 4096 x 4096,
transA = transB = N (the PyTorch ``a @ b`` path), column-major, alpha = 1,
beta = 0, A and B ~ N(0, 1) from a fixed seed, issued through the public
hipBLAS ABI (``hipblasSgemm`` of libvkblas_hipblas.so) on device-resident
buffers.  One step = one 4096^3 GEMM per GPU.  With N GPUs the job is a
strided-batched SGEMM of N such GEMMs sharded by batch (one per rank, no
data-path collective): weak scaling, value = total useful FLOP/s of all ranks.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

``--impl reference`` times the reference's own CPU GEMM (``ref_gemm`` of
test/test_gemm.c, compiled from the reference sources into oracle/_ref; the
oracle's port of it when that build is absent) on the host cores, on a
bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MNK = 4096
FLOP_PER_GEMM = 2.0 * MNK ** 3
METRIC = "SGEMM/HGEMM TFLOPS at 4096^3 (% of peak); decode GEMV HBM GB/s"


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = [("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown")]

    def __init__(self, index: int, period_s: float = 0.02):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._nv = nv
            self._h = nv.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            pass
        self._period = period_s
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, const in self.REASONS:
                    if r & getattr(nv, const, 0):
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._ok:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._ok:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------- CPU reference arm
class CpuReference:
    """Reference ref_gemm (test/test_gemm.c:32-58) on all host threads, row-sampled.

    A 4096^3 NN problem; R rows of C are computed (the reference's own
    row-sampling idea, test/test_gemm.c:36-43), split over all host threads;
    FLOP/s = 2*R*n*k / wall time."""

    def __init__(self):
        import numpy as np
        from oracle import oracle as orc
        self.np = np
        self.threads = os.cpu_count() or 1
        rng = np.random.default_rng(0)
        self.A = rng.standard_normal(MNK * MNK, dtype=np.float32)
        self.B = rng.standard_normal(MNK * MNK, dtype=np.float32)
        self.C = np.zeros(MNK * MNK, np.float32)
        if orc.ref is not None:
            self.fn, self.kind = orc.ref.vkref_ref_gemm_rows_mt, "reference"
        else:
            self.fn, self.kind = orc.lib.orc_sgemm_colmajor_rows_mt, "port"
        self.t_row = None

    def _rows(self, rows):
        t0 = time.perf_counter()
        self.fn(0, 0, MNK, MNK, MNK, 1.0, self.A, MNK, self.B, MNK, 0.0, self.C, MNK, 0, rows,
                self.threads)
        return time.perf_counter() - t0

    def sample(self, target_s: float):
        if self.t_row is None:   # one row per thread calibrates the per-row cost
            self.t_row = self._rows(min(MNK, self.threads))
        per_thread = max(1, min(MNK // self.threads, int(target_s / max(self.t_row, 1e-6))))
        rows = min(MNK, per_thread * self.threads)
        dt = self._rows(rows)
        tf = 2.0 * rows * MNK * MNK / dt / 1e12
        return tf, {"kind": self.kind, "cores": self.threads,
                    "sample": f"{rows} of 4096 rows of the 4096^3 NN SGEMM (ref_gemm, double "
                              f"accumulation), {dt:.2f} s wall on {self.threads} threads"}


# ------------------------------------------------------------ GPU pieces
def _hip_sgemm(vk, hb, h, dA, dB, dC, al, be):
    return vk.lib.hipblasSgemm(h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, MNK, MNK, MNK, al,
                               dA.data_ptr(), MNK, dB.data_ptr(), MNK, be, dC.data_ptr(), MNK)


def _time_loop(fn, iters, stream):
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(iters):
        fn(i)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def secondary_results(vk, hb, torch, peaks, ceil=None):
    """Other BASELINE configs on one GPU (device-resident inputs, CUDA events).
    Fractions are of MEASURED_PEAKS.json (bf16 burst, HBM copy) and of the
    ceilings measured in this run (``ceil``, run_peaks) where one applies."""
    ceil = ceil or {}
    f16_ceil = ceil.get("tcgen05_f16_pair", {}).get("tflops")
    out = {}
    s = torch.cuda.Stream()         # CUDA graphs cannot be captured on the default stream
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    g = torch.Generator(device="cuda").manual_seed(3)
    with hb.Handle() as h, torch.cuda.stream(s):
        h.set_stream(s)
        # config 4 first, before the long compute-bound GEMMs below leave the GPU
        # under its power cap: decode GEMV, 4 rotating weight sets (470 MB > L2).  Timed two
        # ways: back-to-back calls (includes each call's launch gap) and a CUDA
        # graph of 40 calls replayed (kernel time; what a decode loop captures).
        K, O = 4096, 14336
        Ws = [(torch.randn(O, K, device="cuda", generator=g) * 0.02).half() for _ in range(4)]
        for M in (1, 4, 16):
            X = torch.randn(M, K, device="cuda", generator=g).half()
            C = torch.empty(M, O, device="cuda", dtype=torch.float16)

            def run(i, M=M, X=X, C=C):
                vk.lib.hipblasGemmEx(h.h, vk.HIPBLAS_OP_T, vk.HIPBLAS_OP_N, O, M, K, al,
                                     Ws[i % 4].data_ptr(), vk.HIPBLAS_R_16F, K, X.data_ptr(),
                                     vk.HIPBLAS_R_16F, K, be, C.data_ptr(), vk.HIPBLAS_R_16F, O,
                                     vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
            for i in range(4):
                run(i)
            ms = _time_loop(run, 40, s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for i in range(40):
                    run(i)
            graph.replay()
            ms_g = _time_loop(lambda i: graph.replay(), 5, s) / 40
            del graph
            nbytes = 2.0 * (O * K + M * K + M * O)
            gbs, gbs_g = nbytes / ms / 1e6, nbytes / ms_g / 1e6
            out[f"gemv_m{M}"] = {"gbs": round(gbs, 1), "us": round(ms * 1e3, 2),
                                 "gbs_graph": round(gbs_g, 1), "us_graph": round(ms_g * 1e3, 2),
                                 "path": vk.PATH_NAMES[vk.last_path()],
                                 "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4),
                                 "frac_of_hbm_graph": round(gbs_g / peaks["hbm_gbs"], 4)}
        del Ws
        # config 2, second kernel: the exact FFMA SIMT SGEMM at 4096^3 NN (two
        # input sets of 128 MiB, larger than L2, alternated call by call)
        n = 4096
        sets = [(torch.randn(n * n, device="cuda", generator=g),
                 torch.randn(n * n, device="cuda", generator=g),
                 torch.empty(n * n, device="cuda")) for _ in range(2)]

        def run_ffma(i):
            A, B, C = sets[i % 2]
            vk.lib.hipblasSgemm(h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, n, n, n, al, A.data_ptr(),
                                n, B.data_ptr(), n, be, C.data_ptr(), n)
        vk.set_path(vk.PATH_SIMT)
        try:
            for i in range(3):
                run_ffma(i)
            ms = _time_loop(run_ffma, 10, s)
            path = vk.PATH_NAMES[vk.last_path()]
        finally:
            vk.set_path(vk.PATH_AUTO)
        tf = 2.0 * n ** 3 / ms / 1e9
        nominal = 148 * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
        out["sgemm_ffma_nn_4096"] = {"tflops": round(tf, 2), "ms": round(ms, 4), "path": path,
                                     "frac_of_fp32_nominal": round(tf / nominal, 4)}
        if "ffma_fp32" in ceil:
            out["sgemm_ffma_nn_4096"]["frac_of_ffma_measured"] = round(
                tf / ceil["ffma_fp32"]["tflops"], 4)
        del sets
        # config 3: HGEMM T/N 4096^3, 8192^3 and 16384^3
        for n in (4096, 8192, 16384):
            sets = [((torch.randn(n, n, device="cuda", generator=g) * 0.02).half(),
                     (torch.randn(n, n, device="cuda", generator=g) * 0.02).half(),
                     torch.empty(n, n, device="cuda", dtype=torch.float16)) for _ in range(2)]

            def run(i, sets=sets, n=n):
                A, B, C = sets[i % 2]
                vk.lib.hipblasGemmEx_v2(h.h, vk.HIPBLAS_OP_T, vk.HIPBLAS_OP_N, n, n, n, al,
                                        A.data_ptr(), vk.HIP_R_16F, n, B.data_ptr(), vk.HIP_R_16F,
                                        n, be, C.data_ptr(), vk.HIP_R_16F, n,
                                        vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
            for i in range(3):
                run(i)
            ms = _time_loop(run, {4096: 20, 8192: 10, 16384: 5}[n], s)
            tf = 2.0 * n ** 3 / ms / 1e9
            out[f"hgemm_tn_{n}"] = {"tflops": round(tf, 2), "ms": round(ms, 4),
                                    "path": vk.PATH_NAMES[vk.last_path()],
                                    "frac_of_bf16_burst": round(tf / peaks["bf16_tflops"], 4)}
            if f16_ceil:
                out[f"hgemm_tn_{n}"]["frac_of_f16_mma_measured"] = round(tf / f16_ceil, 4)
            del sets
        # config 5: strided-batched 256 x 2048^3 NN
        b, n = 256, 2048
        A = (torch.randn(b, n, n, device="cuda", generator=g) * 0.02).half()
        B = (torch.randn(b, n, n, device="cuda", generator=g) * 0.02).half()
        C = torch.empty(b, n, n, device="cuda", dtype=torch.float16)

        def run(i):
            vk.lib.hipblasGemmStridedBatchedEx_v2(
                h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, n, n, n, al, A.data_ptr(), vk.HIP_R_16F, n,
                n * n, B.data_ptr(), vk.HIP_R_16F, n, n * n, be, C.data_ptr(), vk.HIP_R_16F, n,
                n * n, b, vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
        run(0)
        ms = _time_loop(run, 10, s)
        tf = 256 * 2.0 * n ** 3 / ms / 1e9
        out["hgemm_batched_256x2048"] = {"tflops": round(tf, 2), "ms": round(ms, 3),
                                         "path": vk.PATH_NAMES[vk.last_path()],
                                         "frac_of_bf16_burst": round(tf / peaks["bf16_tflops"], 4)}
        if f16_ceil:
            out["hgemm_batched_256x2048"]["frac_of_f16_mma_measured"] = round(tf / f16_ceil, 4)
        del A, B, C
    return out


def _max_over_ranks(torch, dist, ms):
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


NVLINK_GBS = 770.0      # measured peer copy, GB/s per direction per GPU (this pool's B200s)


def _fused_roofline(r, flop_per_rank, send_bytes, peak_tflops):
    """Roofline of the fused GEMM + replication: the slower of the rank's
    FLOPs at the bf16 burst rate and the bytes it must send over NVLink at
    the measured peer-copy rate; frac = that time / the measured time."""
    t_math = flop_per_rank / (peak_tflops * 1e12) * 1e3
    t_link = send_bytes / (NVLINK_GBS * 1e9) * 1e3
    target = max(t_math, t_link)
    r["p2p_roofline"] = {"target_ms": round(target, 3), "bound": "nvlink" if t_link > t_math else "tensor",
                         "math_ms": round(t_math, 3), "link_ms": round(t_link, 3),
                         "frac": round(target / r["with_p2p_epilogue"]["ms"], 3),
                         "peaks": f"bf16 burst {peak_tflops} TF (MEASURED_PEAKS.json), NVLink {NVLINK_GBS} GB/s"}


def sharded_secondary(vk, torch, dist, rank, world, stream, status_group=None, peaks=None):
    """The sharded BASELINE configs across the ranks (device time, max over
    ranks), each three ways: the GEMM alone (every rank keeps its shard), the
    GEMM followed by one all-gather that replicates C, and the fused form
    whose epilogue stores every tile of C into all ranks' copies over NVLink
    (replicate="p2p"; one one-element all-reduce as the rendezvous):

    * config 5, 256 x 2048^3 fp16 NN strided-batched, sharded by batch;
    * config 3 at 16384^3 (fp16, hipBLAS T/N) sharded by column blocks of C.

    For each: the times, what replication adds over the GEMM alone, and the
    bytes each rank must send (its shard to every other rank)."""
    from vkblas_b200 import shard
    out = {}

    def timed(run, reps):
        run()
        torch.cuda.synchronize()
        dist.barrier()
        return _max_over_ranks(torch, dist, _time_loop(lambda i: run(), reps, stream))

    def three_ways(run, reps, flop, C_full):
        r = {}
        pm = shard.PeerMap(C_full, rank, world, status_group)
        try:
            for key, mode in (("gemm_only", None), ("with_allgather", "gather"),
                              ("with_p2p_epilogue", "p2p")):
                ms = timed(lambda: run(mode, pm), reps)
                r[key] = {"ms": round(ms, 3), "tflops": round(flop / ms / 1e9, 2)}
        finally:
            torch.cuda.synchronize()
            dist.barrier()
            pm.close()
        base = r["gemm_only"]["ms"]
        r["allgather_extra_ms"] = round(r["with_allgather"]["ms"] - base, 3)
        r["p2p_extra_ms"] = round(r["with_p2p_epilogue"]["ms"] - base, 3)
        r["p2p_over_gemm_only"] = round(r["with_p2p_epilogue"]["ms"] / base, 3)
        return r

    # config 5
    b, n = 256, 2048
    b0, cnt = shard.batch_shard(b, rank, world)
    g = torch.Generator(device="cuda").manual_seed(500 + rank)
    A = (torch.randn(cnt * n * n, device="cuda", generator=g) * 0.02).half()
    B = (torch.randn(cnt * n * n, device="cuda", generator=g) * 0.02).half()
    C_full = torch.empty(b * n * n, device="cuda", dtype=torch.float16)
    C_local = C_full[b0 * n * n: (b0 + cnt) * n * n]

    def run5(mode, pm):
        shard.sharded_batched_gemm(vk.DT_F16, 0, 0, n, n, n, 1.0, A, n, n * n, B, n, n * n, 0.0,
                                   C_local, n, n * n, b, rank=rank, world=world,
                                   C_full=C_full if mode else None, status_group=status_group,
                                   replicate=mode or "gather", peer_map=pm)
    r5 = three_ways(run5, 5, b * 2.0 * n ** 3, C_full)
    r5["send_bytes_per_rank"] = cnt * n * n * 2 * (world - 1)
    if peaks:
        _fused_roofline(r5, cnt * 2.0 * n ** 3, r5["send_bytes_per_rank"], peaks["bf16_tflops"])
    out["hgemm_batched_256x2048_sharded"] = r5
    del A, B, C_full, C_local
    torch.cuda.empty_cache()

    # config 3 at 16384^3, column blocks of C (hipBLAS T/N: A is K x M, lda = K)
    m = k = nn = 16384
    c0, cc = shard.column_shard(nn, rank, world, 256)
    g = torch.Generator(device="cuda").manual_seed(600 + rank)
    A = (torch.randn(k * m, device="cuda", generator=g) * 0.02).half()
    Bc = (torch.randn(max(cc, 1) * k, device="cuda", generator=g) * 0.02).half()
    C_full = torch.empty(m * nn, device="cuda", dtype=torch.float16)
    C_cols = C_full[c0 * m: (c0 + cc) * m]

    def run3(mode, pm):
        shard.sharded_column_gemm_hip(vk.DT_F16, 1, 0, m, nn, k, 1.0, A, k, Bc, k, 0.0, C_cols, m,
                                      rank=rank, world=world, C_full=C_full if mode else None,
                                      status_group=status_group, replicate=mode or "gather",
                                      peer_map=pm)
    r3 = three_ways(run3, 3, 2.0 * m * nn * k, C_full)
    r3["send_bytes_per_rank"] = cc * m * 2 * (world - 1)
    if peaks:
        _fused_roofline(r3, 2.0 * m * cc * k, r3["send_bytes_per_rank"], peaks["bf16_tflops"])
    out["hgemm_tn_16384_column_sharded"] = r3
    del A, Bc, C_full, C_cols
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------- single-case runner
CASES = ["sgemm", "sgemm-simt", "hgemm", "gemv", "gemv32", "batched", "dgemm", "zgemm", "peaks",
         "cpu"]


def run_peaks(vk, torch, stream, reps=3):
    """Throughput ceilings of this GPU (vkblas_b200_peak_launch): each kernel
    once untimed, then `reps` launches timed with CUDA events; TFLOP/s of the
    best.  Sized to about 2 ms a launch."""
    import ctypes as C
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    iters = {0: 2048, 1: 8192, 2: 8192, 3: 8192, 4: 8192}
    names = {0: "ffma_fp32", 1: "tcgen05_tf32", 2: "tcgen05_tf32_pair", 3: "tcgen05_f16",
             4: "tcgen05_f16_pair"}
    out = {}
    for which, name in names.items():
        flops = C.c_double()
        ms = []
        for r in range(reps + 1):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            st = vk.lib.vkblas_b200_peak_launch(which, iters[which], stream.cuda_stream,
                                                status.data_ptr(), C.byref(flops))
            e1.record(stream)
            if st != vk.VKBLAS_OK:
                raise RuntimeError(f"vkblas_b200_peak_launch({which}) status {st}")
            torch.cuda.synchronize()
            if r:
                ms.append(e0.elapsed_time(e1))
        if int(status.item()) != 0:
            raise RuntimeError(f"peak kernel {name}: device status {int(status.item())}")
        out[name] = {"tflops": round(flops.value / min(ms) / 1e9, 1), "ms": round(min(ms), 4)}
    return out


def run_cpu_baselines(budget_s: float = 6.0) -> dict:
    """The reference's own CPU GEMMs timed on this host (oracle/_ref, compiled
    from the reference's test/test_gemm.c and test/test_h.c; the oracle's port
    of ref_gemm when that build is absent), for every BASELINE config:

    * ref_gemm (test/test_gemm.c:32-58), config 2 (4096^3 NN), row-sampled as
      the reference itself samples rows (test/test_gemm.c:36-43), on 1 thread
      and on all threads;
    * ref_gemm, config 1 (1024^3, alpha 1.5, beta 0.5) in full, all four ops,
      all threads;
    * cpu_ref (test/test_h.c:63-79), config 3 (fp16, hipBLAS T/N, M=N=K in
      {4096, 8192, 16384}) on a sample of C's columns, all threads;
    * cpu_ref, config 4 (decode, M in {1, 4, 16} x 4096 -> 14336) in full, all
      threads (split over C's columns, so M = 1 uses them too).

    TFLOP/s = 2 x the multiply-adds of what ran / wall time.  ``budget_s``
    bounds each sampled measurement."""
    import platform
    import numpy as np
    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    ref = orc.ref
    out = {"host": {"nproc": threads, "cpu": platform.processor() or platform.machine()},
           "kind": "reference" if ref is not None else "port"}
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    out["host"]["cpu"] = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    rows_fn = ref.vkref_ref_gemm_rows_mt if ref is not None else orc.lib.orc_sgemm_colmajor_rows_mt
    rng = np.random.default_rng(0)

    def sgemm_rows(n, ta, tb, alpha, beta, rows, nthr, A, B, C):
        t0 = time.perf_counter()
        rows_fn(ta, tb, n, n, n, alpha, A, n, B, n, beta, C, n, 0, rows, nthr)
        return time.perf_counter() - t0

    n = 4096
    A = rng.standard_normal(n * n, dtype=np.float32)
    B = rng.standard_normal(n * n, dtype=np.float32)
    C = np.zeros(n * n, np.float32)
    for nthr in (1, threads):
        per_row = sgemm_rows(n, 0, 0, 1.0, 0.0, nthr, nthr, A, B, C) / nthr   # wall per row
        rows = int(min(n, max(nthr, budget_s / max(per_row, 1e-6))))
        rows = max(nthr, rows // nthr * nthr)
        dt = sgemm_rows(n, 0, 0, 1.0, 0.0, rows, nthr, A, B, C)
        out[f"cfg2_sgemm_4096_nn_{nthr}t"] = {
            "tflops": 2.0 * rows * n * n / dt / 1e12, "threads": nthr,
            "sample": f"{rows} of 4096 rows, {dt:.2f} s"}
    n = 1024
    A1 = rng.uniform(-1, 1, n * n).astype(np.float32)
    B1 = rng.uniform(-1, 1, n * n).astype(np.float32)
    for ta, tb in ((0, 0), (0, 1), (1, 0), (1, 1)):
        C1 = rng.uniform(-1, 1, n * n).astype(np.float32)
        dt = sgemm_rows(n, ta, tb, 1.5, 0.5, n, threads, A1, B1, C1)
        out[f"cfg1_sgemm_1024_{'NT'[ta]}{'NT'[tb]}"] = {
            "tflops": 2.0 * n ** 3 / dt / 1e12, "threads": threads, "sample": f"full, {dt:.2f} s"}
    if ref is None:
        return out
    half = ref.vkref_cpu_ref_half_cols_mt
    for n in (4096, 8192, 16384):
        # hipBLAS T/N, column-major C (n x n) = A^T B: the engine call (N, T) with
        # M = n rows of B's columns and N = n; a sample of C's columns
        Ah = orc.f2h((rng.standard_normal(n * n) * 0.02).astype(np.float32))
        Bh = orc.f2h((rng.standard_normal(n * n) * 0.02).astype(np.float32))
        Ch = np.zeros(n * n, np.uint16)
        t0 = time.perf_counter()
        half(0, 0, 1, n, n, n, Bh, n, Ah, n, 1.0, 0.0, Ch, n, 0, threads, threads)
        per_col = (time.perf_counter() - t0) / threads     # wall time per column, all threads
        cols = int(min(n, max(threads, budget_s / max(per_col, 1e-6))))
        cols = max(threads, cols // threads * threads)
        t0 = time.perf_counter()
        half(0, 0, 1, n, n, n, Bh, n, Ah, n, 1.0, 0.0, Ch, n, 0, cols, threads)
        dt = time.perf_counter() - t0
        out[f"cfg3_hgemm_tn_{n}"] = {"tflops": 2.0 * n * n * cols / dt / 1e12, "threads": threads,
                                      "sample": f"{cols} of {n} columns of C, {dt:.2f} s"}
        del Ah, Bh, Ch
    K, O = 4096, 14336
    W = orc.f2h((rng.standard_normal(O * K) * 0.02).astype(np.float32))
    for m in (1, 4, 16):
        X = orc.f2h(rng.standard_normal(m * K).astype(np.float32))
        Cd = np.zeros(m * O, np.uint16)
        t0 = time.perf_counter()
        half(0, 0, 1, m, O, K, X, K, W, K, 1.0, 0.0, Cd, O, 0, O, threads)
        dt = time.perf_counter() - t0
        nbytes = 2.0 * (O * K + m * K + m * O)
        out[f"cfg4_decode_m{m}"] = {"gbs": nbytes / dt / 1e9, "us": dt * 1e6,
                                    "tflops": 2.0 * m * O * K / dt / 1e12, "threads": threads,
                                    "sample": f"full, {dt:.3f} s"}
    return out


def run_case(a) -> int:
    """One GEMM case of the BASELINE configs, `--iters` times on torch's current
    stream after one untimed call (for timing and ncu captures):

        python bench.py --case sgemm  [--n 4096] [--shape M,N,K]   # 3xTF32, N/N
        python bench.py --case sgemm-simt [--n 4096]               # exact FFMA kernel
        python bench.py --case hgemm  [--n 4096] [--shape M,N,K]   # fp16 tcgen05, hipBLAS T/N
        python bench.py --case gemv   [--m 1] [--splitk 4]         # decode, K=4096, N=14336
        python bench.py --case gemv32 [--m 1] [--trans t|n]        # fp32 decode
        python bench.py --case dgemm|zgemm [--n 2048]              # fp64 / complex128 N/N
        python bench.py --case batched                             # 256 x 2048^3 fp16 N/N
        python bench.py --case peaks                               # tcgen05 / FFMA ceilings
        python bench.py --case cpu                                 # the reference's CPU GEMMs

    Inputs are device-resident and seeded; the mean time per call (CUDA
    events) is printed.  --path simt|tc|gemv forces a kernel family; --graph
    replays the calls from a CUDA graph (kernel time without host launch gaps)."""
    if a.case == "cpu":
        print(json.dumps(run_cpu_baselines()))
        return 0
    import torch
    import vkblas_b200 as vk
    from vkblas_b200 import hipblas as hb

    if a.case == "peaks":
        torch.cuda.init()
        s = torch.cuda.current_stream()
        with ClockSampler(torch.cuda.current_device(), period_s=0.005) as clk:
            res = run_peaks(vk, torch, s, reps=max(1, a.iters))
        res["clocks"] = clk.summary()
        print(json.dumps(res))
        return 0
    torch.cuda.init()
    # CUDA graphs cannot be captured on the legacy default stream
    s = torch.cuda.Stream() if a.graph else torch.cuda.current_stream()
    torch.cuda.set_stream(s)
    g = torch.Generator(device="cuda").manual_seed(0)
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    h = hb.Handle()
    h.set_stream(s)
    n = a.n
    M, N, K = (int(x) for x in a.shape.split(",")) if a.shape else (n, n, n)
    if a.case in ("sgemm", "sgemm-simt"):
        A = torch.randn(M * K, device="cuda", generator=g)
        B = torch.randn(K * N, device="cuda", generator=g)
        C = torch.empty(M * N, device="cuda")
        if a.case == "sgemm-simt":
            vk.set_path(vk.PATH_SIMT)
        flop, nbytes = 2.0 * M * N * K, 0.0
        # column-major C (M x N) = A (M x K) * B (K x N)
        call = lambda: vk.lib.hipblasSgemm(h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, M, N, K, al,  # noqa: E731
                                           A.data_ptr(), M, B.data_ptr(), K, be, C.data_ptr(), M)
    elif a.case == "hgemm":
        A = (torch.randn(M * K, device="cuda", generator=g) * 0.02).half()
        B = (torch.randn(K * N, device="cuda", generator=g) * 0.02).half()
        C = torch.empty(M * N, device="cuda", dtype=torch.float16)
        flop, nbytes = 2.0 * M * N * K, 0.0
        # column-major C (M x N) = A^T (A stored K x M) * B (K x N)
        call = lambda: vk.lib.hipblasGemmEx_v2(h.h, vk.HIPBLAS_OP_T, vk.HIPBLAS_OP_N, M, N, K, al,  # noqa: E731
                                               A.data_ptr(), vk.HIP_R_16F, K, B.data_ptr(),
                                               vk.HIP_R_16F, K, be, C.data_ptr(), vk.HIP_R_16F, M,
                                               vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
    elif a.case == "gemv":
        K, O, M = 4096, 14336, a.m
        # four weight sets (470 MB > 126 MB L2), rotated call by call
        Ws = [(torch.randn(O * K, device="cuda", generator=g) * 0.02).half() for _ in range(4)]
        X = torch.randn(M * K, device="cuda", generator=g).half()
        C = torch.empty(M * O, device="cuda", dtype=torch.float16)
        if a.splitk:
            vk.set_splitk(a.splitk)
        flop, nbytes = 2.0 * M * O * K, 2.0 * (O * K + M * K + M * O)
        turn = [0]

        def call():
            turn[0] += 1
            return vk.lib.hipblasGemmEx(h.h, vk.HIPBLAS_OP_T, vk.HIPBLAS_OP_N, O, M, K, al,
                                        Ws[turn[0] % 4].data_ptr(), vk.HIPBLAS_R_16F, K, X.data_ptr(),
                                        vk.HIPBLAS_R_16F, K, be, C.data_ptr(), vk.HIPBLAS_R_16F, O,
                                        vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
    elif a.case == "gemv32":
        K, O, M = 4096, 14336, a.m
        # four fp32 weight sets (940 MB > 126 MB L2), rotated call by call
        Ws = [torch.randn(O * K, device="cuda", generator=g) * 0.02 for _ in range(4)]
        X = torch.randn(M * K, device="cuda", generator=g)
        C = torch.empty(M * O, device="cuda")
        if a.splitk:
            vk.set_splitk(a.splitk)
        flop, nbytes = 2.0 * M * O * K, 4.0 * (O * K + M * K + M * O)
        tA = vk.HIPBLAS_OP_T if a.trans == "t" else vk.HIPBLAS_OP_N
        lda = K if a.trans == "t" else O
        turn = [0]

        def call():
            turn[0] += 1
            return vk.lib.hipblasSgemm(h.h, tA, vk.HIPBLAS_OP_N, O, M, K, al,
                                       Ws[turn[0] % 4].data_ptr(), lda, X.data_ptr(), K, be,
                                       C.data_ptr(), O)
    elif a.case in ("dgemm", "zgemm"):
        cplx = a.case == "zgemm"
        w = 2 if cplx else 1
        A = torch.randn(w * M * K, device="cuda", generator=g, dtype=torch.float64)
        B = torch.randn(w * K * N, device="cuda", generator=g, dtype=torch.float64)
        C = torch.zeros(w * M * N, device="cuda", dtype=torch.float64)
        vk.set_stream(s)
        # useful FLOP: a complex multiply-add is 4 real ones
        flop, nbytes = (8.0 if cplx else 2.0) * M * N * K, 0.0
        if cplx:
            call = lambda: vk.lib.vkblas_gemm_z64(0, 0, M, N, K, 1.0, 0.0, A.data_ptr(), K,  # noqa: E731
                                                  B.data_ptr(), N, 0.0, 0.0, C.data_ptr(), N, 1,
                                                  0, 0, 0)
        else:
            call = lambda: vk.lib.vkblas_gemm_f64(0, 0, M, N, K, 1.0, A.data_ptr(), K,  # noqa: E731
                                                  B.data_ptr(), N, 0.0, C.data_ptr(), N, 1, 0, 0, 0)
    else:
        b, n = 256, 2048
        A = (torch.randn(b * n * n, device="cuda", generator=g) * 0.02).half()
        B = (torch.randn(b * n * n, device="cuda", generator=g) * 0.02).half()
        C = torch.empty(b * n * n, device="cuda", dtype=torch.float16)
        flop, nbytes = b * 2.0 * n ** 3, 0.0
        call = lambda: vk.lib.hipblasGemmStridedBatchedEx_v2(  # noqa: E731
            h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, n, n, n, al, A.data_ptr(), vk.HIP_R_16F, n,
            n * n, B.data_ptr(), vk.HIP_R_16F, n, n * n, be, C.data_ptr(), vk.HIP_R_16F, n, n * n,
            b, vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)

    if a.path != "auto":
        vk.set_path({"simt": vk.PATH_SIMT, "tc": vk.PATH_TC, "gemv": vk.PATH_GEMV}[a.path])
    st = call()
    if st != 0:
        raise SystemExit(f"status {st}")
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if a.graph:
        # the calls captured once and replayed: no host launch gaps
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for _ in range(a.iters):
                call()
        graph.replay()
        torch.cuda.synchronize()
        reps = 5
        e0.record(s)
        for _ in range(reps):
            graph.replay()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * max(1, a.iters))
        del graph
    else:
        kev = []
        if a.kernel_events:      # the library's event pair around each call's main kernel
            kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(a.iters)]
            for x, y in kev:
                x.record(s)
                y.record(s)
            torch.cuda.synchronize()
        e0.record(s)
        for i in range(a.iters):
            if kev:
                vk.set_kernel_events(*kev[i])
            call()
        e1.record(s)
        torch.cuda.synchronize()
        vk.set_kernel_events(None, None)
        ms = e0.elapsed_time(e1) / max(1, a.iters)
        if kev:
            kms = sum(x.elapsed_time(y) for x, y in kev) / len(kev)
            print(f"kernel events: {kms * 1e3:.2f} us/call between the events")
    st = vk.device_status(True)
    line = f"{a.case}: {ms * 1e3:.2f} us/call, {flop / ms / 1e9:.2f} TFLOP/s"
    if nbytes:
        line += f", {nbytes / ms / 1e6:.1f} GB/s"
    print(line + f", path={vk.PATH_NAMES[vk.last_path()]}, status={st}")
    h.close()
    return 0 if st == 0 else 1



def _roofline(path, tile_n, pair, split, gemm_ms, ms_step, peaks, peaks_kind, ceil=None):
    """The bench line's `roofline` object for the headline GEMM kernel: its
    useful FLOP/s against the ceiling measured in the same run (``ceil``, from
    run_peaks: the tcgen05 kind::tf32 MMA loop / 3, or the FFMA loop), with the
    peak derived from MEASURED_PEAKS.json's bf16 burst beside it, the tile
    configuration that ran, and its ncu DRAM traffic per launch where a capture
    of that configuration is committed under profiles/."""
    kernel_tflops = FLOP_PER_GEMM / (ms_step / 1e3) / 1e12
    gemm_tflops = FLOP_PER_GEMM / (gemm_ms / 1e3) / 1e12
    traffic, traffic_src = None, None
    extra = {}
    if path == "tc":
        tiles = f"{256 if pair else 128}x{tile_n} tiles" + (" on CTA pairs" if pair else "")
        kernel_name = f"3xTF32 tcgen05 SGEMM (umma_gemm_kernel, {tiles}" + (
            f"; last wave split {split} ways, then split_reduce_kernel)" if split > 1 else ")")
        derived = peaks["bf16_tflops"] / 2.0 / 3.0
        key = "tcgen05_tf32_pair" if pair else "tcgen05_tf32"
        if ceil and key in ceil:
            peak = ceil[key]["tflops"] / 3.0
            peak_note = (f"measured in this run: tcgen05.mma kind::tf32 loop on every SM "
                         f"({key}, bench.py --case peaks) {ceil[key]['tflops']} TF / 3 "
                         "(three TF32 MMAs per useful FLOP)")
        else:
            peak = derived
            peak_note = (f"{peaks_kind} bf16 burst {peaks['bf16_tflops']} TF / 2 (TF32 rate) / 3 "
                         "(three TF32 MMAs per useful FLOP)")
        # cuBLAS's own bf16 rate, not the hardware's, halved for tf32
        extra["cublas_derived"] = {"peak": round(derived, 2), "frac": round(gemm_tflops / derived, 4),
                                   "source": f"{peaks_kind} bf16 burst {peaks['bf16_tflops']} TF "
                                             "/ 2 / 3"}
        extra["nominal"] = {"peak": round(1100.0 / 3.0, 1),
                            "frac": round(gemm_tflops / (1100.0 / 3.0), 4),
                            "source": "nominal dense tf32 1.1 PFLOP/s / 3"}
        # dram__bytes_read.sum + dram__bytes_write.sum of one launch of this kernel
        # at 4096^3, from the committed ncu captures
        if pair and tile_n == 256:
            traffic = 695.2e6
            traffic_src = "ncu --set full, profiles/umma_gemm_tf32x3_256x256_sgemm_nn_4096.md"
        elif pair and tile_n == 128:
            traffic = 923.4e6
            traffic_src = "ncu --set full, profiles/umma_gemm_tf32x3_256x128_sgemm_nn_4096.md"
        else:
            traffic_src = "no ncu capture of this tile configuration"
        extra["algorithmic_bytes"] = 4 * 4096 * 4096 * 4 + 4096 * 4096 * 4
    else:
        kernel_name = "FFMA SIMT SGEMM"
        if ceil and "ffma_fp32" in ceil:
            peak = ceil["ffma_fp32"]["tflops"]
            peak_note = "measured in this run: FFMA loop on every SM (bench.py --case peaks)"
        else:
            peak = 148 * 128 * 2 * (peaks.get("sm_max_mhz", 1965.0) * 1e6) / 1e12
            peak_note = "FP32 SIMT nominal: 148 SMs x 128 lanes x 2 FLOP x max SM clock"
    roof = {"bound": "tensor", "kernel": kernel_name, "achieved": round(gemm_tflops, 2),
            "peak": round(peak, 2), "unit": "TFLOP/s", "frac": round(gemm_tflops / peak, 4),
            "kernel_ms": round(gemm_ms, 4),
            "achieved_note": "2*4096^3 FLOP per launch / the GEMM kernel's mean duration "
                             "(CUDA events around it, every timed step); the whole step "
                             "(split pre-pass + GEMM) runs at step_achieved",
            "step_achieved": round(kernel_tflops, 2),
            "peak_source": peak_note, "traffic": traffic, "traffic_unit": "bytes per launch",
            "traffic_source": traffic_src}
    roof.update(extra)
    return roof


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-seconds", type=float, default=60.0,
                    help="--impl reference: host CPU time to spend over all timed steps")
    ap.add_argument("--case", choices=CASES, help="run one case (see run_case) and exit")
    ap.add_argument("--trans", default="t", choices=["t", "n"],
                    help="--case gemv32: hipBLAS transA of the weights (t: N x K rows, n: K x N)")
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--shape", default="", help="--case: M,N,K (default n,n,n)")
    ap.add_argument("--m", type=int, default=1, help="--case gemv/gemv32: tokens")
    ap.add_argument("--splitk", type=int, default=0)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--path", default="auto", choices=["auto", "simt", "tc", "gemv"],
                    help="--case: force a kernel family (vkblas_b200_set_path)")
    ap.add_argument("--kernel-events", action="store_true",
                    help="--case: record the library's kernel events around every call")
    ap.add_argument("--graph", action="store_true",
                    help="--case: capture the --iters calls in a CUDA graph and time 5 replays")
    args = ap.parse_args()
    if args.case:
        return run_case(args)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        ref = CpuReference()
        tfs = []
        for _ in range(args.warmup):
            ref.sample(0.2)
        info = None
        per_step = max(0.2, args.ref_seconds / max(1, args.steps))
        for _ in range(args.steps):
            tf, info = ref.sample(per_step)
            tfs.append(tf)
        v = statistics.median(tfs)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "sgemm_nn_4096^3 (ref_gemm row sample)"},
            "cpu_baseline": dict(value=v, unit="TFLOPS", **info),
            "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return 0

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        # host-side status exchange of the sharded GEMMs (shard.py): a rank's
        # failure reaches the others before any data collective
        status_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
    import vkblas_b200 as vk
    from vkblas_b200 import hipblas as hb
    peaks, peaks_kind = _peaks()

    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    # Two rotating buffer sets: 2 x 192 MB working set > 126 MB L2.
    sets = [(torch.randn(MNK * MNK, device="cuda", generator=g),
             torch.randn(MNK * MNK, device="cuda", generator=g),
             torch.empty(MNK * MNK, device="cuda")) for _ in range(2)]
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    h = hb.Handle()
    h.set_stream(stream)

    def step(i):
        A, B, C = sets[i % 2]
        st = _hip_sgemm(vk, hb, h, A, B, C, al, be)
        if st != 0:
            raise RuntimeError(f"hipblasSgemm status {st}")

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    path = vk.PATH_NAMES[vk.last_path()]
    tile_n, pair, split = vk.last_tile_n(), vk.last_pair(), vk.last_split()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # One event pair per step, recorded by the library around its main kernel
    # (after the 3xTF32 split pre-pass): the GEMM kernel's own duration inside
    # the timed stream of calls, for the roofline.
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for a, b in kev:                   # creates the CUDA events
        a.record(stream)
        b.record(stream)
    torch.cuda.synchronize()
    l0 = vk.launch_count()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, period_s=0.005) as clk:
        e0.record(stream)
        for i in range(args.steps):
            vk.set_kernel_events(*kev[i])
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    vk.set_kernel_events(None, None)
    gemm_ms = sum(a.elapsed_time(b) for a, b in kev) / args.steps
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches = vk.launch_count() - l0
    ms_total = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms_total, gemm_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total, gemm_ms = float(t[0].item()), float(t[1].item())
    ms_step = ms_total / args.steps
    value = world * FLOP_PER_GEMM * args.steps / (ms_total / 1e3) / 1e12

    # e2e through the public ABI with host buffers: every step copies its A and
    # B from pinned host memory, calls hipblasSgemm and copies its C back, all
    # inside the timed region.  Steps rotate over E2E_STREAMS streams, each with
    # its own device buffers and hipBLAS handle, so a step's host-to-device
    # copies overlap earlier steps' GEMMs and device-to-host copies (PCIe is
    # full duplex) -- how a caller streaming GEMMs through host memory runs it.
    # With two streams a step's upload could wait for the download two steps
    # back on its stream; three keep the upload direction busy.
    E2E_STREAMS = 3
    hA = torch.randn(MNK * MNK, generator=torch.Generator().manual_seed(7)).pin_memory()
    hB = torch.randn(MNK * MNK, generator=torch.Generator().manual_seed(8)).pin_memory()
    hCs = [torch.empty(MNK * MNK).pin_memory() for _ in range(E2E_STREAMS)]
    e2e_sets = sets + [(torch.empty(MNK * MNK, device="cuda"), torch.empty(MNK * MNK, device="cuda"),
                        torch.empty(MNK * MNK, device="cuda"))
                       for _ in range(E2E_STREAMS - len(sets))]
    e2e_streams = [torch.cuda.Stream() for _ in range(E2E_STREAMS)]
    e2e_handles = [hb.Handle() for _ in range(E2E_STREAMS)]
    for hh, ss in zip(e2e_handles, e2e_streams):
        hh.set_stream(ss)

    def e2e_step(i):
        j = i % E2E_STREAMS
        dA, dB, dC = e2e_sets[j]
        with torch.cuda.stream(e2e_streams[j]):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            st = _hip_sgemm(vk, hb, e2e_handles[j], dA, dB, dC, al, be)
            if st != 0:
                raise RuntimeError(f"hipblasSgemm status {st}")
            hCs[j].copy_(dC, non_blocking=True)

    def e2e_loop(n):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for ss in e2e_streams:
            ss.wait_event(e0)
        for i in range(n):
            e2e_step(i)
        for ss in e2e_streams:
            done = torch.cuda.Event()
            done.record(ss)
            stream.wait_event(done)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    e2e_steps = max(4, min(args.steps, 20))
    e2e_loop(2)
    if world > 1:
        dist.barrier()
    e2e_ms = e2e_loop(e2e_steps)
    for hh in e2e_handles:
        hh.close()
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = world * FLOP_PER_GEMM / (e2e_ms / 1e3) / 1e12

    # Ceilings of this GPU measured now (tcgen05 tf32 / f16 MMA loops, FFMA
    # loop; about 50 ms): the roofline's denominators.
    try:
        ceil = run_peaks(vk, torch, stream)
    except Exception as exc:      # the derived peaks stand in; the error is reported
        ceil = {"error": repr(exc)}
    roof = _roofline(path, tile_n, pair, split, gemm_ms, ms_step, peaks, peaks_kind,
                     ceil if "error" not in ceil else None)

    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (A,B ~ N(0,1) fp32, seeded per rank)",
        "config": {"workload": "sgemm_nn_4096^3: hipblasSgemm(N, N, 4096, 4096, 4096), "
                               "column-major, alpha=1 beta=0 (BASELINE config 2)",
                   "per_gpu": "one 4096^3 GEMM per step (strided-batched SGEMM sharded by batch)",
                   "parallelism": f"batch-shard x{world}", "path": path,
                   "l2": "2 rotating A/B/C sets (384 MB working set > 126 MB L2)"},
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 3), "unit": "TFLOPS",
                "h2d_bytes_per_step": 2 * MNK * MNK * 4, "d2h_bytes_per_step": MNK * MNK * 4,
                "ms_per_step": round(e2e_ms, 4),
                "pipelining": f"steps rotate over {E2E_STREAMS} streams: a step's H2D copies "
                              "overlap earlier steps' GEMMs and D2H copies"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "measured_ceilings": ceil,
    }
    del sets, e2e_sets, hA, hB, hCs
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, info = CpuReference().sample(8.0)
        result["cpu_baseline"] = dict(value=tf, unit="TFLOPS", **info)
    if rank == 0 and world == 1 and not args.no_secondary:
        try:
            result["secondary"] = secondary_results(vk, hb, torch, peaks,
                                                    ceil if "error" not in ceil else None)
        except Exception as exc:   # secondary numbers never hide the headline
            result["secondary"] = {"error": repr(exc)}
    if world > 1 and not args.no_secondary:
        # every rank takes the same collective steps; an error ends the run
        result["secondary"] = sharded_secondary(vk, torch, dist, rank, world, stream,
                                                status_group, peaks)
        torch.cuda.empty_cache()
    h.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result))
    return 0


if __name__ == "__main__":
    sys.exit(main())
