"""Replicated-output GEMM (vkblas_b200_gemm_replicated) on one B200.

The peer copies are other buffers on the same GPU: the kernel's stores to a
peer are plain global stores to an address, and an address on this GPU
exercises the same epilogue code as one mapped from another GPU.  Every case
fills the peers with a NaN sentinel first and checks, through the C ABI:

* C is within the oracle's tolerance (relative Frobenius error <= 2e-3 fp16,
  8e-3 bf16, 1e-5 fp32 on 3xTF32) and bit for bit equal to the regular
  engine call on the tensor-core path (same kernel, same tiles and splits:
  the peer stores change nothing in what C receives);
* every peer holds C's bits at every element of the problem, and the
  sentinel everywhere else (ldc padding, gaps between batch entries);
* the tile plan (CTA pairs, K splits reported by vkblas_b200_last_pair /
  last_split) is the regular call's and vkblas_b200_tc_plan's, so the cases
  cover pair, single-CTA and split-reduce epilogues;
* the epilogue that stages C boxes in shared memory and stores them with TMA
  gives the same bits as the one that stores straight from registers
  (VKBLAS_EPI_TMA=0), each run in its own process;
* a problem the replicated kernel does not take (small-M transposed) returns
  VKBLAS_ERR_FALLBACK with C and the peers untouched; more than 7 peers and a
  null peer are VKBLAS_ERR_PARAM.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import check_status  # noqa: E402

KIND = {vk.DT_F16: 0, vk.DT_BF16: 1, vk.DT_F32: 2}
SENTINEL = {vk.DT_F16: 0x7E00, vk.DT_BF16: 0x7FC0, vk.DT_F32: 0x7FC00000}
TOL = {vk.DT_F16: 2e-3, vk.DT_BF16: 8e-3, vk.DT_F32: 1e-5}

# dtype, op_a, op_b, M, N, K, batch, ldc pad, sc pad, peers.  Their tile plans
# (vkblas_b200_tc_plan on 148 SMs): pairs without a split, pairs with a K
# split, single CTAs with and without one, 128- and 256-wide fp32 tiles.
CASES = [
    (vk.DT_F16, 0, 1, 512, 512, 256, 1, 0, 0, 2),        # pairs
    (vk.DT_BF16, 0, 1, 256, 256, 4096, 1, 0, 0, 3),      # pair tile split 16 ways
    (vk.DT_F32, 0, 0, 192, 320, 256, 1, 0, 0, 1),        # 3xTF32 128 x 128 tiles
    (vk.DT_F32, 0, 0, 128, 384, 1024, 1, 0, 0, 2),       # 3xTF32 single CTAs, split 4 ways
    (vk.DT_F32, 1, 0, 1024, 1024, 512, 1, 0, 0, 7),      # 3xTF32 256 x 256 pairs, 7 peers
    (vk.DT_F16, 0, 0, 160, 136, 128, 3, 8, 24, 2),       # batch, padded ldc, single CTAs
    (vk.DT_F32, 0, 1, 300, 200, 96, 2, 3, 5, 1),         # scalar stores (odd ldc)
    (vk.DT_F16, 1, 1, 128, 100, 64, 1, 0, 0, 1),         # scalar stores (N % 8)
    (vk.DT_BF16, 0, 1, 200, 100, 64, 1, 4, 0, 2),        # N % 8 with aligned ldc: direct stores
    (vk.DT_BF16, 0, 1, 200, 104, 64, 1, 8, 0, 2),        # staged boxes, ragged N chunk and M
]


def _rand(dtype, n, rng):
    x = rng.uniform(-1, 1, n).astype(np.float32)
    return x if dtype == vk.DT_F32 else orc.narrow(KIND[dtype], x)


def _to_dev(dtype, arr):
    import torch
    a = np.ascontiguousarray(arr)
    if dtype == vk.DT_F32:
        return torch.from_numpy(a.view(np.int32)).cuda().view(torch.float32)
    t = torch.from_numpy(a.view(np.int16)).cuda()
    return t.view(torch.bfloat16 if dtype == vk.DT_BF16 else torch.float16)


def _bits(dtype, t):
    import torch
    if dtype == vk.DT_F32:
        return t.view(torch.int32).cpu().numpy().view(np.uint32)
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _sentinel_buf(dtype, n):
    bits = np.full(n, SENTINEL[dtype], np.uint32 if dtype == vk.DT_F32 else np.uint16)
    return _to_dev(dtype, bits)


def _problem(dtype, op_a, op_b, M, N, K, batch, ldc_pad, sc_pad, seed):
    rng = np.random.default_rng(seed)
    ra, ca = (K, M) if op_a else (M, K)
    rb, cb = (N, K) if op_b else (K, N)
    lda, ldb, ldc = ca, cb, N + ldc_pad
    sa, sb, sc = ra * lda, rb * ldb, M * ldc + sc_pad
    A = _rand(dtype, sa * batch, rng)
    B = _rand(dtype, sb * batch, rng)
    C0 = _rand(dtype, sc * batch, rng)
    return A, B, C0, lda, ldb, ldc, sa, sb, sc


def _written(M, N, ldc, sc, batch):
    mask = np.zeros(sc * batch, bool)
    for b in range(batch):
        idx = b * sc + np.arange(M)[:, None] * ldc + np.arange(N)[None, :]
        mask[idx.ravel()] = True
    return mask


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_replicated_gemm_matches_engine_and_fills_peers(case, cuda):
    import torch
    dtype, op_a, op_b, M, N, K, batch, ldc_pad, sc_pad, npeers = case
    plan = vk.tc_plan(dtype, op_a, op_b, M, N, K, batch,
                      num_sms=torch.cuda.get_device_properties(0).multi_processor_count)
    A, B, C0, lda, ldb, ldc, sa, sb, sc = _problem(dtype, op_a, op_b, M, N, K, batch, ldc_pad,
                                                   sc_pad, 7 * M + N)
    alpha, beta = 1.25, -0.5
    dA, dB = _to_dev(dtype, A), _to_dev(dtype, B)
    dC, dR = _to_dev(dtype, C0), _to_dev(dtype, C0)
    peers = [_sentinel_buf(dtype, C0.size) for _ in range(npeers)]
    stream = torch.cuda.current_stream()
    st = vk.gemm_replicated(dtype, op_a, op_b, M, N, K, alpha, dA.data_ptr(), lda, dB.data_ptr(),
                            ldb, beta, dC.data_ptr(), ldc, [p.data_ptr() for p in peers], batch,
                            sa, sb, sc, stream=stream)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK
    check_status()
    assert vk.last_path() == vk.PATH_TC
    rep_plan = (vk.last_pair(), vk.last_split())
    vk.set_path(vk.PATH_TC)
    try:
        vk.set_stream(stream)
        st = vk.gemm(dtype, op_a, op_b, M, N, K, alpha, dA.data_ptr(), lda, dB.data_ptr(), ldb,
                     beta, dR.data_ptr(), ldc, batch, sa, sb, sc)
        torch.cuda.synchronize()
    finally:
        vk.set_path(vk.PATH_AUTO)
    assert st == vk.VKBLAS_OK
    assert rep_plan == (vk.last_pair(), vk.last_split()), "the replicated call ran another plan"
    assert rep_plan == (plan["pair"], plan["splits"]), (rep_plan, plan)
    got = _bits(dtype, dC)
    assert np.array_equal(got, _bits(dtype, dR)), "C differs from the regular engine call"
    mask = _written(M, N, ldc, sc, batch)
    for j, p in enumerate(peers):
        pb = _bits(dtype, p)
        assert np.array_equal(pb[mask], got[mask]), f"peer {j} differs from C"
        assert (pb[~mask] == SENTINEL[dtype]).all(), f"peer {j} written outside the problem"
    assert np.array_equal(got[~mask], C0.view(got.dtype)[~mask]), "C padding was written"
    if dtype == vk.DT_F32:
        want = orc.gemm_rowmajor_f64(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C0, ldc,
                                     batch, sa, sb, sc)
        vals = got.view(np.float32)
    else:
        want = orc.hgemm_rowmajor_f64(KIND[dtype], op_a, op_b, M, N, K, alpha, A, lda, B, ldb,
                                      beta, C0, ldc, batch, sa, sb, sc)
        vals = orc.widen(KIND[dtype], got)
    out = np.stack([vals[b * sc: b * sc + M * ldc].reshape(M, ldc)[:, :N] for b in range(batch)])
    err = orc.rel_frobenius(out, np.asarray(want).reshape(batch, M, N))
    assert err <= TOL[dtype], f"relative error {err}"


def test_replicated_gemm_declines_and_rejects(cuda):
    import torch
    dtype, M, N, K = vk.DT_F16, 16, 256, 128          # small-M: runs transposed elsewhere
    A, B, C0, lda, ldb, ldc, sa, sb, sc = _problem(dtype, 0, 1, M, N, K, 1, 0, 0, 3)
    dA, dB, dC = _to_dev(dtype, A), _to_dev(dtype, B), _to_dev(dtype, C0)
    peers = [_sentinel_buf(dtype, C0.size) for _ in range(8)]
    ptrs = [p.data_ptr() for p in peers]
    n0 = vk.launch_count()

    def call(pp):
        st = vk.gemm_replicated(dtype, 0, 1, M, N, K, 1.0, dA.data_ptr(), lda, dB.data_ptr(), ldb,
                                0.0, dC.data_ptr(), ldc, pp, stream=torch.cuda.current_stream())
        torch.cuda.synchronize()
        return st
    assert call(ptrs[:1]) == vk.VKBLAS_ERR_FALLBACK
    assert call(ptrs) == vk.VKBLAS_ERR_PARAM                    # 8 peers
    assert call([ptrs[0], 0]) == vk.VKBLAS_ERR_PARAM            # a null peer
    assert vk.launch_count() == n0, "a declined call launched a kernel"
    assert np.array_equal(_bits(dtype, dC), C0)
    for p in peers:
        assert (_bits(dtype, p) == SENTINEL[dtype]).all()
    check_status()


_STAGED_SCRIPT = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import vkblas_b200 as vk
from oracle import oracle as orc
out = {}
# dtype, op_a, op_b, M, N, K, batch, ldc, sc
for i, (dt, oa, ob, M, N, K, batch, ldc, sc) in enumerate([
        (vk.DT_F16, 0, 0, 512, 512, 256, 1, 512, 0),
        (vk.DT_BF16, 0, 1, 160, 136, 128, 3, 144, 160 * 144 + 24),
        (vk.DT_F16, 1, 0, 200, 104, 64, 1, 112, 0),
        (vk.DT_BF16, 0, 1, 384, 640, 512, 2, 648, 384 * 648 + 8)]):
    rng = np.random.default_rng(i)
    kind = 1 if dt == vk.DT_BF16 else 0
    ra, ca = (K, M) if oa else (M, K)
    rb, cb = (N, K) if ob else (K, N)
    sa, sb = ra * ca, rb * cb
    A = orc.narrow(kind, rng.uniform(-1, 1, sa * batch).astype(np.float32))
    B = orc.narrow(kind, rng.uniform(-1, 1, sb * batch).astype(np.float32))
    C = orc.narrow(kind, rng.uniform(-1, 1, max(sc, M * ldc) * batch).astype(np.float32))
    tdt = torch.bfloat16 if kind else torch.float16
    d = [torch.from_numpy(x.view(np.int16)).cuda().view(tdt) for x in (A, B, C)]
    vk.set_stream(torch.cuda.current_stream())
    vk.set_path(vk.PATH_TC)
    st = vk.gemm(dt, oa, ob, M, N, K, 1.25, d[0].data_ptr(), ca, d[1].data_ptr(), cb, -0.5,
                 d[2].data_ptr(), ldc, batch, sa, sb, sc)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK and vk.last_path() == vk.PATH_TC, (i, st, vk.last_path())
    assert vk.device_status(True) == 0
    out[f"c{i}"] = d[2].view(torch.int16).cpu().numpy()
np.savez(sys.argv[2], **out)
"""


def test_staged_epilogue_matches_direct_stores(cuda, tmp_path):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = {}
    for flag in ("1", "0"):
        path = str(tmp_path / f"c_{flag}.npz")
        r = subprocess.run([sys.executable, "-c", _STAGED_SCRIPT, root, path], capture_output=True,
                           text=True, timeout=300, env=dict(os.environ, VKBLAS_EPI_TMA=flag))
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        res[flag] = np.load(path)
    for k in res["1"].files:
        assert np.array_equal(res["1"][k], res["0"][k]), f"{k}: staged and direct epilogues differ"
