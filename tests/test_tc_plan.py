"""Tile and split planning of the tcgen05 GEMM, as pure host logic (no GPU).

vkblas_b200_tc_plan reports, for an engine call, the tiles the kernel runs
and how the tiles of the last, partial wave are cut along K -- the B200
counterpart of the reference's split-K gate (src/vkblas.c:2850-2867: split
when there are few tiles and K is long).  The GPU tests check the same plan
from the launch side (vkblas_b200_last_split / last_pair / last_tile_n);
these check it without a device: pinned plans for the BASELINE configurations
and the shapes whose split timings are recorded in the design notes, and
invariants over a seeded sweep.
"""
import numpy as np
import pytest

import vkblas_b200 as vk

F32, F16, BF16 = vk.DT_F32, vk.DT_F16, vk.DT_BF16
SMS = 148


def _plan(dt, oa, ob, M, N, K, batch=1, sms=SMS, wide=True):
    return vk.tc_plan(dt, oa, ob, M, N, K, batch, sms, wide)


@pytest.mark.parametrize("name, call, want", [
    # BASELINE config 2, SGEMM 4096^3 NN: 256x256 pair tiles, 256 tiles on 74 SM
    # pairs -> 3 full waves and 34 tiles cut into 2 K ranges of 64 k-blocks.
    ("sgemm_4096_wide", (F32, 0, 0, 4096, 4096, 4096),
     dict(tile_m=256, tile_n=256, pair=1, transposed=0, tiles=256, full_tiles=222, splits=2,
          kblocks=128, kblocks_per_split=64, partial_bytes=34 * 2 * 256 * 256 * 4)),
    # the same with 256x128 tiles: 512 tiles, 68 in the last wave, no split
    ("sgemm_4096_narrow", (F32, 0, 0, 4096, 4096, 4096, 1, SMS, False),
     dict(tile_m=256, tile_n=128, pair=1, tiles=512, full_tiles=512, splits=1, kblocks=128)),
    # BASELINE config 3, HGEMM T/N 4096^3: a split would save 32 k-blocks, fewer
    # than 48, so the 34 tiles of the last wave run whole (no narrow tail either)
    ("hgemm_4096", (F16, 1, 0, 4096, 4096, 4096),
     dict(tile_m=256, tile_n=256, pair=1, tiles=256, full_tiles=256, splits=1, kblocks=64,
          tail_tiles=0)),
    # HGEMM 16384^3: 4096 pair tiles; where a 2-way K split of the 26 left over
    # would pay, they run as 52 halves instead (the narrow tail)
    ("hgemm_16384", (F16, 1, 0, 16384, 16384, 16384),
     dict(tiles=4096, full_tiles=4070, splits=1, kblocks=256, tail_tiles=26)),
    # HGEMM 8192^3: 62 tiles in the last wave, more than half the pairs: whole tiles
    ("hgemm_8192", (F16, 1, 0, 8192, 8192, 8192),
     dict(tiles=1024, full_tiles=1024, splits=1, tail_tiles=0)),
    # one pair tile, long K: 16 K ranges of 4 k-blocks (recorded split: S = 16)
    ("hgemm_256x256x4096", (F16, 0, 1, 256, 256, 4096),
     dict(tile_m=256, tile_n=256, pair=1, tiles=1, full_tiles=0, splits=16, kblocks=64,
          kblocks_per_split=4)),
    # fp32 splits keep whole 8-k-block accumulation segments
    ("sgemm_512x512x8192", (F32, 0, 0, 512, 512, 8192),
     dict(tile_m=256, tile_n=256, tiles=4, full_tiles=0, splits=16, kblocks=256,
          kblocks_per_split=16)),
    # BASELINE config 4 at M = 16: decode runs transposed (weight rows on the
    # MMA lanes, tokens on a 64-wide tile), 112 tiles on 148 SMs, no split
    ("decode_m16", (F16, 0, 1, 16, 14336, 4096),
     dict(tile_m=128, tile_n=64, transposed=1, pair=0, tiles=112, full_tiles=112, splits=1)),
    # BASELINE config 5, 256 x 2048^3: 16384 pair tiles; 30 left over, a split
    # would save only 16 k-blocks, so they run whole
    ("batched_256x2048", (F16, 0, 0, 2048, 2048, 2048, 256),
     dict(tile_m=256, tile_n=256, pair=1, tiles=16384, full_tiles=16384, splits=1,
          tail_tiles=0)),
    # 75 pair tiles of K = 4096 (the GPU wave-tail test): fewer than 8 waves,
    # so the last one is split along K
    ("hgemm_wave_tail", (F16, 0, 0, 256, 40, 4096, 75),
     dict(tiles=75, full_tiles=74, splits=16, tail_tiles=0)),
    # 1186 pair tiles (16 waves + 2) of K = 3584: the 2 left over as halves
    ("hgemm_narrow_tail", (F16, 0, 0, 256, 320, 3584, 593),
     dict(tiles=1186, full_tiles=1184, splits=1, tail_tiles=2)),
    # M < 256: single-CTA tiles
    ("sgemm_200x300", (F32, 0, 0, 200, 300, 136),
     dict(tile_m=128, tile_n=128, pair=0, tiles=6, splits=1)),
])
def test_pinned_plans(name, call, want):
    got = _plan(*call)
    for k, v in want.items():
        assert got[k] == v, f"{name}: {k} = {got[k]}, want {v} ({got})"


def _check_invariants(dt, oa, ob, M, N, K, batch, sms, wide):
    p = _plan(dt, oa, ob, M, N, K, batch, sms, wide)
    assert p["tile_m"] in (128, 256) and (p["pair"] == 1) == (p["tile_m"] == 256)
    assert p["transposed"] == (1 if dt != F32 and M <= 64 and N >= 128 else 0)
    if p["transposed"]:
        assert dt != F32 and M <= 64 and N >= 128
        assert (p["tile_m"], p["tile_n"], p["pair"]) == (128, 64, 0)
        mq, nq = N, M
    else:
        mq, nq = M, N
        assert p["tile_n"] == (256 if dt != F32 else (256 if wide and p["pair"] and N >= 256 else 128))
        assert p["pair"] == (1 if M >= 256 else 0)
    tiles = -(-mq // p["tile_m"]) * -(-nq // p["tile_n"]) * batch
    assert p["tiles"] == tiles
    assert p["kblocks"] == -(-K // (32 if dt == F32 else 64))
    workers = sms // 2 if p["pair"] else sms
    tail = p["tail_tiles"]
    if tail:
        # narrow tail: 2-byte 256x256 pair tiles, 8 waves or more, a last
        # wave that fills at most half of the SM pairs, and a K split that
        # would have paid; no K split then
        assert dt != F32 and p["pair"] and p["tile_n"] == 256 and not p["transposed"]
        assert p["splits"] == 1 and p["partial_bytes"] == 0
        assert tiles >= 8 * workers and tail == tiles % workers and 2 * tail <= workers
        assert p["full_tiles"] == tiles - tail
        return p
    if p["splits"] == 1:
        assert p["full_tiles"] == tiles and p["partial_bytes"] == 0
        return p
    s, kbps, kb = p["splits"], p["kblocks_per_split"], p["kblocks"]
    assert 2 <= s <= 16
    assert (s - 1) * kbps < kb <= s * kbps, "K ranges cover the k-blocks exactly once"
    assert kbps >= (8 if dt == F32 else 4)
    if dt == F32:
        assert kbps % 8 == 0, "fp32 K ranges hold whole accumulation segments"
    rem = tiles - p["full_tiles"]
    assert 0 < rem < workers and p["full_tiles"] % workers == 0, "only the last wave is split"
    min_saved = 16 if dt == F32 else (8 if p["tile_n"] == 64 else 48)
    assert kb - kbps >= min_saved
    assert p["partial_bytes"] == rem * s * p["tile_m"] * p["tile_n"] * 4
    return p


def test_invariants_over_a_seeded_sweep():
    rng = np.random.default_rng(7)
    splits = tails = 0
    for _ in range(600):
        dt = int(rng.choice([F32, F16, BF16]))
        M = int(rng.choice([int(rng.integers(1, 65)), int(rng.integers(65, 5000))]))
        N = int(rng.integers(1, 9000))
        K = int(rng.choice([int(rng.integers(1, 512)), int(rng.integers(512, 40000))]))
        batch = int(rng.choice([1, 1, 1, int(rng.integers(2, 300))]))
        sms = int(rng.choice([148, 132, 148, 8, 2]))
        p = _check_invariants(dt, int(rng.integers(0, 2)), int(rng.integers(0, 2)), M, N, K,
                              batch, sms, bool(rng.integers(0, 2)))
        splits += p["splits"] > 1
        tails += p["tail_tiles"] > 0
    assert splits > 50, "the sweep reaches the split rule"
    assert tails > 5, "the sweep reaches the narrow tail"


def test_rejects_bad_arguments():
    for args in ((F32, 0, 0, 0, 8, 8, 1, SMS), (F32, 0, 0, 8, 8, 8, 0, SMS),
                 (F32, 0, 0, 8, 8, 8, 1, 0), (7, 0, 0, 8, 8, 8, 1, SMS)):
        with pytest.raises(vk.VkblasError):
            vk.tc_plan(*args)


def test_rejects_tile_counts_the_launch_path_rejects():
    """2^31 tiles or more: the tensor-core launch refuses the call, so the plan
    query reports VKBLAS_ERR_PARAM instead of a truncated tile count."""
    for dt in (F32, F16):
        with pytest.raises(vk.VkblasError):
            vk.tc_plan(dt, 0, 0, 4096, 4096, 64, 1 << 24, SMS)     # 16 x 16 x 2^24 = 2^32 tiles
    p = vk.tc_plan(F16, 0, 0, 4096, 4096, 64, (1 << 23) - 1, SMS)  # just under 2^31
    assert p["tiles"] == 256 * ((1 << 23) - 1)
