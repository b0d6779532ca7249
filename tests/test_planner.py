"""CPU checks of the GEMM planners and of workspace sizing (no device work).

The planners choose kernels, tiles and reduction splits from a time model
fitted to B200 measurements; the workspace query must cover whatever they
choose, or a split's fp32 partials would overrun the caller's buffer.  These
properties are checked over the benchmark shapes and a seeded spread of
others."""
import ctypes

import numpy as np
import pytest

from reels_b200 import _native as nat
from reels_b200 import build as native_build

SMS = 148


@pytest.fixture(scope="module")
def lib():
    native_build.build()
    return nat.lib()


def q8(lib, M, Nout, Kred, act=0):
    info = (ctypes.c_int64 * 7)()
    assert lib.reels_q8_plan(M, Nout, Kred, act, SMS, info) == 0
    return dict(zip(["kernel", "tokens", "stage", "splits", "kb_per", "ntiles", "mtiles"], list(info)))  # kb_per: stages


def sk(lib, rows, red, r):
    info = (ctypes.c_int64 * 2)()
    assert lib.reels_sk_plan(rows, red, r, SMS, info) == 0
    return info[0], info[1]


def test_bench_shapes_take_the_256_token_tmem_tiles(lib):
    # Wan 1.3B block linears at 32760 tokens: forward (Nout = N) and dX (Nout = K)
    for M, K, N in [(32760, 1536, 1536), (32760, 1536, 8960), (32760, 8960, 1536)]:
        for Nout, Kred in ((N, K), (K, N)):
            p = q8(lib, M, Nout, Kred)
            assert p["kernel"] in (1, 2) and p["tokens"] == 256 and p["splits"] == 1, (M, Nout, Kred, p)
            assert p["ntiles"] == -(-Nout // 128) and p["mtiles"] == -(-M // 256)


def test_small_token_counts_take_the_wide_stage_tiles(lib):
    # the Wan 2.1 14B FFN up-projection at 128 tokens: one 128-token tile, 128-wide stages
    p = q8(lib, 128, 13824, 5120)
    assert p["kernel"] in (1, 2) and p["tokens"] == 128 and p["stage"] == 128
    assert p["splits"] * p["kb_per"] * p["stage"] >= 5120  # the splits cover the reduction


def test_splits_cover_the_reduction_exactly(lib):
    rng = np.random.default_rng(0)
    for _ in range(300):
        M = int(rng.integers(1, 40000))
        Nout = 16 * int(rng.integers(1, 1200))
        Kred = 16 * int(rng.integers(1, 1200))
        for act in (0, 1):
            p = q8(lib, M, Nout, Kred, act)
            kb = -(-Kred // p["stage"])
            assert p["splits"] >= 1 and p["kb_per"] >= 1
            assert (p["splits"] - 1) * p["kb_per"] < kb <= p["splits"] * p["kb_per"], (M, Nout, Kred, p)


def test_workspace_covers_every_split(lib):
    """reels_q8lora_workspace_bytes >= the fp32 partials of the splits the
    planners pick, for both passes, with and without the fused activation."""
    rng = np.random.default_rng(1)
    shapes = [(128, 5120, 13824, 8), (512, 5120, 13824, 64), (32760, 1536, 8960, 32), (96, 3072, 256, 8)]
    for _ in range(200):
        shapes.append((int(rng.integers(1, 9000)), 16 * int(rng.integers(1, 700)), 16 * int(rng.integers(1, 700)),
                       int(rng.integers(0, 257))))
    for M, K, N, r in shapes:
        np_ = max(16, -(-max(r, 1) // 16) * 16)
        for pas in (nat.PASS_FORWARD, nat.PASS_BACKWARD):
            ws = lib.reels_q8lora_workspace_bytes(M, K, N, r, nat.BF16, pas)
            need = 0
            q8_shapes = [(M, N, K)] if pas == nat.PASS_FORWARD else [(M, K, N)]
            for rows, cols, red in q8_shapes:
                for act in (0, 1):
                    p = q8(lib, rows, cols, red, act)
                    if p["splits"] > 1:
                        need = max(need, p["splits"] * rows * cols * 4)
                    if p["kernel"] == 2:  # stream-K: flags and one accumulator tile per CTA
                        need = max(need, 256 + SMS * 128 * p["tokens"] * 4)
            if r > 0:
                sk_shapes = [(M, K)] if pas == nat.PASS_FORWARD else [(M, K), (M, N), (K, M), (N, M)]
                for rows, red in sk_shapes:
                    splits, _ = sk(lib, rows, red, r)
                    if splits > 1:
                        need = max(need, splits * rows * np_ * 4)
            assert ws >= need, (M, K, N, r, pas, ws, need)


def test_small_token_counts_fill_the_gpu_with_stream_k(lib):
    """At 128 tokens the 13824-row weight makes 108 tiles for 148 SMs (and dX
    40): the planner hands out (tile, stage) units evenly instead."""
    assert q8(lib, 128, 13824, 5120)["kernel"] == 2
    assert q8(lib, 128, 5120, 13824)["kernel"] == 2


def test_plan_queries_reject_bad_arguments(lib):
    info = (ctypes.c_int64 * 7)()
    assert lib.reels_q8_plan(0, 16, 16, 0, SMS, info) == nat.EINVAL
    assert lib.reels_q8_plan(16, 16, 16, 5, SMS, info) == nat.EINVAL
    assert lib.reels_q8_plan(16, 16, 16, 0, SMS, None) == nat.EINVAL
    assert lib.reels_sk_plan(16, 16, 300, SMS, info) == nat.EINVAL


def _sk_pieces(T, U, kb_total, tdp, W, G, b):
    """The device's ts_piece sequence for CTA b (q8ts_gemm.cuh), restated:
    (tile, first unit, end unit, give, take) per piece."""
    out = []
    dp = tdp // G
    for idx in range(dp):
        out.append((b + idx * G, 0, U, 0, 0))
    s, e = b * W // G, (b + 1) * W // G
    idx = dp
    while True:
        tr = s // U + (idx - dp)
        if s >= e or tr * U >= e:
            break
        lo, hi = max(s, tr * U) - tr * U, min(e, (tr + 1) * U) - tr * U
        take = 0
        if lo == 0 and hi < U:
            x = (tr + 1) * U - 1
            bl = x * G // W
            while bl + 1 < G and (bl + 1) * W // G <= x:
                bl += 1
            while bl > 0 and bl * W // G > x:
                bl -= 1
            take = bl - b
        out.append((tdp + tr, lo, hi, 1 if lo > 0 else 0, take))
        idx += 1
    return out


def test_stream_k_schedule_covers_every_unit_once():
    rng = np.random.default_rng(5)
    shapes = [(108, 41), (40, 109), (320, 9), (1536, 25), (148, 1), (149, 3), (300, 17)]
    shapes += [(int(rng.integers(1, 700)), int(rng.integers(1, 120))) for _ in range(200)]
    for T, U in shapes:
        for G in (148, 132, 7):
            tdp = (T // G - 1) * G if T >= 2 * G else 0
            W = (T - tdp) * U
            if W < G:
                continue
            cover = {}
            pieces = {b: _sk_pieces(T, U, U - 1, tdp, W, G, b) for b in range(G)}
            for b, ps in pieces.items():
                assert sum(p[3] for p in ps) <= 1                      # at most one handed-over piece
                if any(p[3] for p in ps):
                    assert ps[len([q for q in ps if q[2] - q[1] == U and q[3] == 0 and q[4] == 0 and
                                   q[0] < tdp])][3] == 1               # ... and it is the first stream-K piece
                for (t, lo, hi, give, take) in ps:
                    assert 0 <= lo < hi <= U and 0 <= t < T
                    for u in range(lo, hi):
                        assert (t, u) not in cover
                        cover[(t, u)] = b
                    if take:
                        # the next `take` CTAs hold this tile's remaining units, each as a handed-over piece
                        assert lo == 0 and hi < U
                        rest = [p for k in range(1, take + 1) for p in pieces[b + k] if p[0] == t]
                        assert all(p[3] == 1 for p in rest) and len(rest) == take
                        assert sorted((p[1], p[2]) for p in rest)[-1][1] == U
            assert len(cover) == T * U, (T, U, G)
