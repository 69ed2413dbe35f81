"""CPU replay of the B200 kernel's work mapping (paia-project_b200/csrc/gemv_launch.cuh choose_ks / launch_variant and
gemv_kernel.cuh gemv_kernel), in the spirit of the reference's src/tests/emulate_mapping.py: for many shapes and
launch configurations it checks, before anything runs on a GPU, that

  * every (row, 16-byte chunk) of W is loaded exactly once and every load is inside the row and inside W,
  * every output row is stored exactly once, by exactly one lane,
  * x (shared memory) and the per-chunk x sums are read only inside [0, K) and [0, K/32),
  * the cross-warp reduction buffer and the named-barrier ids stay in range,
  * the double-buffered iteration order visits every (tile, batch) exactly once, in order.
"""
import itertools
import random

import numpy as np
import pytest

ELEMS = {"bf16": 8, "fp8": 16, "int4": 32, "int4_asym": 32}
ROWBYTES = {"bf16": lambda K: 2 * K, "fp8": lambda K: K, "int4": lambda K: K // 2, "int4_asym": lambda K: K // 2}


def choose_ks(nchunk, rows_per_cta, W, R, U):
    steps = (nchunk + 31) // 32
    ks_k = 1
    while ks_k * 2 <= W and steps >= ks_k * 2 * U:
        ks_k *= 2
    slots = (rows_per_cta + R - 1) // R
    nr = 1
    while nr * 2 <= W and nr * 2 <= slots:
        nr *= 2
    ks = max(ks_k, W // nr)
    cap = 1
    while cap * 2 <= W and cap * 2 <= steps:
        cap *= 2
    return min(ks, cap)


def grid(N, sms, per_sm):
    return min(sms * per_sm, N)


def iteration_order(nit, nbatch):
    """The (t, b) sequence of the kernel's ping-pong loop, with which buffer is loaded/computed."""
    seq, loads = [], [(0, 0, "a")] if nit > 0 else []
    t = b = it = 0
    while it < nit:
        t1, b1 = t, b + 1
        if b1 == nbatch:
            b1, t1 = 0, t1 + 1
        if it + 1 < nit:
            loads.append((t1, b1, "b"))
        seq.append((t, b, "a"))
        it, t, b = it + 1, t1, b1
        if it >= nit:
            break
        t2, b2 = t, b + 1
        if b2 == nbatch:
            b2, t2 = 0, t2 + 1
        if it + 1 < nit:
            loads.append((t2, b2, "a"))
        seq.append((t, b, "b"))
        it, t, b = it + 1, t2, b2
    return seq, loads


def replay(fmt, N, K, W, R, U, sms=148, per_sm=2, ks=None):
    E = ELEMS[fmt]
    nchunk = ROWBYTES[fmt](K) // 16
    G = grid(N, sms, per_sm)
    rows_per_cta = (N + G - 1) // G
    KS = ks or choose_ks(nchunk, rows_per_cta, W, R, U)
    assert W % KS == 0 and KS & (KS - 1) == 0
    ksl = KS.bit_length() - 1
    NR = W >> ksl
    loads = np.zeros((N, nchunk), dtype=np.int32)
    stores = np.zeros(N, dtype=np.int32)
    lanes = np.arange(32)
    for blk in range(G):
        rb, re = blk * N // G, (blk + 1) * N // G
        tile_rows = NR * R
        ntiles = (re - rb + tile_rows - 1) // tile_rows
        barriers = {}
        for warp in range(W):
            rslot, kslot = warp >> ksl, warp & (KS - 1)
            cb, ce = (nchunk * kslot) >> ksl, (nchunk * (kslot + 1)) >> ksl
            nsteps = (ce - cb + 31) >> 5
            nbatch = (nsteps + U - 1) // U if nsteps > U else 1
            nit = ntiles * nbatch
            seq, lds = iteration_order(nit, nbatch)
            assert [(t, b) for t, b, _ in seq] == [(i // nbatch, i % nbatch) for i in range(nit)]
            assert sorted((t, b) for t, b, _ in lds) == [(t, b) for t, b, _ in seq]
            for t, b, _ in seq:
                for r in range(R):
                    row = rb + t * tile_rows + rslot * R + r
                    if row >= re:
                        continue
                    for u in range(U):
                        c = cb + ((b * U + u) << 5) + lanes
                        c = c[c < ce]
                        assert c.size == 0 or (c.min() >= 0 and c.max() < nchunk)
                        np.add.at(loads[row], c, 1)
                # x reads (only for c < ce): chunk c covers x[c*E, c*E+E)
                for u in range(U):
                    c = cb + ((b * U + u) << 5) + lanes
                    c = c[c < ce]
                    if c.size:
                        assert c.max() * E + E <= K
                        if fmt.startswith("int4"):
                            assert c.max() < K // 32
                if b == nbatch - 1:
                    rl = {1: 0, 2: 1, 4: 2, 8: 3}[R]
                    for lane in range(32):
                        if lane & ((32 >> rl) - 1):
                            continue
                        rr = lane >> (5 - rl)
                        assert 0 <= rr < R and warp * R + rr < W * R
                        if KS > 1:
                            assert 1 + rslot <= 15
                            barriers[(rslot, t)] = barriers.get((rslot, t), 0) + 1
                            if kslot != 0:
                                continue
                        row = rb + t * tile_rows + rslot * R + rr
                        if row < re:
                            stores[row] += 1
        if KS > 1:
            # every warp of a slot arrives once per tile (the leader-lane count is R per warp)
            for (rslot, t), n in barriers.items():
                assert n == KS * R, (rslot, t, n)
    assert np.all(loads == 1), f"{fmt} N={N} K={K} W={W} R={R} U={U}: loads min {loads.min()} max {loads.max()}"
    assert np.all(stores == 1), f"{fmt} N={N} K={K} W={W} R={R} U={U}: stores min {stores.min()} max {stores.max()}"
    return KS


SHAPES = {
    "bf16": [(1, 8), (1, 256), (3, 264), (7, 520), (33, 1032), (129, 4104), (513, 3584), (1000, 3584), (4097, 4096),
             (64, 14336), (300, 18944)],
    "fp8": [(1, 16), (5, 384), (33, 1152), (96, 4096), (513, 3584), (1000, 14336), (4097, 4096)],
    "int4": [(1, 128), (5, 384), (33, 1152), (96, 4096), (513, 3584), (1000, 18944), (4097, 4096)],
}
SHAPES["int4_asym"] = SHAPES["int4"]


@pytest.mark.parametrize("fmt", list(SHAPES))
def test_mapping_exactly_once(fmt):
    Rs = (1, 2, 4, 8) if fmt.startswith("int4") else (1, 2, 4)
    Us = (1, 2, 4, 8) if fmt == "bf16" else (1, 2, 4)
    rnd = random.Random(0)
    combos = list(itertools.product(SHAPES[fmt], (4, 8), Rs, Us, (1, 2, 3)))
    for (N, K), W, R, U, per_sm in rnd.sample(combos, 60):
        replay(fmt, N, K, W, R, U, sms=rnd.choice((148, 7, 1)), per_sm=per_sm)


def test_mapping_explicit_ks():
    for ks in (1, 2, 4, 8):
        replay("int4", 257, 4096, 8, 2, 1, sms=13, per_sm=2, ks=ks)
        replay("bf16", 100, 2048, 8, 1, 2, sms=5, per_sm=1, ks=ks)


def test_choose_ks_real_shapes():
    # INT4 K=4096 rows are 128 chunks (4 steps): with U=1 four warps share a row, each one full 512-byte step.
    assert choose_ks(128, 28, 8, 4, 1) == 4
    # BF16 K=4096 (512 chunks = 16 steps), U=4: four warps per row, each 4 steps (one batch).
    assert choose_ks(512, 28, 8, 2, 4) == 4
    # few rows per CTA push the K-split up, but never past the number of steps
    assert choose_ks(128, 2, 8, 1, 1) == 4
    assert choose_ks(1, 1, 8, 1, 1) == 1


# ------------------------------------------------------------------ tensor-core kernel (gemv_mma.cuh)

MMA_STEP_K = {"bf16": 32, "fp8": 64, "int4": 128, "int4_asym": 128}


def replay_mma(fmt, N, K, W, U, sms=148, per_sm=2):
    """Replay of gemv_mma_kernel: CTA rows, 16-row tiles, 64-byte steps split over warps, lane (g, c) loading the
    16-byte chunk q = 4 s + c of rows g and g + 8, x reads at s * SK + c * SK/4 .. + SK/4 (padded to Kp)."""
    SK = MMA_STEP_K[fmt]
    nchunk = ROWBYTES[fmt](K) // 16
    Kp = (K + SK - 1) // SK * SK
    G = grid(N, sms, per_sm)
    S = (nchunk + 3) // 4
    assert S * SK == Kp, (fmt, K, S, Kp)
    loads = np.zeros((N, nchunk), dtype=np.int32)
    stores = np.zeros(N, dtype=np.int32)
    for blk in range(G):
        rb, re = blk * N // G, (blk + 1) * N // G
        ntiles = (re - rb + 15) >> 4
        arrivals = {}
        for warp in range(W):
            sb, se = S * warp // W, S * (warp + 1) // W
            nbatch = (se - sb + U - 1) // U if (se - sb) > U else 1
            nit = ntiles * nbatch
            seq, lds = iteration_order(nit, nbatch)
            assert [(t, b) for t, b, _ in seq] == [(i // nbatch, i % nbatch) for i in range(nit)]
            for t, b, _ in seq:
                for u in range(U):
                    s = sb + b * U + u
                    if s >= se:
                        continue
                    assert s * SK + SK <= Kp                      # x reads (all lanes c) inside the padded x
                    if fmt.startswith("int4"):
                        assert s < Kp // 128                      # gsum index
                    for g in range(8):
                        for r in (rb + t * 16 + g, rb + t * 16 + g + 8):
                            if r >= re:
                                continue
                            for c in range(4):
                                q = 4 * s + c
                                if q < nchunk:
                                    loads[r, q] += 1
                if b == nbatch - 1:
                    arrivals[t] = arrivals.get(t, 0) + 1
                    if warp == 0:
                        for lane in range(16):
                            r = rb + t * 16 + lane
                            if r < re:
                                stores[r] += 1
        assert all(v == W for v in arrivals.values()) and len(arrivals) == ntiles
    assert np.all(loads == 1), f"{fmt} N={N} K={K} W={W} U={U}: loads min {loads.min()} max {loads.max()}"
    assert np.all(stores == 1), f"{fmt} N={N} K={K} W={W} U={U}: stores"


@pytest.mark.parametrize("fmt", list(SHAPES))
def test_mma_mapping_exactly_once(fmt):
    rnd = random.Random(1)
    combos = list(itertools.product(SHAPES[fmt], (4, 8, 16), (1, 2, 4), (1, 2, 3, 4)))
    for (N, K), W, U, per_sm in rnd.sample(combos, 60):
        replay_mma(fmt, N, K, W, U, sms=rnd.choice((148, 7, 1)), per_sm=per_sm)
