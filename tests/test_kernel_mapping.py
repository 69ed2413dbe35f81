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
    """Replay of gemv_mma_kernel (stream-K inside the CTA): CTA rows [rb, re) cut into 16-row tiles, the T x S
    (tile, step) space split into NW equal warp ranges, iterations of <= U steps that never cross a tile, loads of
    chunk q = 4 s + c of rows g and g + 8 (clamped to the CTA's last row), whole tiles stored by their warp, and the
    straddling tiles finished by the cleanup pass from the partial-sum slots."""
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
        T = (re - rb + 15) >> 4
        total = T * S
        contrib = {}                                          # (tile, row) -> steps summed into it
        slots = {}
        for warp in range(W):
            wb, we = total * warp // W, total * (warp + 1) // W
            first_tile = wb // S if S else 0

            def it_n(cur):
                return min(S - cur % S, U, we - cur)

            cur, seg_s = wb, -1
            prev_next = None
            while cur < we:
                t, s, n = cur // S, cur % S, it_n(cur)
                assert 1 <= n <= U and s + n <= S
                if prev_next is not None:
                    assert prev_next == cur                   # the prefetched iteration is the next computed one
                for g in range(8):
                    for r in (rb + t * 16 + g, rb + t * 16 + g + 8):
                        rc = min(r, re - 1)
                        assert rb <= rc < re
                        for u in range(n):
                            assert (s + u) * SK + SK <= Kp        # x reads inside the padded x
                            if fmt.startswith("int4"):
                                assert s + u < Kp // 128          # gsum / scale group index
                            for c in range(4):
                                q = 4 * (s + u) + c
                                if q < nchunk:
                                    assert 0 <= rc * nchunk + q < N * nchunk
                                    if r < re:
                                        loads[r, q] += 1
                if seg_s < 0:
                    seg_s = s
                if s + n == S or cur + n == we:
                    whole = seg_s == 0 and s + n == S
                    for g in range(16):
                        r = rb + t * 16 + g
                        if whole:
                            if r < re:
                                stores[r] += 1
                        else:
                            slot = (warp, 0 if t == first_tile else 1)
                            assert (slot, g) not in slots, "a partial slot written twice"
                            slots[(slot, g)] = t
                    seg_s = -1
                prev_next = cur + n
                cur += n
        # cleanup pass: straddling tiles, summed from the slots of the warps that touched them
        for w in range(1, W):
            bw = total * w // W
            if bw % S == 0 or bw >= total:
                continue
            t = bw // S
            if total * (w - 1) // W > t * S:
                continue
            for r in range(16):
                used = 0
                for v2 in range(w - 1, W):
                    vb, ve = total * v2 // W, total * (v2 + 1) // W
                    if vb >= (t + 1) * S:
                        break
                    if ve <= t * S or vb >= ve:
                        continue
                    slot = (v2, 0 if t == vb // S else 1)
                    assert slots.get((slot, r)) == t, (blk, w, t, v2, slot)
                    used += 1
                assert used >= 2
                row = rb + t * 16 + r
                if row < re:
                    stores[row] += 1
    assert np.all(loads == 1), f"{fmt} N={N} K={K} W={W} U={U}: loads min {loads.min()} max {loads.max()}"
    assert np.all(stores == 1), f"{fmt} N={N} K={K} W={W} U={U}: stores min {stores.min()} max {stores.max()}"


@pytest.mark.parametrize("fmt", list(SHAPES))
def test_mma_mapping_exactly_once(fmt):
    rnd = random.Random(1)
    combos = list(itertools.product(SHAPES[fmt], (4, 8, 16), (1, 2, 4), (1, 2, 3, 4)))
    for (N, K), W, U, per_sm in rnd.sample(combos, 60):
        replay_mma(fmt, N, K, W, U, sms=rnd.choice((148, 7, 1)), per_sm=per_sm)


# ------------------------------------------------------------------ TMA-fed tensor-core kernel (gemv_tma.cuh)

SMEM_CAP = 232448                                             # B200 opt-in shared memory per block
SM_SMEM = 232448                                              # per SM, less one CTA's reservation


def share_cap(share):
    return min(SMEM_CAP, SM_SMEM // share - (1024 if share > 1 else 0))


def tma_meta_row(cs):
    return (cs + 3) & ~1


def tma_meta_bytes(fmt, cs):
    i4 = 16 * tma_meta_row(cs) * 2 * (2 if fmt == "int4_asym" else 1) if fmt.startswith("int4") else 0
    return (112 + i4 + 15) // 16 * 16


def tma_part_bufs(ring, nch):
    return (ring - 1 + nch - 1) // nch + 2


def tma_smem_bytes(fmt, NC, K, ring, nch, kc, st_bytes, dec=0):
    SK = MMA_STEP_K[fmt]
    kp = (K + SK - 1) // SK * SK
    nb = tma_part_bufs(max(ring, 2), nch)
    i4 = fmt.startswith("int4")
    return (640 + ring * (st_bytes + tma_meta_bytes(fmt, kc // 64)) + kp * (3 if i4 and dec == 2 else 2) + 64
            + (kp // 128 * (8 if dec == 2 else 2) * 4 if i4 else 0) + nb * NC * 16 * 4 + 160)


def tma_prep(fmt, NC, K, ring=0, cap=SMEM_CAP, dec=0, ops=None):
    """Mirror of tma_prep<F, NC>: (kc, nch, rs, st_bytes, ring, smem) or None when the shape cannot be staged.
    Layer mode (`ops`: a list of (N, K)): K is the largest K, one chunk size for all ops, nch the smallest op NCH, and
    a seventh element, the list of per-op NCH."""
    if ops:
        K = max(k for _, k in ops)
    rowbytes = ROWBYTES[fmt](K)
    if ring == 1 or ring > 16:
        return None
    fixed = tma_smem_bytes(fmt, NC, K, 0, 1, 64, 0, dec) + 3 * (NC * 64 + 4)
    if fixed >= cap:
        return None
    per_stage_cap = (cap - fixed) // (ring if ring >= 2 else 3)
    if per_stage_cap < 1536 + 17 * 64:
        return None
    kc_max = min((per_stage_cap - 1536) // 17, 65536 // 16)
    if fmt.startswith("int4"):
        kc_max = min(kc_max, 2048)
    kc_max = kc_max // 64 * 64
    if kc_max < 64:
        return None
    need = (rowbytes + 63) // 64 * 64
    kc0 = min(need, kc_max)
    nch = (rowbytes + kc0 - 1) // kc0
    kc = ((rowbytes + nch - 1) // nch + 63) // 64 * 64
    op_nch = None
    if ops:
        best = -1.0
        for c in range(kc0, max(kc_max // 4, 64) - 1, -64):
            used = sum(ROWBYTES[fmt](k) * n for n, k in ops)
            held = sum((ROWBYTES[fmt](k) + c - 1) // c * c * n for n, k in ops)
            if used / held > best + 0.005:
                best, kc = used / held, c
        op_nch = [(ROWBYTES[fmt](k) + kc - 1) // kc for _, k in ops]
        nch = min(op_nch)
    rs = kc + 64 if kc % 128 == 0 else kc
    st_bytes = (16 * rs + 127) // 128 * 128
    auto_ring = ring == 0
    if ring == 0:
        ring = min(16, (cap - fixed) // (st_bytes + tma_meta_bytes(fmt, kc // 64)))
        if ring < 2:
            return None
    total = tma_smem_bytes(fmt, NC, K, ring, nch, kc, st_bytes, dec)
    while auto_ring and total > cap and ring > 2:
        ring -= 1
        total = tma_smem_bytes(fmt, NC, K, ring, nch, kc, st_bytes, dec)
    if total > cap:
        return None
    return (kc, nch, rs, st_bytes, ring, total) + ((op_nch,) if ops else ())


def meta_copy_u16(mod, T, e0, n, slot, lanes=32):
    """Mirror of u16_words / u16_word_copy for a 2-byte array at byte address `mod` (mod 4) with T elements: every word
    copied with cp.async lies inside the array, partial words are read half by half inside it, the copy fits its
    shared-memory slot of `slot` halves, and every element of [e0, e0 + n) lands at parity + (e - e0)."""
    b = mod + 2 * e0
    nw = ((b + 2 * n - 1) >> 2) - (b >> 2) + 1
    assert 1 <= nw and (lanes is None or nw <= lanes) and 2 * nw <= slot
    lo, hi = mod, mod + 2 * T
    got = {}
    for k in range(nw):
        w = (b & ~3) + 4 * k
        halves = [w, w + 2] if (w >= lo and w + 4 <= hi) else [h for h in (w, w + 2) if h >= lo and h + 2 <= hi]
        for h in halves:
            assert lo <= h and h + 2 <= hi
            got[2 * k + (h - w) // 2] = (h - mod) // 2                # smem half index -> element
    par = (b >> 1) & 1
    for e in range(e0, e0 + n):
        assert got.get(par + e - e0) == e, (mod, T, e0, n, e)


def replay_tma(fmt, N, K, NC, ring, U, sms=148, per_sm=1, share=1):
    """Replay of gemv_tma_kernel: per CTA the producer streams T x NCH stages through a ring of ST stages (one bulk copy
    per valid row, KC bytes except the ragged last chunk) while the consumers split each stage's 64-byte steps into NC
    equal ranges of <= U-step iterations. Checks copies in bounds of W and of the stage, every (row, chunk) copied and
    consumed exactly once, metadata indices (INT4 scales per row and group, FP8 row scales, bias) in range, every
    output stored once, and that the full/empty mbarrier protocol (metadata one stage behind) always makes progress."""
    cap = share_cap(share)
    geo = tma_prep(fmt, NC, K, ring, cap)
    assert geo is not None, (fmt, K, NC, ring, share)
    KC, NCH, RS, ST_BYTES, ST, smem = geo
    G = grid(N, sms, per_sm)
    nsts = replay_tma_op(fmt, N, K, NC, U, KC, NCH, RS, ST_BYTES, ST, smem, cap, G)
    for nst in nsts:
        replay_ring(nst, ST, NC, [i // NCH for i in range(nst)], tma_part_bufs(ST, NCH))


def replay_tma_op(fmt, N, K, NC, U, KC, NCH, RS, ST_BYTES, ST, smem, cap, G):
    """Stage-level checks of one GEMV streamed with geometry (KC, NCH, RS, ST_BYTES) by G CTAs; returns the number of
    stages of every CTA."""
    assert smem <= cap and KC % 64 == 0 and RS % 16 == 0 and ST_BYTES % 128 == 0 and 2 <= ST <= 16
    assert 16 * RS <= ST_BYTES
    CS = KC // 64
    if fmt.startswith("int4"):
        assert CS <= 32                                       # 2 x 16 metadata words per producer lane pair
    SK = MMA_STEP_K[fmt]
    rowbytes = ROWBYTES[fmt](K)
    nchunk = rowbytes // 16
    S = (nchunk + 3) // 4
    Kp = (K + SK - 1) // SK * SK
    groups = K // 128
    assert NCH * KC >= rowbytes and (NCH - 1) * KC < rowbytes
    copied = np.zeros((N, nchunk), dtype=np.int32)
    consumed = np.zeros((N, nchunk), dtype=np.int32)
    stores = np.zeros(N, dtype=np.int32)
    nsts = []
    for blk in range(G):
        rb, re = blk * N // G, (blk + 1) * N // G
        T = (re - rb + 15) >> 4
        nst = T * NCH
        nsts.append(nst)
        # --- producer: copies and metadata
        for i in range(nst):
            t, j = divmod(i, NCH)
            r0 = rb + 16 * t
            nrows = min(re - r0, 16)
            assert 1 <= nrows <= 16
            nsteps = S - j * CS if j == NCH - 1 else CS
            assert 1 <= nsteps <= CS
            nbytes = rowbytes - j * KC if j == NCH - 1 else KC
            assert 16 <= nbytes <= KC and nbytes % 16 == 0 and j * KC % 16 == 0
            assert nrows * nbytes < 2 ** 20                       # mbarrier transaction count range
            for rr in range(nrows):
                src = (r0 + rr) * rowbytes + j * KC
                assert 0 <= src and src + nbytes <= N * rowbytes and src % 16 == 0
                assert rr * RS + nbytes <= ST_BYTES
                copied[r0 + rr, j * KC // 16: j * KC // 16 + nbytes // 16] += 1
            if fmt.startswith("int4"):
                MR = tma_meta_row(CS)
                if NCH == 1:                                       # the tile's contiguous run, words over 32 lanes
                    assert S <= CS and 16 * groups + 2 <= 16 * MR
                    for mod in (0, 2):
                        meta_copy_u16(mod, N * groups, r0 * groups, nrows * groups, 16 * MR, lanes=None)
                    if groups % 8 == 0:                            # the bulk-copy form of the same run
                        assert (2 * r0 * groups) % 16 == 0 and (2 * nrows * groups) % 16 == 0
                        assert (112 + 32 * MR) % 16 == 0 and MR % 2 == 0
                else:
                    for rr in range(nrows):
                        e0 = (r0 + rr) * groups + j * CS
                        for mod in (0, 2):                         # array base address 0 or 2 modulo 4
                            meta_copy_u16(mod, N * groups, e0, nsteps, MR)
            if j == 0:
                for lane in range(min(nrows, 32)):
                    assert 0 <= r0 + lane < N                      # FP8 row scales (4-byte cp.async)
                for mod in (0, 2):
                    meta_copy_u16(mod, N, r0, nrows, 18)           # bias words
        # --- consumers: steps of each stage, loads inside the stage, x inside Kp
        for i in range(nst):
            t, j = divmod(i, NCH)
            r0 = rb + 16 * t
            nsteps = S - j * CS if j == NCH - 1 else CS
            covered = np.zeros(nsteps, dtype=np.int32)
            rend = min(r0 + 16, re)
            assert (8 + 7) * RS + 64 * (nsteps - 1) + 16 * 3 + 16 <= ST_BYTES   # rows g, g+8, last step, lane c=3
            assert ((j * CS + nsteps) * SK) <= Kp                               # x reads inside the padded x
            if fmt.startswith("int4"):
                assert j * CS + nsteps <= Kp // 128 and nsteps <= CS            # gsum and metadata indices
            for warp in range(NC):
                sa, sb = warp * nsteps // NC, (warp + 1) * nsteps // NC
                its = list(range(sa, sb, U))
                assert all(1 <= min(sb - sl, U) <= U for sl in its)
                covered[sa:sb] += 1
                q0, q1 = 4 * (j * CS + sa), min(4 * (j * CS + sb), nchunk)
                if q1 > q0:
                    consumed[r0:rend, q0:q1] += 1
            assert np.all(covered == 1)
            if j == NCH - 1:
                for g in range(16):
                    if r0 + g < re:
                        stores[r0 + g] += 1
    assert np.all(copied == 1), f"{fmt} N={N} K={K}: copies min {copied.min()} max {copied.max()}"
    assert np.all(consumed == 1), f"{fmt} N={N} K={K}: consumed min {consumed.min()} max {consumed.max()}"
    assert np.all(stores == 1)
    return nsts


def replay_ring(nst, ST, NC, tile_of, NB):
    """The full/empty mbarrier protocol of one CTA's stream of nst stages (tile_of[i]: the tile, numbered over the whole
    stream, that stage i belongs to): the producer may fill stage i once stage i - ST is released by all NC warps; a
    stage is readable once filled. A warp may run up to ST - 1 stages ahead of the slowest one, so the tiles in flight
    between them must fit the NB tile-partial buffers (one more for the epilogue's read)."""
    for i in range(nst):
        assert tile_of[i] - tile_of[max(0, i - (ST - 1))] + 2 <= NB, (i, ST, NB)
    released = [0] * nst
    issued, consumed_upto, steps = 0, 0, 0
    while consumed_upto < nst:
        steps += 1
        assert steps < 4 * nst + 16, "mbarrier protocol stalled"
        progressed = False
        if issued < nst and (issued < ST or released[issued - ST] == NC):
            issued += 1
            progressed = True
        if consumed_upto < issued:
            released[consumed_upto] = NC
            consumed_upto += 1
            progressed = True
        assert progressed, "deadlock"
    # producer/consumer mbarrier parities follow the rounds of the ring: wait k of slot s has parity k & 1
    ph, s = 0, 0
    for i in range(nst):
        if i >= ST:
            assert ph == ((i // ST) - 1) & 1
        s += 1
        if s == ST:
            s = 0
            if i >= ST:
                ph ^= 1


def replay_layer(fmt, ops, NC, U, sms=148, dec=0):
    """Replay of a layer launch (one CTA per SM): one stage geometry for every op, each op's stages checked as a GEMV of
    its own, and the ring protocol over the concatenated stream of all ops' stages (slots, parities and tile-partial
    buffers continue across op boundaries). Also the x region: every op's staged x fits the one sized for the
    largest K."""
    geo = tma_prep(fmt, NC, 0, 0, SMEM_CAP, dec, ops=ops)
    assert geo is not None, (fmt, ops)
    KC, NCH_MIN, RS, ST_BYTES, ST, smem, op_nch = geo
    G = min(sms, max(n for n, _ in ops))
    Kmax = max(k for _, k in ops)
    SK = MMA_STEP_K[fmt]
    per_cta = [[] for _ in range(G)]
    for (N, K), nch in zip(ops, op_nch):
        assert (K + SK - 1) // SK * SK <= (Kmax + SK - 1) // SK * SK
        nsts = replay_tma_op(fmt, N, K, NC, U, KC, nch, RS, ST_BYTES, ST, smem, SMEM_CAP, G)
        for blk in range(G):
            per_cta[blk].append((nsts[blk], nch))
    NB = tma_part_bufs(ST, NCH_MIN)
    for blk in range(G):
        tile_of, base = [], 0
        for nst, nch in per_cta[blk]:
            tile_of += [base + i // nch for i in range(nst)]
            base += nst // nch
        replay_ring(len(tile_of), ST, NC, tile_of, NB)
    return geo


TMA_SHAPES = dict(SHAPES)
TMA_SHAPES["bf16"] = SHAPES["bf16"] + [(37, 65536), (20, 98304), (5, 8200)]
TMA_SHAPES["fp8"] = SHAPES["fp8"] + [(37, 98304), (3, 28672)]
TMA_SHAPES["int4"] = SHAPES["int4"] + [(9, 98304), (17, 28672)]
TMA_SHAPES["int4_asym"] = TMA_SHAPES["int4"]


@pytest.mark.parametrize("fmt", list(TMA_SHAPES))
def test_tma_mapping_exactly_once(fmt):
    rnd = random.Random(2)
    combos = list(itertools.product(TMA_SHAPES[fmt], (4, 8), (0, 2, 3, 16), (2, 4), (1, 2)))
    for (N, K), NC, ring, U, share in rnd.sample(combos, 16):
        if tma_prep(fmt, NC, K, ring, share_cap(share)) is None:
            assert K > 16384 or ring == 16, (fmt, K, ring, share)   # only long rows or deep rings may not fit
            continue
        replay_tma(fmt, N, K, NC, ring, U, sms=rnd.choice((148, 7, 1)), per_sm=rnd.choice((1, 2)), share=share)


LAYERS = {
    # Llama-3.1-8B decode layer (qkv, o, gate_up, down) and Qwen2.5-7B, plus a chain with ragged and tiny N
    "llama": [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)],
    "qwen": [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944)],
    "ragged": [(1536, 1024), (1024, 1536), (14336, 1024), (100, 14336), (40, 256), (3000, 128)],
}


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4", "int4_asym"])
@pytest.mark.parametrize("name", list(LAYERS))
def test_layer_mapping(fmt, name):
    ops = LAYERS[name]
    if name == "ragged":
        replay_layer(fmt, ops, 8, 2, sms=rnd_sms(fmt))
    kc, nch, rs, st_bytes, ring, smem, op_nch = tma_prep(fmt, 8, 0, 0, SMEM_CAP, 0, ops=ops)
    # real layers: the stages are >= 97% full over the layer's weight bytes and the ring still holds >= 3 stages
    if name != "ragged":
        used = sum(ROWBYTES[fmt](k) * n for n, k in ops)
        held = sum(c * kc * n for (n, _), c in zip(ops, op_nch))
        assert used / held >= 0.97, (fmt, name, kc, used / held)
        assert ring >= 3 and smem <= SMEM_CAP


def rnd_sms(fmt):
    return {"bf16": 148, "fp8": 7, "int4": 148, "int4_asym": 3}[fmt]


def test_tma_prep_geometry():
    # real decode shapes stage with >= ~2 KB per row piece and fit in one CTA per SM
    for fmt, K in (("bf16", 4096), ("bf16", 8192), ("bf16", 14336), ("fp8", 4096), ("fp8", 8192), ("fp8", 28672),
                   ("int4", 4096), ("int4", 8192), ("int4", 14336)):
        for share in (1, 2):
            geo = tma_prep(fmt, 8, K, 0, share_cap(share))
            assert geo is not None
            kc, nch, rs, st_bytes, ring, smem = geo
            assert kc >= min(ROWBYTES[fmt](K), 1024 // share) and ring >= 2
            assert smem <= share_cap(share)
    # the largest K the C ABI accepts still stages (smaller pieces)
    for fmt in ("bf16", "fp8", "int4"):
        assert tma_prep(fmt, 8, 98304, 2) is not None
