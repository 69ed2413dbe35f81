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


def tma_meta_row(cs, chunked):
    return (cs + 21) & ~7 if chunked else (cs + 8) & ~7


def tma_meta_bytes(fmt, mr):
    i4 = 16 * mr * 2 * (2 if fmt == "int4_asym" else 1) if fmt.startswith("int4") else 0
    return (112 + i4 + 15) // 16 * 16


def tma_part_bufs(ring, nch):
    return (ring - 1 + nch - 1) // nch + 2


def tma_smem_bytes(fmt, NC, K, ring, nch, mr, st_bytes, dec=0, xm=0):
    """Mirror of tma_smem_bytes; xm > 0: the batched kernel with xm x rows."""
    SK = MMA_STEP_K[fmt]
    kp = (K + SK - 1) // SK * SK
    nb = tma_part_bufs(max(ring, 2), nch)
    i4 = fmt.startswith("int4")
    rows = xm if xm else 1
    if (i4 and dec == 2) or (fmt == "fp8" and dec == 3):      # four byte planes (x_plane_stride)
        xrow = 4 * ((((kp + 127) & ~127) + 64) if fmt == "fp8" else kp + 16)
    else:
        xrow = kp * 2 + 64
    return (640 + ring * (st_bytes + tma_meta_bytes(fmt, mr)) + rows * xrow
            + (rows * (kp // 128) * (8 if dec == 2 else 2) * 4 if i4 else 0) + nb * NC * 16 * (8 if xm else 1) * 4
            + (256 if xm else 160))


BLOCK_ROW = 3072                                               # kTmaBlockRow


def tma_blocked(nch, kc, rs):
    return nch == 1 and rs == kc and kc < BLOCK_ROW


def tma_row_off(r, rs, blocked):
    """Byte offset of tile row r in a stage: padded rows r x rs, or two 8-row blocks 8 rs + 64 apart."""
    return (r >> 3) * (8 * rs + 64) + (r & 7) * rs if blocked else r * rs


def tma_tile_row(m, blocked):
    """Tile row that MMA row m (0..15) reads."""
    return (((m & 1) << 3) | ((m >> 1) & 3) | (4 if m & 8 else 0)) if blocked else m


def tma_stage_bytes(rs, blocked):
    return (16 * rs + (64 if blocked else 0) + 127) // 128 * 128


def tma_op_geometry(nchunk, kcs, tensor=False):
    """Mirror of tma_op_geometry: (nch, kc, rs) of a row of nchunk 16-byte chunks in a slot of kcs bytes per row;
    tensor: the layout of the tiled tensor copy (never blocked, chunks of an odd piece count where one fits)."""
    rb = nchunk * 16
    c, n = rb, 1
    if rb > kcs:
        n = (rb + kcs - 1) // kcs
        c = ((rb + n - 1) // n + 63) // 64 * 64
        if tensor:
            for m in range(n, n + 4):
                cm = ((rb + m - 1) // m + 63) // 64 * 64
                if (cm // 64) % 2 == 0:
                    cm += 64
                if cm <= kcs and (rb + cm - 1) // cm == m:
                    n, c = m, cm
                    break
    if not tensor and n == 1 and rb % 64 == 0 and rb < BLOCK_ROW:
        return n, c, rb
    c64 = (c + 63) // 64 * 64
    return n, c, c64 + 64 if c64 % 128 == 0 else c64


def tma_apply_slot(fmt, K, rowbytes, kcs, ops, tensor=False):
    """Mirror of tma_apply_slot: (kc, nch, rs, st_bytes, mr, geos) for a slot of kcs bytes per row."""
    if not ops:
        n = (rowbytes + kcs - 1) // kcs
        kb = kcs if tensor else ((rowbytes + n - 1) // n + 63) // 64 * 64
        nch, kc, rs = tma_op_geometry(rowbytes // 16, kb, tensor)
        blocked = not tensor and tma_blocked(nch, kc, rs)
        return kc, nch, rs, tma_stage_bytes(rs, blocked), tma_meta_row(kb // 64, nch > 1), None
    geos = [tma_op_geometry(ROWBYTES[fmt](k) // 16, kcs) for _, k in ops]
    st = max(tma_stage_bytes(g[2], tma_blocked(*g)) for g in geos)
    mr = tma_meta_row(kcs // 64, any(g[0] > 1 for g in geos))
    return kcs, min(g[0] for g in geos), max(g[2] for g in geos), st, mr, geos


def tma_tensor(fmt, K, ops=None, xm=0, tensor_on=False):
    """Whether a launch uses the tiled-tensor stage layout (on request: a single GEMV of whole 64-byte row pieces)."""
    return bool(tensor_on) and not ops and not xm and ROWBYTES[fmt](K) % 64 == 0


def tma_prep(fmt, NC, K, ring=0, cap=SMEM_CAP, dec=0, ops=None, xm=0, tensor_on=False):
    """Mirror of tma_prep<F, NC>: (kc, nch, rs, st_bytes, ring, smem) or None when the shape cannot be staged.
    Layer mode (`ops`: a list of (N, K)): K is the largest K, one slot size (kc = the slot's bytes per row) for all
    ops, nch the smallest op NCH, rs the largest op row stride, and a seventh element, the list of per-op
    (nch, kc, rs)."""
    if ops:
        K = max(k for _, k in ops)
    rowbytes = max(ROWBYTES[fmt](k) for _, k in ops) if ops else ROWBYTES[fmt](K)
    if ring == 1 or ring > 16:
        return None
    tensor = tma_tensor(fmt, K, ops, xm, tensor_on)
    top = min((rowbytes + 63) // 64 * 64, 4096)
    kmin = min(top, 2048) if xm else 64
    geo = None
    for rmin in ([ring] if ring >= 2 else ([3] if xm else [3, 2])):
        for kcs in range(top, kmin - 1, -64):
            kc, nch, rs, st, mr, geos = tma_apply_slot(fmt, K, rowbytes, kcs, ops, tensor)
            if tma_smem_bytes(fmt, NC, K, rmin, nch, mr, st, dec, xm) <= cap:
                geo = (kc, nch, rs, st, mr, geos)
                break
        if geo:
            break
    if geo is None:
        return None
    if fmt == "fp8" and dec == 3 and not xm and ring == 0 and not ops and geo[1] > 1:
        # chunked e4m3 rows: 4 stages of pieces >= 2.5 KB when they fit (kTmaMinPiece4)
        for kcs in range(top, 2560 - 1, -64):
            cand = tma_apply_slot(fmt, K, rowbytes, kcs, ops, tensor)
            if tma_smem_bytes(fmt, NC, K, 4, cand[1], cand[4], cand[3], dec, xm) <= cap:
                geo = cand
                break
    kc, nch, rs, st, mr, geos = geo
    if ring == 0:
        ring = 2
        while ring < 16 and tma_smem_bytes(fmt, NC, K, ring + 1, nch, mr, st, dec, xm) <= cap:
            ring += 1
    total = tma_smem_bytes(fmt, NC, K, ring, nch, mr, st, dec, xm)
    if total > cap:
        return None
    return (kc, nch, rs, st, ring, total) + ((geos,) if ops else ())


def check_banks(rs, blocked):
    """Every shared-memory access phase of the consumers' 16-byte fragment loads (8 lanes: MMA rows 2m', 2m'+1 of the
    first or second load, bytes 16c of one 64-byte step) touches each of the 32 banks once."""
    for second in (0, 8):
        for mp in range(4):
            for step_off in (0, 64, 128, 192, 64 * 37):
                banks = []
                for m in (2 * mp + second, 2 * mp + 1 + second):
                    r = tma_tile_row(m, blocked)
                    for c in range(4):
                        a = tma_row_off(r, rs, blocked) + step_off + 16 * c
                        banks += [(a // 4 + w) % 32 for w in range(4)]
                assert sorted(banks) == list(range(32)), (rs, second, mp, step_off)


def meta_copy_u16(mod, T, e0, n, slot, lanes=32):
    """Mirror of u16_blocks16 / u16_block_copy for a 2-byte array at byte address `mod` (mod 16) with T elements: every
    16-byte block copied holds at least one byte of the array (so it lies in a page the array occupies), the copy fits
    its shared-memory slot of `slot` halves, and every element of [e0, e0 + n) lands at off16 + (e - e0)."""
    b = mod + 2 * e0
    nb = ((b + 2 * n - 1) >> 4) - (b >> 4) + 1
    assert 1 <= nb and (lanes is None or nb <= lanes) and 8 * nb <= slot, (mod, e0, n, nb, slot)
    lo, hi = mod, mod + 2 * T
    got = {}
    for k in range(nb):
        blk = (b & ~15) + 16 * k
        assert blk < hi and blk + 16 > lo                          # the block overlaps the array
        for h in range(blk, blk + 16, 2):
            if lo <= h < hi:
                got[8 * k + (h - blk) // 2] = (h - mod) // 2           # smem half index -> element
    off = (b >> 1) & 7
    for e in range(e0, e0 + n):
        assert got.get(off + e - e0) == e, (mod, T, e0, n, e)


def replay_tma(fmt, N, K, NC, ring, U, sms=148, per_sm=1, share=1, dec=0, tensor_on=False):
    """Replay of gemv_tma_kernel: per CTA the producer streams T x NCH stages through a ring of ST stages (two block
    copies per whole-row stage, else one copy per valid row, KC bytes except the ragged last chunk) while the
    consumers split each stage's 64-byte steps into NC equal ranges of <= U-step iterations. Checks copies in bounds
    of W and of the stage, every (row, chunk) copied and consumed exactly once, metadata indices (INT4 scales per row
    and group, bias) in range, every output stored once, conflict-free fragment loads, and that the full/empty
    mbarrier protocol always makes progress."""
    cap = share_cap(share)
    geo = tma_prep(fmt, NC, K, ring, cap, dec, tensor_on=tensor_on)
    assert geo is not None, (fmt, K, NC, ring, share)
    KC, NCH, RS, ST_BYTES, ST, smem = geo
    G = grid(N, sms, per_sm)
    tensor = tma_tensor(fmt, K, tensor_on=tensor_on)
    nsts = replay_tma_op(fmt, N, K, NC, U, KC, NCH, RS, ST_BYTES, ST, smem, cap, G, slot_steps(fmt, K, KC, tensor),
                         tensor=tensor)
    for nst in nsts:
        replay_ring(nst, ST, NC, [i // NCH for i in range(nst)], tma_part_bufs(ST, NCH))


def slot_steps(fmt, K, KC, tensor):
    """64-byte steps of the stage slot the metadata ring is sized for: the chunk, or with the tensor layout the slot
    the geometry search stopped at (at least the chunk; the mirror takes the chunk, the smallest slot it allows)."""
    return (KC + 63) // 64


def replay_tma_op(fmt, N, K, NC, U, KC, NCH, RS, ST_BYTES, ST, smem, cap, G, CS_SLOT, CHUNKED=False, tensor=False):
    """Stage-level checks of one GEMV streamed with geometry (KC, NCH, RS) in stage slots of ST_BYTES (metadata slots
    for CS_SLOT steps per row) by G CTAs; returns the number of stages of every CTA. tensor: the stage layout of the
    tiled tensor copy (full tiles: one 16-row box of RS bytes per row, RS / 64 pieces <= 256, 128-byte aligned)."""
    assert smem <= cap and RS % 64 == 0 and ST_BYTES % 128 == 0 and 2 <= ST <= 16
    blocked = not tensor and tma_blocked(NCH, KC, RS)
    if tensor:
        assert RS // 64 <= 256 and 16 * RS <= ST_BYTES and (RS // 64) % 2 == 1 and KC % 64 == 0
    assert tma_row_off(15, RS, blocked) + RS <= ST_BYTES
    check_banks(RS, blocked)
    CS = KC // 64
    SK = MMA_STEP_K[fmt]
    rowbytes = ROWBYTES[fmt](K)
    nchunk = rowbytes // 16
    S = (nchunk + 3) // 4
    Kp = (K + SK - 1) // SK * SK
    groups = K // 128
    dense = blocked
    assert NCH * KC >= rowbytes and (NCH - 1) * KC < rowbytes and KC <= RS
    if NCH > 1:
        assert KC % 64 == 0 and CS <= CS_SLOT
    else:
        assert KC == rowbytes and (rowbytes + 63) // 64 <= max(CS_SLOT, 1) + 1
    MR = tma_meta_row(CS_SLOT, NCH > 1 or CHUNKED)
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
            assert 1 <= nsteps and (NCH == 1 or nsteps <= CS)
            nbytes = rowbytes - j * KC if j == NCH - 1 else KC
            assert 16 <= nbytes <= KC and nbytes % 16 == 0 and j * KC % 16 == 0
            assert nrows * nbytes < 2 ** 20                       # mbarrier transaction count range
            if dense:
                for b in range(2):
                    nb = min(8, nrows - 8 * b)
                    if nb <= 0:
                        continue
                    src = (r0 + 8 * b) * rowbytes
                    dst = b * (8 * RS + 64)
                    assert src % 16 == 0 and dst % 16 == 0 and (nb * rowbytes) % 16 == 0
                    assert src + nb * rowbytes <= N * rowbytes and dst + nb * rowbytes <= ST_BYTES
                    for rr in range(8 * b, 8 * b + nb):
                        assert tma_row_off(rr, RS, True) == dst + (rr - 8 * b) * rowbytes
                        copied[r0 + rr, :] += 1
            else:
                for rr in range(nrows):
                    src = (r0 + rr) * rowbytes + j * KC
                    assert 0 <= src and src + nbytes <= N * rowbytes and src % 16 == 0
                    assert rr * RS % 16 == 0 and rr * RS + nbytes <= ST_BYTES
                    copied[r0 + rr, j * KC // 16: j * KC // 16 + nbytes // 16] += 1
            if fmt.startswith("int4"):
                if NCH == 1:                                       # the tile's contiguous run, words over 32 lanes
                    assert S <= CS_SLOT + 1 and 16 * groups + 2 <= 16 * MR
                    for mod in range(0, 16, 2):
                        meta_copy_u16(mod, N * groups, r0 * groups, nrows * groups, 16 * MR, lanes=None)
                    if groups % 8 == 0:                            # the bulk-copy form of the same run
                        assert (2 * r0 * groups) % 16 == 0 and (2 * nrows * groups) % 16 == 0
                        assert (112 + 32 * MR) % 16 == 0 and MR % 2 == 0
                else:
                    for rr in range(nrows):
                        e0 = (r0 + rr) * groups + j * CS
                        for mod in range(0, 16, 2):                # array base address modulo 16
                            meta_copy_u16(mod, N * groups, e0, nsteps, MR, lanes=None)
                        assert 16 * ((nsteps + 21) >> 3) >= 16 * 1 and (nsteps + 21) >> 3 >= (nsteps + 14) // 8
        # --- consumers: steps of each stage, loads inside the stage, x inside Kp
        for i in range(nst):
            t, j = divmod(i, NCH)
            r0 = rb + 16 * t
            nsteps = S - j * CS if j == NCH - 1 else CS
            covered = np.zeros(nsteps, dtype=np.int32)
            rend = min(r0 + 16, re)
            for m in range(16):                                    # every MMA row's last 16-byte load in its slot
                r = tma_tile_row(m, blocked)
                assert 64 * (nsteps - 1) + 16 * 3 + 16 <= RS
            assert sorted(tma_tile_row(m, blocked) for m in range(16)) == list(range(16))
            assert ((j * CS + nsteps) * SK) <= Kp                               # x reads inside the padded x
            if fmt.startswith("int4"):
                assert j * CS + nsteps <= Kp // 128                            # gsum and metadata indices
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
    KCS, NCH_MIN, RS_MAX, ST_BYTES, ST, smem, geos = geo
    G = min(sms, max(n for n, _ in ops))
    Kmax = max(k for _, k in ops)
    SK = MMA_STEP_K[fmt]
    per_cta = [[] for _ in range(G)]
    for (N, K), (nch, kc, rs) in zip(ops, geos):
        assert (K + SK - 1) // SK * SK <= (Kmax + SK - 1) // SK * SK and kc <= KCS and rs <= RS_MAX
        nsts = replay_tma_op(fmt, N, K, NC, U, kc, nch, rs, ST_BYTES, ST, smem, SMEM_CAP, G, KCS // 64,
                             any(g[0] > 1 for g in geos))
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


def test_fp8_chunked_rows_take_four_stages():
    """The default FP8 decode (e4m3 tensor cores) stages chunked rows in a 4-stage ring (slots >= 2.5 KB, pieces
    >= 2.25 KB next to the four x planes), whole rows keep one piece per row; the long-K projections replay cleanly
    in that geometry; rows too long for four x planes next to two stages leave the kernel (-2: the next decode)."""
    assert tma_prep("fp8", 8, 4096, 0, SMEM_CAP, 3)[:5] == tma_prep("fp8", 8, 4096, 0, SMEM_CAP, 0)[:5]
    for N, K in ((4096, 14336), (3584, 18944), (4096, 11008), (37, 98304), (300, 8208)):
        geo = tma_prep("fp8", 8, K, 0, SMEM_CAP, 3)
        if K > 65536:                                  # four x planes leave no room for stages: the C ABI falls back
            assert geo is None and tma_prep("fp8", 8, K, 0, SMEM_CAP, 0) is not None, K
            continue
        kc, nch, rs, st, ring, smem = geo
        assert nch > 1 and kc >= 2304 and ring >= 4 and smem <= SMEM_CAP, (K, kc, nch, ring)
        replay_tma("fp8", N, K, 8, 0, 2, sms=148 if N > 1000 else 7, dec=3)


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
    kcs, nch, rs, st_bytes, ring, smem, geos = tma_prep(fmt, 8, 0, 0, SMEM_CAP, 0, ops=ops)
    # real layers: every op's stage pieces are >= 1.5 KB per row (few, large copies) and the ring holds >= 3 stages
    if name != "ragged":
        assert all(kc >= 1536 for _, kc, _ in geos), (fmt, name, geos)
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


def batched_groups(fmt, M, K):
    """Mirror of paia_gemv_batched's grouping: launches of 2 to 8 x rows, each as many as fit with >= 3 stages of >= 2 KB
    pieces; 1 = a single-row call."""
    out, m0 = [], 0
    while m0 < M:
        mg = min(8, M - m0)
        while mg >= 2 and tma_prep(fmt, 8, K, 0, SMEM_CAP, 0, xm=mg) is None:
            mg -= 1
        out.append(max(mg, 1))
        m0 += max(mg, 1)
    return out


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4", "int4_asym"])
def test_batched_geometry(fmt):
    """Batched x: every real shape stages at least one x row next to a 2+ stage ring, short rows take 8 x rows per
    launch, and the replay of the weight stream (unchanged by the x rows) holds."""
    for K in (3584, 4096, 14336, 18944):
        geo = tma_prep(fmt, 8, K, 0, SMEM_CAP, 0, xm=2)
        assert geo is not None and geo[4] >= 3, (fmt, K)
    for K in (3584, 4096):
        assert batched_groups(fmt, 16, K) == [8, 8], (fmt, K, batched_groups(fmt, 16, K))
    for K in (14336, 18944):
        g = batched_groups(fmt, 16, K)
        assert sum(g) == 16 and max(g) >= 2, g
    kc, nch, rs, st, ring, smem = tma_prep(fmt, 8, 4096, 0, SMEM_CAP, 0, xm=8)
    replay_tma_op(fmt, 300, 4096, 8, 2, kc, nch, rs, st, ring, smem, SMEM_CAP, 7, (kc + 63) // 64)


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4", "int4_asym"])
def test_tensor_copy_layout_replays(fmt):
    """The stage layout of the optional tiled tensor copies (never blocked, odd piece counts): whole and chunked rows
    replay cleanly, fragment loads stay conflict-free, and a full tile's box (16 rows x RS) fits its stage."""
    dec = 2 if fmt.startswith("int4") else (3 if fmt == "fp8" else 0)
    for N, K in ((4096, 4096), (300, 14336), (1000, 3584), (37, 18944)):
        replay_tma(fmt, N, K, 8, 0, 2, sms=148 if N > 1000 else 7, dec=dec, tensor_on=True)
