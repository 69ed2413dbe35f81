// TMA-fed tensor-core GEMV for B200 (sm_100a): the streaming design of the decode GEMV family.
//
// Measured on B200: loading MMA fragments straight from HBM (each warp instruction touching 16 rows x 64 B) stops at
// ~4.4-5.4 TB/s, while bulk copies stream at up to ~6.6 TB/s. A CTA's copy throughput is bounded by the number of
// bulk copies (about 15 million per second per SM), not only by the bytes in flight: at ~190 KB in flight per SM,
// 4 KB copies reach HBM speed and 0.7 KB copies a quarter of it. So a producer warp moves the weights in as few,
// large cp.async.bulk copies as possible (1-D TMA, completion counted on an mbarrier) into a ring of shared-memory
// stages, and consumer warps read the MMA fragments from shared memory.
//
//   CTA       one persistent CTA per SM; rows [c N/G, (c+1) N/G), cut into 16-row tiles; a tile is streamed as NCH
//             stages of 16 rows x KC bytes (a whole row when it fits the slot, else equal chunks, a multiple of 64).
//   producer  warp NC. Lane 0 waits for the slot; then a whole-row stage of short rows (< 3 KB) is two bulk copies
//             (tile rows 0-7 and 8-15, contiguous in global memory) and any other stage one copy per row (rows
//             beyond the CTA's range are not copied; their MMA rows compute garbage that is never stored). The two
//             8-row blocks sit 8 RS + 64 bytes apart and MMA rows are mapped to tile rows so that the two rows a
//             fragment load phase touches lie in different blocks (different bank halves). The producer starts at
//             launch, before the programmatic-dependency wait: weights never depend on the preceding kernel. All 32
//             lanes then copy the stage's metadata (INT4 scales and zeros of its rows and groups) with one bulk copy
//             per array when the run is 16-byte aligned, else as the 16-byte blocks that hold it (cp.async), whose
//             completion is also counted on the stage's `full` mbarrier, so no register ever waits on a load: under
//             a saturated memory system a plain load takes as long as the whole ring's copies.
//   consumers warps 0..NC-1 wait for the dependency, stage x (as gemv_mma.cuh), then for every stage take an equal
//             share of its 64-byte steps, load A fragments from the stage (MMA rows g and g+8, bytes 16c of each
//             step), B fragments from x, and run the dequantisation and mma.sync of the format. The step loop is
//             branch-free (U steps per iteration; the remainder and the ragged last step of a row run one at a time)
//             and keeps two accumulator chains per step. At the last stage of a tile each warp leaves its 16 partial
//             sums in a shared-memory buffer and arrives on the buffer's `tile_done` mbarrier; no consumer waits
//             for another except through the ring.
//   epilogue  warp NC+1 adds each tile's NC partials in warp order (deterministic), applies the row scale, the x
//             scale and the bias (loaded from global memory while the tile is computed), writes the 16 outputs and
//             frees the buffer (`part_free`), so the tile-end work never stalls the consumers.
//   layer     one launch may stream a sequence of GEMVs (layer mode: Params::nops); the ring, the partial buffers
//             and their phases run on across op boundaries, and the consumers of op j wait for every CTA's outputs
//             of op j - 1 (a per-op completion counter) before they stage x of op j.
//   waits     every wait gives up after ~2 s (%globaltimer), records an error code that paia_gemv_device_error()
//             reports, and carries on without waiting, so a fault can never hang the GPU; once one wait has given
//             up, every wait that has run for 1 ms gives up at once. Only the byte-counted `full` barriers can be
//             broken by a warp out of step (one more arrival on a phase whose bytes are in flight); a consumer warp
//             releases a slot only after it saw the slot's `full` phase complete, so the producer re-arms only
//             phases that completed, and stops arriving at its first failed wait (keeping the CTA alive 200 us for
//             its copies in flight). The other barriers count arrivals only, which a warp out of step cannot
//             break; its results are garbage and the error code says so.
//   rope      an instance with ROPE = true rotates q / k row pairs in the epilogue (paia_gemv_rope); the other
//             instances carry no rotary code.
//   tp        row-sharded tensor parallelism: the epilogue stores every output into every rank's y over NVLink; the
//             ranks count calls started and CTAs finished in each other's counter blocks, and CTA 0 waits until every
//             rank's CTAs are done, so a rank's y is complete when its grid ends (tp_enter / tp_leave).
#pragma once
#include "gemv_mma.cuh"

namespace pb2 {

static __device__ int g_tma_error;     // first error code of a bounded wait that gave up (0 = none)

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* m, int count) {
    asm volatile("mbarrier.init.shared.b64 [%0], %1;" :: "r"(smem_addr(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* m) {
    asm volatile("mbarrier.arrive.shared.b64 _, [%0];" :: "r"(smem_addr(m)) : "memory");
}
// Relaxed: orders nothing before it (used to say "my loads are issued" without waiting for them to complete).
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* m) {
    asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" :: "r"(smem_addr(m)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* m, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" :: "r"(smem_addr(m)), "r"(bytes) : "memory");
}
// try_wait may suspend the thread for a system-dependent time before it reports an incomplete phase.
__device__ __forceinline__ bool mbar_test(uint64_t* m, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_addr(m)), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Whether a bounded wait has already given up (this launch or an earlier one whose error the host has not cleared).
__device__ __forceinline__ bool tma_aborted() { return *reinterpret_cast<volatile int*>(&g_tma_error) != 0; }
// A wait that has run for 1 ms checks tma_aborted(): once one wait of any CTA gave up, the launch's pipeline is out
// of step, so every further wait gives up at once instead of spinning its own full limit.
constexpr uint64_t kAbortCheckNs = 1000000ull;

// Wait for phase `parity` of m for at most ~2 s; on timeout record `code` and return false (the caller carries on).
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity, int code) {
    if (mbar_test(m, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_test(m, parity)) {
        const uint64_t dt = global_ns() - t0;
        if (dt > kAbortCheckNs && tma_aborted()) return false;
        if (dt > 2000000000ull) {
            atomicCAS(&g_tma_error, 0, code);
            return false;
        }
    }
    return true;
}
// Weights are read exactly once: mark their L2 lines evict-first so activations and outputs stay resident.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_copy_g2s_ef(void* dst, const void* src, uint32_t bytes, uint64_t* m, uint64_t pol) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(m)), "l"(pol) : "memory");
}
// A box of the 3-D weight map (64 bytes x pieces x 16 rows) at piece `piece`, row `row` (x = 0: 16-byte aligned).
__device__ __forceinline__ void tensor_copy_g2s_ef(void* dst, const CUtensorMap* map, int piece, int row, uint64_t* m,
                                                   uint64_t pol) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%2, %3, %4}], [%5], %6;"
                 :: "r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(piece), "r"(row),
                    "r"(smem_addr(m)), "l"(pol) : "memory");
}
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* m) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(m)) : "memory");
}
__device__ __forceinline__ void consumer_barrier(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(smem_addr(dst)), "l"(src) : "memory");
}
// One arrival on m once all of this thread's earlier cp.async copies have landed (counted in m's arrival count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* m) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared.b64 [%0];" :: "r"(smem_addr(m)) : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_addr(dst)), "l"(src) : "memory");
}
// Block k of the copy of elements [e0, e0 + n) of a 2-byte array a (any 2-byte alignment) into dst (16-byte aligned):
// the 16-byte aligned blocks that hold the range land in dst[8k .. 8k + 7], so element e sits at
// dst[u16_off16(a + e0) + e - e0]. The first and last block may reach a few bytes past the array's ends; an aligned
// 16-byte block that holds a byte of the array lies in the same memory page, so those bytes are readable (and unused).
__device__ __forceinline__ int u16_off16(const void* p) { return (int)(((uintptr_t)p >> 1) & 7u); }
__device__ __forceinline__ int u16_blocks16(const uint16_t* a, long long e0, int n) {
    const uintptr_t b = (uintptr_t)(a + e0);
    return (int)(((b + 2 * (uintptr_t)n - 1) >> 4) - (b >> 4) + 1);
}
__device__ __forceinline__ void u16_block_copy(uint16_t* dst, const uint16_t* a, long long e0, int k) {
    cp_async16(dst + 8 * k, (const void*)((((uintptr_t)(a + e0)) & ~(uintptr_t)15) + 16 * (uintptr_t)k));
}

constexpr int kTmaMaxRing = 16;        // ring stages at most
constexpr int kTmaMaxParts = kTmaMaxRing + 1;   // tile-partial buffers at most
// mbarriers: full[16], empty[16], tile_done[17], part_free[17], x_ready (67 x 8 bytes), the producer's stop flag
// (4 bytes), padded to 640
constexpr int kTmaBarBytes = 640;
static_assert((2 * kTmaMaxRing + 2 * kTmaMaxParts + 1) * 8 + 4 <= kTmaBarBytes, "barrier region");
constexpr int kTmaTailBytes = 160;     // x scale of two ops (2 x 4 floats) + x staging scratch (32 floats)

// Metadata slot of a stage (bytes): INT4 scales and (INT4A) zeros at 112, 16 rows x tma_meta_row(CS) halves each
// (CS: 64-byte steps per row the slot holds; a row's run is copied as the 16-byte blocks that hold it, which span
// at most CS + 14 halves, and a whole-row tile's run of 16 x CS halves as blocks spanning at most 16 CS + 14).
// Halves per metadata row, a multiple of 8 (16-byte rows): >= CS + 14 when some row is chunked (a chunk's run copied as
// 16-byte blocks), else >= CS + 1 (whole-row tiles: 16 G halves plus at most 14 of block slack in 16 rows).
__host__ __device__ constexpr int tma_meta_row(int cs, bool chunked) { return chunked ? (cs + 21) & ~7 : (cs + 8) & ~7; }
template <int F>
__host__ __device__ constexpr int tma_meta_bytes(int mr) {
    return 112 + ((F == kINT4 || F == kINT4A) ? 16 * mr * 2 * (F == kINT4A ? 2 : 1) : 0);
}
// INT4 per-group sums in shared memory: 8 words per group for the integer path (digit sums and sum x), else 2.
__host__ __device__ constexpr int tma_gsum_words(int dec) { return dec == 2 ? 8 : 2; }
// Tile-partial buffers: consumers run at most ring - 1 stages ahead of the slowest, i.e. ceil((ring - 1) / NCH) + 1
// tiles; one more lets the epilogue warp lag a tile before a consumer waits for a free buffer.
__host__ __device__ constexpr int tma_part_bufs(int ring, int nch) { return (ring - 1 + nch - 1) / nch + 2; }

// Staged x length: K rounded up to whole 64-byte weight steps (32 BF16, 64 FP8, 128 INT4 weights), so that every
// x read of a row's ragged last step lands on staged zeros.
template <int F>
__host__ __device__ constexpr int tma_kx(int K) {
    return F == kBF16 ? (K + 31) / 32 * 32 : (F == kFP8 ? (K + 63) / 64 * 64 : (K + 127) / 128 * 128);
}

// Shared-memory layout (bytes): [0,640) mbarriers; ring x st_bytes; metadata ring x tma_meta_bytes (16-byte
// multiples); x: Kx x 2 + 64, or four byte planes x_plane_stride apart (FP8 e4m3 terms, INT4 integer digits);
// INT4 group sums (tma_gsum_words per group); tile partials NB x NC x 16 floats; per consumer warp its x scale
// (4 floats) and a staging scratch word (kTmaTailBytes).
// Batched kernels (BAT): x rows xm, each with its own x region, group sums and scale; partial buffers of 16 rows x 8
// columns; tail = 8 rows' x scales (32 floats) + staging scratch (32 floats).
constexpr int kTmaTailBytesBat = 256;
template <int F, int DEC>
__host__ __device__ constexpr int tma_xrow_bytes(int K) {   // one staged x row (16-byte multiple)
    return ((F == kFP8 && DEC == 3) || ((F == kINT4 || F == kINT4A) && DEC == 2))
               ? 4 * x_plane_stride<F, DEC>(tma_kx<F>(K))          // four byte planes
               : tma_kx<F>(K) * 2 + 64;
}
template <int F, int NC, int DEC, bool BAT = false>
__host__ __device__ inline size_t tma_smem_bytes(int K, int ring, int nch, int mr, int st_bytes, int xm = 1) {
    const int kp = tma_kx<F>(K);
    const size_t mb = (size_t)(tma_meta_bytes<F>(mr) + 15) / 16 * 16;
    const int nb = tma_part_bufs(ring < 2 ? 2 : ring, nch);
    const int rows = BAT ? xm : 1;
    return kTmaBarBytes + (size_t)ring * st_bytes + (size_t)ring * mb + (size_t)rows * tma_xrow_bytes<F, DEC>(K) +
           ((F == kINT4 || F == kINT4A) ? (size_t)rows * (kp / 128) * tma_gsum_words(DEC) * 4 : 0) +
           (size_t)nb * NC * 16 * (BAT ? 8 : 1) * 4 + (BAT ? kTmaTailBytesBat : kTmaTailBytes);
}

// Stage layouts (bytes from the stage base). Chunked and long rows: row r at r x RS, RS = KC (+ 64 when KC is a
// multiple of 128), so the two rows of a fragment load phase (MMA rows g, g + 1) sit in different bank halves; MMA
// row m reads tile row m; every row is one bulk copy of its chunk. Short whole rows (a multiple of 64 bytes, below
// kTmaBlockRow; RS = row bytes): rows 0-7 and rows 8-15 of a tile are two blocks 8 RS + 64 bytes apart, each one bulk
// copy (contiguous rows in global memory and in the block), and MMA row m reads tile row tma_tile_row(m), so that the
// two rows of an access phase lie in different blocks (64 bytes apart modulo 128).
// Rows at least kTmaBlockRow long stream at full speed one copy per row; shorter rows go 8 per copy (measured on
// B200: 2 KB copies cap a CTA near 30 GB/s, 4 KB copies do not limit it).
constexpr int kTmaBlockRow = 3072;
__host__ __device__ constexpr bool tma_blocked(int nch, int kc, int rs) {
    return nch == 1 && rs == kc && kc < kTmaBlockRow;
}
__host__ __device__ constexpr int tma_row_off(int r, int rs, bool blocked) {
    return blocked ? (r >> 3) * (8 * rs + 64) + (r & 7) * rs : r * rs;
}
__host__ __device__ constexpr int tma_tile_row(int m, bool blocked) {
    return blocked ? (((m & 1) << 3) | ((m >> 1) & 3) | (m & 8 ? 4 : 0)) : m;
}
__host__ __device__ constexpr int tma_stage_bytes(int rs, bool blocked) {
    return (16 * rs + (blocked ? 64 : 0) + 127) / 128 * 128;
}

// Host: the stage geometry of a row of `nchunk` 16-byte chunks in a slot of `kcs` bytes per row (a multiple of 64):
// the whole row when it fits (nch 1, kc = row bytes), else nch equal chunks of kc bytes (a multiple of 64), and the
// row stride of the layout above.
// tensor: the layout the tiled tensor copy lands (never blocked); chunks of an odd number of 64-byte pieces when one fits
// the slot, so that the row stride needs no padding piece (which the copy would read from the next chunk).
inline void tma_op_geometry(int nchunk, int kcs, int* nch, int* kc, int* rs, bool tensor = false) {
    const long rb = (long)nchunk * 16;
    long c = rb;
    int n = 1;
    if (rb > kcs) {
        n = (int)((rb + kcs - 1) / kcs);
        c = ((rb + n - 1) / n + 63) / 64 * 64;
        if (tensor) {
            for (int m = n; m <= n + 3; ++m) {                // the fewest chunks of an odd piece count
                long cm = ((rb + m - 1) / m + 63) / 64 * 64;
                if ((cm / 64) % 2 == 0) cm += 64;
                if (cm <= kcs && (rb + cm - 1) / cm == m) {
                    n = m;
                    c = cm;
                    break;
                }
            }
        }
    }
    *nch = n;
    *kc = (int)c;
    if (!tensor && n == 1 && rb % 64 == 0 && rb < kTmaBlockRow) {
        *rs = (int)rb;                                         // blocked layout
    } else {
        const long c64 = (c + 63) / 64 * 64;
        *rs = (int)(c64 % 128 == 0 ? c64 + 64 : c64);
    }
}

// Host: the stage geometry of every op of p (the single GEMV, or the layer list `ops`) for a slot of kcs bytes per row
// (single GEMV: the row split into the fewest equal chunks that fit); sets p.cs_slot, p.mr, p.st_bytes and p.nch (the
// smallest op NCH).
template <int F>
inline void tma_apply_slot(Params& p, GemvOp* ops, long kcs) {
    if (p.nops == 0) {
        const long rb = (long)p.nchunk * 16;
        const long n = (rb + kcs - 1) / kcs;
        if (!p.tlayout) kcs = ((rb + n - 1) / n + 63) / 64 * 64;
        tma_op_geometry(p.nchunk, (int)kcs, &p.nch, &p.kc, &p.rs, p.tlayout != 0);
        p.st_bytes = tma_stage_bytes(p.rs, !p.tlayout && tma_blocked(p.nch, p.kc, p.rs));
        p.mr = tma_meta_row((int)(kcs / 64), p.nch > 1);
    } else {
        int mn = 1 << 30, rs_max = 0, sb_max = 0;
        bool chunked = false;
        for (int j = 0; j < p.nops; ++j) {
            GemvOp& o = ops[j];
            tma_op_geometry(o.nchunk, (int)kcs, &o.nch, &o.kc, &o.rs);
            mn = o.nch < mn ? o.nch : mn;
            rs_max = o.rs > rs_max ? o.rs : rs_max;
            const int sb = tma_stage_bytes(o.rs, tma_blocked(o.nch, o.kc, o.rs));
            sb_max = sb > sb_max ? sb : sb_max;
            chunked = chunked || o.nch > 1;
        }
        p.nch = mn;
        p.kc = (int)kcs;
        p.rs = rs_max;
        p.st_bytes = sb_max;
        p.mr = tma_meta_row((int)(kcs / 64), chunked);
    }
    p.cs_slot = (int)(kcs / 64);
}

// Host: choose the stage geometry within `cap` bytes of shared memory and return the dynamic shared memory size (0 when
// the shape cannot be staged). The slot is the largest (a multiple of 64 bytes per row, at most 4096 so that a stage
// stays <= 64 KB) for which the exact layout fits p.ring stages, or, with p.ring 0 (auto), 3 stages (2 if no slot
// fits 3); the ring then holds as many stages as fit (2..16). Layer mode (p.nops > 0): one slot for every op (next
// to x of the largest K), each op staged in its own geometry within it; p.K and p.nchunk become the largest K and row.
constexpr long kTmaMinPiece4 = 2560;                          // smallest row piece of the 4-stage FP8 ring

int encode_weight_map(Params& p);       // host, gemv_abi.cu: 1 when p.tmap_w holds the 16-row box map of p.W

template <int F, int NC, int DEC, bool BAT = false>
size_t tma_prep(Params& p, size_t cap) {
    if (BAT != (p.xm > 0) || (BAT && (p.xm > 8 || p.nops > 0 || p.tp_world > 0))) return 0;
    GemvOp* ops = p.host_ops ? p.host_ops : p.ops;
    // on request, a single GEMV whose rows are whole 64-byte pieces streams full tiles as one tiled tensor copy per stage
    p.tlayout = (p.nops == 0 && !BAT && (p.nchunk & 3) == 0 && p.tensor_on) ? 1 : 0;
    p.tmap_ok = 0;
    if (p.nops > 0) {
        int K = 0, nchunk = 0;
        for (int j = 0; j < p.nops; ++j) {
            K = ops[j].K > K ? ops[j].K : K;
            nchunk = ops[j].nchunk > nchunk ? ops[j].nchunk : nchunk;
        }
        p.K = K;
        p.nchunk = nchunk;
    }
    const long need = ((long)p.nchunk * 16 + 63) / 64 * 64;
    const int want = p.ring;
    if (want == 1 || want > kTmaMaxRing) return 0;
    const long top = need < 4096 ? need : 4096;
    // batched x: no slot below 2 KB per row (smaller pieces make the launch copy-bound); the caller stages fewer x
    // rows instead
    const long kmin = BAT ? (top < 2048 ? top : 2048) : 64;
    bool found = false;
    long kfound = 0;
    // batched x: at least 3 stages (with 2 a launch is latency-bound, measured 2-4x slower than separate calls);
    // the caller stages fewer x rows instead
    for (int rmin = want >= 2 ? want : 3; !found && rmin >= (BAT && want == 0 ? 3 : 2); --rmin) {
        for (long kcs = top; kcs >= kmin; kcs -= 64) {
            tma_apply_slot<F>(p, ops, kcs);
            if (tma_smem_bytes<F, NC, DEC, BAT>(p.K, rmin, p.nch, p.mr, p.st_bytes, p.xm) <= cap) {
                found = true;
                kfound = kcs;
                break;
            }
        }
        if (want >= 2) break;                                 // an explicit ring depth is not lowered
    }
    if (!found) return 0;
    if constexpr (F == kFP8 && DEC == 3 && !BAT) {
        // e4m3 rows that are split into chunks anyway: 4 stages of pieces >= 2.5 KB beat 3 of larger pieces (the
        // 4096 x 14336 projection: 12.9 against 13.9 us); whole rows keep their single-copy slot
        if (want == 0 && p.nops == 0 && p.nch > 1) {
            bool four = false;
            for (long kcs = top; kcs >= kTmaMinPiece4; kcs -= 64) {
                tma_apply_slot<F>(p, ops, kcs);
                if (tma_smem_bytes<F, NC, DEC, BAT>(p.K, 4, p.nch, p.mr, p.st_bytes, p.xm) <= cap) {
                    four = true;
                    break;
                }
            }
            if (!four) tma_apply_slot<F>(p, ops, kfound);
        }
    }
    int ring = want;
    if (ring == 0) {
        ring = 2;
        while (ring < kTmaMaxRing && tma_smem_bytes<F, NC, DEC, BAT>(p.K, ring + 1, p.nch, p.mr, p.st_bytes, p.xm) <= cap)
            ++ring;
    }
    p.ring = ring;
    const size_t total = tma_smem_bytes<F, NC, DEC, BAT>(p.K, ring, p.nch, p.mr, p.st_bytes, p.xm);
    if (total > cap) return 0;
    if (p.tlayout && p.W) p.tmap_ok = encode_weight_map(p);
    return total;
}

// Accumulators of one consumer warp: two chains per unrolled step (BF16: the two k-halves of a step; FP8: even and odd
// 4-byte words; INT4: even and odd 32-weight quarters), so consecutive mma.sync never wait on each other.
template <int U>
struct TmaAcc {
    float a[U][2][4];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int h = 0; h < 2; ++h) a[u][h][0] = a[u][h][1] = a[u][h][2] = a[u][h][3] = 0.f;
    }
};

// NU consecutive 64-byte steps (stage-local step sl, global step gs) of rows g and g + 8 through the tensor cores.
// CHECK: zero the 16-byte chunks beyond the row (only the ragged last step of a BF16/FP8 row needs it).
// INT4: the per-group fold s (D - 136 sum x) (+ z sum x) goes into acc0/acc1 (row g / row g + 8).
template <int F, int DEC, int NU, bool CHECK, int U>
__device__ __forceinline__ void tma_steps(TmaAcc<U>& A, float& acc0, float& acc1, const uint8_t* r0p, const uint8_t* r1p,
                                          const uint16_t* xs, const float* gsum, const uint16_t* sc0,
                                          const uint16_t* sc1, const uint16_t* zr0, const uint16_t* zr1, int sl, int gs,
                                          int c, int nchunk, int xps) {
    constexpr int SK = MmaStep<F>::k;
    uint4 w0[NU], w1[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        w0[u] = *reinterpret_cast<const uint4*>(r0p + 64 * (sl + u));
        w1[u] = *reinterpret_cast<const uint4*>(r1p + 64 * (sl + u));
        if (CHECK && 4 * (gs + u) + c >= nchunk) w0[u] = w1[u] = make_uint4(0u, 0u, 0u, 0u);
    }
    const uint16_t* xb = xs + (size_t)gs * SK + c * (SK / 4);
    if constexpr (F == kBF16) {
        uint4 xv[NU];
#pragma unroll
        for (int u = 0; u < NU; ++u) xv[u] = *reinterpret_cast<const uint4*>(xb + u * SK);
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            mma_bf16(A.a[u][0], w0[u].x, w1[u].x, w0[u].y, w1[u].y, xv[u].x, xv[u].y);
            mma_bf16(A.a[u][1], w0[u].z, w1[u].z, w0[u].w, w1[u].w, xv[u].z, xv[u].w);
        }
    } else if constexpr (F == kFP8 && DEC == 3) {
        // e4m3 weights straight into the tensor cores. x = hi0 + lo0 + 2^-16 (hi1 + lo1) (four e4m3 terms) rides in
        // MMA columns 0-3: lanes of group g supply B column g from plane g & 3, so one mma.sync per 32 weights and row
        // yields all four dot products (columns 4-7 repeat planes 0-3 and are never read).
        const int grp = (int)(threadIdx.x & 31) >> 2;
        const uint8_t* xb8 = reinterpret_cast<const uint8_t*>(xs) + (size_t)gs * 64 + 16 * c + (size_t)(grp & 3) * xps;
        uint4 xv[NU];
#pragma unroll
        for (int u = 0; u < NU; ++u) xv[u] = *reinterpret_cast<const uint4*>(xb8 + 64 * u);
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            mma_e4m3(A.a[u][0], w0[u].x, w1[u].x, w0[u].y, w1[u].y, xv[u].x, xv[u].y);
            mma_e4m3(A.a[u][1], w0[u].z, w1[u].z, w0[u].w, w1[u].w, xv[u].z, xv[u].w);
        }
    } else if constexpr (F == kFP8) {
        uint4 xa[NU], xc[NU];
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            xa[u] = *reinterpret_cast<const uint4*>(xb + u * SK);
            xc[u] = *reinterpret_cast<const uint4*>(xb + u * SK + 8);
        }
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            const uint32_t xv[8] = {xa[u].x, xa[u].y, xa[u].z, xa[u].w, xc[u].x, xc[u].y, xc[u].z, xc[u].w};
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
                const uint32_t a = (&w0[u].x)[t4], b = (&w1[u].x)[t4];
                const bool alu = (DEC == 1) || (DEC == 2 && t4 >= 2);
                float (&d)[4] = A.a[u][DEC == 2 ? (alu ? 1 : 0) : (t4 & 1)];
                if (alu)
                    mma_f16(d, e4m3_pair02_div256(a), e4m3_pair02_div256(b), e4m3_pair13_div256(a),
                            e4m3_pair13_div256(b), xv[2 * t4], xv[2 * t4 + 1]);
                else
                    mma_f16(d, e4m3x2_to_f16x2(a & 0xFFFFu), e4m3x2_to_f16x2(b & 0xFFFFu), e4m3x2_to_f16x2(a >> 16),
                            e4m3x2_to_f16x2(b >> 16), xv[2 * t4], xv[2 * t4 + 1]);
            }
        }
    } else if constexpr (DEC == 2) {
        // INT4, integer MMA against x as four int8 digit planes (balanced base 256); lane group g reads plane g & 3,
        // so MMA column d carries digit d (columns 4-7 repeat them and are never read). One LOP3 per word and nibble
        // half: low nibbles go in as u8 n (chain L), high nibbles unshifted as u8 16 n (chain H), each mma.sync taking
        // two words of one half against the matching even / odd x of those words. Per group:
        // sum_d 256^d (L_d + H_d / 16 - 8 S_d) = sum_d (16 L_d + H_d) 256^d / 16 - C, with C = 8 sum_d 256^d S_d of the
        // lane's digits staged per group (lanes c = 0 / 1 hold digits 0-1 / 2-3; c = 2, 3 hold unused columns).
        // t_d = 16 L_d + H_d stays below 2^22, so a lane's two digits merge in int32 as t_a + 256 t_b (below 2^31)
        // and convert once: (t_a + 256 t_b) 256^a / 16 - C.
        const int grp = (int)(threadIdx.x & 31) >> 2;
        const uint8_t* xp = reinterpret_cast<const uint8_t*>(xs) + (size_t)(grp & 3) * xps + (size_t)gs * 128 + 32 * c;
        const float flo = c == 0 ? 0.0625f : (c == 1 ? 4096.f : 0.f);          // 256^a / 16, a = 0 or 2
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            const uint4 xa = *reinterpret_cast<const uint4*>(xp + 128 * u);
            const uint4 xq = *reinterpret_cast<const uint4*>(xp + 128 * u + 16);
            const uint32_t bx[8] = {xa.x, xa.y, xa.z, xa.w, xq.x, xq.y, xq.z, xq.w};
            int dl[4] = {0, 0, 0, 0}, dh[4] = {0, 0, 0, 0};
#pragma unroll
            for (int h = 0; h < 2; ++h) {                     // words 2h, 2h + 1 of rows g (w0) and g + 8 (w1)
                const uint32_t a0 = (&w0[u].x)[2 * h], b0 = (&w1[u].x)[2 * h];
                const uint32_t a1 = (&w0[u].x)[2 * h + 1], b1 = (&w1[u].x)[2 * h + 1];
                mma_u8s8(dl, a0 & 0x0F0F0F0Fu, b0 & 0x0F0F0F0Fu, a1 & 0x0F0F0F0Fu, b1 & 0x0F0F0F0Fu, bx[4 * h],
                         bx[4 * h + 2]);
                mma_u8s8(dh, a0 & 0xF0F0F0F0u, b0 & 0xF0F0F0F0u, a1 & 0xF0F0F0F0u, b1 & 0xF0F0F0F0u, bx[4 * h + 1],
                         bx[4 * h + 3]);
            }
            const int gidx = 8 * (gs + u);
            const float cg = gsum[gidx + 5 + (c & 1)];
            const int t0 = 16 * dl[0] + dh[0] + 256 * (16 * dl[1] + dh[1]);   // row g
            const int t1 = 16 * dl[2] + dh[2] + 256 * (16 * dl[3] + dh[3]);   // row g + 8
            const float r0 = fmaf((float)t0, flo, -cg);
            const float r1 = fmaf((float)t1, flo, -cg);
            if constexpr (F == kINT4) {
                acc0 = fmaf(__half2float(__ushort_as_half(sc0[sl + u])), r0, acc0);
                acc1 = fmaf(__half2float(__ushort_as_half(sc1[sl + u])), r1, acc1);
            } else {
                const float sx = c == 0 ? gsum[gidx + 4] : 0.f;   // zero term once per row (lane c = 0)
                acc0 = fmaf(bf_lo(sc0[sl + u]), r0, fmaf(bf_lo(zr0[sl + u]), sx, acc0));
                acc1 = fmaf(bf_lo(sc1[sl + u]), r1, fmaf(bf_lo(zr1[sl + u]), sx, acc1));
            }
        }
    } else if constexpr (DEC == 1) {
        // INT4, f16 decode: even k as 1024 + n, odd k as 1024 + 16 n (one LOP3 per pair, one shift per word), each
        // parity in its own MMA chain; fold (D_even + D_odd / 16 - C_g) per group, C_g from the x staging
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            float de[4] = {0.f, 0.f, 0.f, 0.f}, dq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 xq = *reinterpret_cast<const uint4*>(xb + u * SK + 8 * q);
                const uint32_t a = (&w0[u].x)[q], b = (&w1[u].x)[q];
                const uint32_t a8 = a >> 8, b8 = b >> 8;
                mma_f16(de, nib_lo_f16(a), nib_lo_f16(b), nib_lo_f16(a8), nib_lo_f16(b8), xq.x, xq.y);
                mma_f16(dq, nib_hi_f16(a), nib_hi_f16(b), nib_hi_f16(a8), nib_hi_f16(b8), xq.z, xq.w);
            }
            const float cg = gsum[2 * (gs + u)];
            const float r0 = fmaf(dq[0], 0.0625f, de[0]) - cg, r1 = fmaf(dq[2], 0.0625f, de[2]) - cg;
            if constexpr (F == kINT4) {
                acc0 = fmaf(__half2float(__ushort_as_half(sc0[sl + u])), r0, acc0);
                acc1 = fmaf(__half2float(__ushort_as_half(sc1[sl + u])), r1, acc1);
            } else {
                const float sx = gsum[2 * (gs + u) + 1];
                acc0 = fmaf(bf_lo(sc0[sl + u]), r0, fmaf(bf_lo(zr0[sl + u]), sx, acc0));
                acc1 = fmaf(bf_lo(sc1[sl + u]), r1, fmaf(bf_lo(zr1[sl + u]), sx, acc1));
            }
        }
    } else {
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 xq = *reinterpret_cast<const uint4*>(xb + u * SK + 8 * q);
                const uint32_t a = (&w0[u].x)[q], b = (&w1[u].x)[q];
                mma_bf16(d[q & 1], nib_pair_bf16(a, 0), nib_pair_bf16(b, 0), nib_pair_bf16(a, 1), nib_pair_bf16(b, 1),
                         xq.x, xq.y);
                mma_bf16(d[q & 1], nib_pair_bf16(a, 2), nib_pair_bf16(b, 2), nib_pair_bf16(a, 3), nib_pair_bf16(b, 3),
                         xq.z, xq.w);
            }
            // every lane holds rows g and g + 8 (all 8 MMA columns carry the same x), so all lanes fold alike
            const float sx = gsum[2 * (gs + u)];
            const float off = -136.f * sx;
            const float r0 = d[0][0] + d[1][0] + off, r1 = d[0][2] + d[1][2] + off;
            if constexpr (F == kINT4) {
                acc0 = fmaf(__half2float(__ushort_as_half(sc0[sl + u])), r0, acc0);
                acc1 = fmaf(__half2float(__ushort_as_half(sc1[sl + u])), r1, acc1);
            } else {
                acc0 = fmaf(bf_lo(sc0[sl + u]), r0, fmaf(bf_lo(zr0[sl + u]), sx, acc0));
                acc1 = fmaf(bf_lo(sc1[sl + u]), r1, fmaf(bf_lo(zr1[sl + u]), sx, acc1));
            }
        }
    }
}

// Batched INT4 (bf16 128 + n decode, DEC 0): as tma_steps' INT4 DEC 0 branch, but every MMA column is its own x row,
// so the per-group fold uses the column's own sum of x (gl0: column 2c, gl1: column 2c + 1) and keeps four sums per
// lane: rows g, g + 8 x columns 2c, 2c + 1.
template <int F, int NU, bool CHECK>
__device__ __forceinline__ void tma_steps_i4_bat(float (&acc)[4], const uint8_t* r0p, const uint8_t* r1p,
                                                 const uint16_t* xl, const float* gl0, const float* gl1,
                                                 const uint16_t* sc0, const uint16_t* sc1, const uint16_t* zr0,
                                                 const uint16_t* zr1, int sl, int gs, int c, int nchunk) {
    constexpr int SK = MmaStep<F>::k;
    uint4 w0[NU], w1[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        w0[u] = *reinterpret_cast<const uint4*>(r0p + 64 * (sl + u));
        w1[u] = *reinterpret_cast<const uint4*>(r1p + 64 * (sl + u));
        if (CHECK && 4 * (gs + u) + c >= nchunk) w0[u] = w1[u] = make_uint4(0u, 0u, 0u, 0u);
    }
    const uint16_t* xb = xl + (size_t)gs * SK + c * (SK / 4);
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 xq = *reinterpret_cast<const uint4*>(xb + u * SK + 8 * q);
            const uint32_t a = (&w0[u].x)[q], b = (&w1[u].x)[q];
            mma_bf16(d[q & 1], nib_pair_bf16(a, 0), nib_pair_bf16(b, 0), nib_pair_bf16(a, 1), nib_pair_bf16(b, 1),
                     xq.x, xq.y);
            mma_bf16(d[q & 1], nib_pair_bf16(a, 2), nib_pair_bf16(b, 2), nib_pair_bf16(a, 3), nib_pair_bf16(b, 3),
                     xq.z, xq.w);
        }
        const float sx0 = gl0[2 * (gs + u)], sx1 = gl1[2 * (gs + u)];
        const float r[4] = {d[0][0] + d[1][0] - 136.f * sx0, d[0][1] + d[1][1] - 136.f * sx1,
                            d[0][2] + d[1][2] - 136.f * sx0, d[0][3] + d[1][3] - 136.f * sx1};
        if constexpr (F == kINT4) {
            const float s0 = __half2float(__ushort_as_half(sc0[sl + u])), s1 = __half2float(__ushort_as_half(sc1[sl + u]));
            acc[0] = fmaf(s0, r[0], acc[0]); acc[1] = fmaf(s0, r[1], acc[1]);
            acc[2] = fmaf(s1, r[2], acc[2]); acc[3] = fmaf(s1, r[3], acc[3]);
        } else {
            const float s0 = bf_lo(sc0[sl + u]), s1 = bf_lo(sc1[sl + u]);
            const float z0 = bf_lo(zr0[sl + u]), z1 = bf_lo(zr1[sl + u]);
            acc[0] = fmaf(s0, r[0], fmaf(z0, sx0, acc[0])); acc[1] = fmaf(s0, r[1], fmaf(z0, sx1, acc[1]));
            acc[2] = fmaf(s1, r[2], fmaf(z1, sx0, acc[2])); acc[3] = fmaf(s1, r[3], fmaf(z1, sx1, acc[3]));
        }
    }
}

// First row of CTA c (c = gridDim.x: N): equal shares; even rows when the rotary epilogue pairs adjacent rows.
__device__ __forceinline__ int tma_row_begin(const Params& p, int N, unsigned int c) {
    const int r = (int)((long long)c * N / gridDim.x);
    return (p.rope_rows > 0 && c < gridDim.x) ? (r & ~1) : r;
}

// Op j of the launch: the single GEMV of Params (nops == 0) or the layer list.
__device__ __forceinline__ GemvOp tma_op(const Params& p, int j) {
    if (p.op_table) return p.op_table[j];
    if (p.nops > 0) return p.ops[j];
    GemvOp o;
    o.W = p.W; o.s = p.s; o.z = p.z; o.x = p.x; o.bias = p.bias; o.y = p.y;
    o.N = p.N; o.K = p.K; o.nchunk = p.nchunk; o.groups = p.groups; o.nch = p.nch; o.act = 0;
    o.kc = p.kc; o.rs = p.rs;
    return o;
}

// Bounded wait (~2 s) until *c >= target (acquire, gpu scope); on timeout records `code` and returns.
__device__ __forceinline__ void wait_count(const unsigned int* c, unsigned int target, int code) {
    const uint64_t t0 = global_ns();
    for (;;) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= target) return;
        const uint64_t dt = global_ns() - t0;
        if (dt > kAbortCheckNs && tma_aborted()) return;
        if (dt > 2000000000ull) {
            atomicCAS(&g_tma_error, 0, code);
            return;
        }
        __nanosleep(32);
    }
}

// ---------------------------------------------------------------- row-sharded tensor parallelism (tp_world > 0)
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* a) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void red_add_sys(unsigned int* a, unsigned int v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" :: "l"(a), "r"(v) : "memory");
}
// Bounded wait (~1 s over all of them) until blk[base + s] reaches target (wrap-safe) for every rank s but `skip`;
// on timeout records `code` and returns false.
__device__ __forceinline__ bool tp_wait_counts(const unsigned int* blk, int base, int world, int skip,
                                               unsigned int target, int code) {
    const uint64_t t0 = global_ns();
    for (int s = 0; s < world; ++s) {
        if (s == skip) continue;
        while ((int)(ld_acquire_sys(blk + base + s) - target) < 0) {
            const uint64_t dt = global_ns() - t0;
            if (dt > kAbortCheckNs && tma_aborted()) return false;
            if (dt > 1000000000ull) {
                atomicCAS(&g_tma_error, 0, code);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}
// Start of a TP call in one CTA's epilogue warp, after the grid-dependency wait (so the previous call on this rank has
// ended): returns the calls this rank has completed, e. CTA 0 tells every rank that this rank has started call e + 1,
// which orders its readers of call e's y (earlier in its stream) before any peer's stores of this call; then the CTA
// waits (bounded, error 8) until every other rank has started call e + 1 before it stores into their y.
// Every CTA counts itself in on [kTpReaders] after reading the epoch (in both forms, so the count stays (calls) x
// CTAs); in the deferred form tp_leave's CTA 0 advances the epoch only once every CTA of the call has read it.
__device__ __forceinline__ unsigned int tp_enter(const Params& p, int lane) {
    unsigned int* mine = p.tp_flag[p.tp_rank];
    unsigned int e = 0;
    if (lane == 0) {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(e) : "l"(mine + kTpEpoch) : "memory");
        asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" :: "l"(mine + kTpReaders) : "memory");
        if (blockIdx.x == 0)
            for (int r = 0; r < p.tp_world; ++r) red_add_sys(p.tp_flag[r] + kTpReady + p.tp_rank, 1u);
        tp_wait_counts(mine, kTpReady, p.tp_world, p.tp_rank, e + 1u, 8);
    }
    e = __shfl_sync(0xffffffffu, e, 0);
    return e;
}
// End of a TP call in one CTA's epilogue warp: every lane's stores into the ranks' y are released (warp barrier, then
// a system-scope fence by lane 0, cumulative) before this CTA counts itself in on every rank. CTA 0 then waits
// (bounded, error 6) until all CTAs of every rank have counted in on this rank, and advances the epoch: the grid ends
// only when this rank's y is complete.
__device__ __forceinline__ void tp_leave(const Params& p, int lane, unsigned int e) {
    if (p.tp_defer) {                                    // published by the next paia_gemv_tp_exchange
        if (blockIdx.x == 0 && lane == 0) {
            unsigned int* mine = p.tp_flag[p.tp_rank];
            const uint64_t t0 = global_ns();
            unsigned int v;
            for (;;) {
                asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + kTpReaders) : "memory");
                if ((int)(v - (e + 1u) * gridDim.x) >= 0) break;
                const uint64_t dt = global_ns() - t0;
                if (dt > kAbortCheckNs && tma_aborted()) break;
                if (dt > 1000000000ull) { atomicCAS(&g_tma_error, 0, 9); break; }
                __nanosleep(64);
            }
            *reinterpret_cast<volatile unsigned int*>(mine + kTpEpoch) = e + 1u;
        }
        return;
    }
    __syncwarp();
    if (lane == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < p.tp_world; ++r) red_add_sys(p.tp_flag[r] + kTpArrive + p.tp_rank, 1u);
        if (blockIdx.x == 0) {
            // arrivals count complete-form calls only ([kTpComplete], touched by CTA 0 alone), so a buffer set may
            // also take deferred calls, which count none
            unsigned int* mine = p.tp_flag[p.tp_rank];
            const unsigned int cc = *reinterpret_cast<volatile unsigned int*>(mine + kTpComplete);
            tp_wait_counts(mine, kTpArrive, p.tp_world, -1, (cc + 1u) * gridDim.x, 6);
            *reinterpret_cast<volatile unsigned int*>(mine + kTpComplete) = cc + 1u;
            *reinterpret_cast<volatile unsigned int*>(mine + kTpEpoch) = e + 1u;
        }
    }
}

// The exchange after deferred TP calls (one thread): a system-scope fence makes every store this rank's earlier
// kernels made (stream order: they have completed) visible system-wide, then the rank counts itself in on every rank's
// exchange block and waits (bounded, error 6) until every rank has done the same for this exchange.
struct TpExchangeArgs {
    unsigned int* flag[8];
    int world, rank;
};
__global__ void tp_exchange_kernel(const __grid_constant__ TpExchangeArgs a) {
    if (threadIdx.x != 0) return;
    asm volatile("fence.sc.sys;" ::: "memory");
    for (int r = 0; r < a.world; ++r) red_add_sys(a.flag[r] + kTpArrive + a.rank, 1u);
    unsigned int* mine = a.flag[a.rank];
    const unsigned int e = *reinterpret_cast<volatile unsigned int*>(mine + kTpEpoch);
    tp_wait_counts(mine, kTpArrive, a.world, -1, e + 1u, 6);
    *reinterpret_cast<volatile unsigned int*>(mine + kTpEpoch) = e + 1u;
}

// BAT: batched x (p.xm rows, 1..8): x row m rides in MMA column m (lanes of group g read x row g), every D element
// is a (weight row, x row) output, partial buffers hold 16 rows x 8 columns per warp, and y row m is written at
// y + m ldy. Decodes with a per-column fold only: BF16, FP8 DEC 0 (cvt to f16, x scaled per row), INT4 DEC 0.
template <int F, int NC, int U, int DEC = 0, bool BAT = false, bool ROPE = false>
__global__ void __launch_bounds__((NC + 2) * 32, 1) gemv_tma_kernel(const __grid_constant__ Params p) {
    constexpr bool I4 = (F == kINT4 || F == kINT4A);
    static_assert(!BAT || DEC == 0, "batched x uses the per-column decodes");
    constexpr int PC = BAT ? 8 : 1;                           // partial-sum columns per row
    extern __shared__ __align__(128) uint8_t smem[];
    // geometry shared by every op of the launch (p.K: the largest K, p.nch: the smallest NCH, p.cs_slot: the slot)
    const int ST = p.ring;                                    // 2..16 stages (the host checks)
    const int NB = tma_part_bufs(ST, p.nch);
    const int MR = p.mr;
    const int MB = (tma_meta_bytes<F>(MR) + 15) & ~15;
    const int Kpm = tma_kx<F>(p.K);
    const int nops = p.nops > 0 ? p.nops : 1;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kTmaMaxRing;
    uint64_t* tdone = empty + kTmaMaxRing;                    // tile t's NC partials are in buffer t mod NB
    uint64_t* pfree = tdone + kTmaMaxParts;                   // the epilogue warp has read buffer t mod NB
    uint64_t* xready = pfree + kTmaMaxParts;                  // every consumer thread has issued its x loads (op 0)
    volatile int* pstop = reinterpret_cast<volatile int*>(xready + 1);   // producer lane 0 stopped (BF16 / FP8)
    uint8_t* ring = smem + kTmaBarBytes;
    uint8_t* meta = ring + (size_t)ST * p.st_bytes;
    uint16_t* xs = reinterpret_cast<uint16_t*>(meta + (size_t)ST * MB);
    const int XM = BAT ? p.xm : 1;
    const int XROW = tma_xrow_bytes<F, DEC>(p.K);             // bytes per staged x row
    constexpr int GW = tma_gsum_words(DEC);
    const int GR = I4 ? GW * (Kpm / 128) : 0;                 // group-sum floats per x row
    float* gsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + (size_t)XM * XROW);
    float* part = gsum + (size_t)XM * GR;
    float* xscale = part + (size_t)NB * NC * 16 * PC;         // [2][4] (BAT: [8][4]): the x scale per op / x row
    float* xscr = xscale + (BAT ? 32 : 8);                    // 32 floats of x staging scratch

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        // full: INT4 the producer's expect_tx arrival, 32 lanes' cp.async arrivals (metadata) and its closing
        // arrival; BF16 / FP8 (bulk copies only) the expect_tx arrival alone
        for (int s = 0; s < ST; ++s) { mbar_init(&full[s], I4 ? 34 : 1); mbar_init(&empty[s], NC); }
        for (int b = 0; b < NB; ++b) { mbar_init(&tdone[b], NC); mbar_init(&pfree[b], 1); }
        mbar_init(xready, NC * 32);
        *pstop = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NC) {
        // ------------------------------------------------------------ producer warp
        // Streams every op's stages back to back: op j + 1's weights never wait for op j's x.
        const int pre = (p.pre >= 0 && p.pre < ST) ? p.pre : -1;   // -1: never wait
        const uint64_t wpol = l2_evict_first();
        // tiled tensor copies land at 128-byte aligned stage addresses (stage sizes are multiples of 128)
        const bool tensor = p.tmap_ok && p.nops == 0 && (smem_addr(ring) & 127u) == 0;
        int s = 0, g = 0;                                     // ring slot, stage count over all ops
        uint32_t ph = 0;                                      // parity of the slot's previous release
        // Lane 0's slot waits decide whether the warp still refills: a consumer warp releases a slot only after its
        // own wait saw the slot's `full` phase complete, so a successful `empty` wait proves that phase complete
        // and re-arming it is safe. Once an `empty` wait gives up, that is no longer known (a `full` phase can sit
        // at zero pending arrivals while its bytes are in flight, and one more arrival would take the count below
        // zero), so lane 0 arrives on nothing more, and the other lanes stop at the next point where they learn
        // it: INT4 (a shuffle) before their metadata arrivals of the same stage; BF16 / FP8 (no arrivals but lane
        // 0's) from a shared flag that they read at the end of each stage, off the copy-issue path, so at most one
        // stage's bytes land on a phase lane 0 did not arm (its transaction count stays within range). Every other
        // barrier counts arrivals only, which a warp put out of step by a failed wait cannot break.
        bool live = true;
        for (int jo = 0; jo < nops; ++jo) {
            const GemvOp op = tma_op(p, jo);
            const int NCH = op.nch, KC = op.kc, RS = op.rs, CS = KC >> 6;
            const bool dense = !p.tlayout && tma_blocked(NCH, KC, RS);   // short whole rows: one copy per 8-row block
            const int S = (op.nchunk + 3) >> 2;
            const size_t rowbytes = (size_t)op.nchunk * 16;
            const int rb = tma_row_begin(p, op.N, blockIdx.x);
            const int re = tma_row_begin(p, op.N, blockIdx.x + 1);
            const int nst = ((re - rb + 15) >> 4) * NCH;
            const long long NG = (long long)op.N * op.groups;
            // INT4 whole-row stages whose scale (zero) runs start and end on 16-byte boundaries: one bulk copy per
            // tile
            bool meta_bulk = false;
            if constexpr (I4)
                meta_bulk = NCH == 1 && (op.groups & 7) == 0 && (((uintptr_t)op.s & 15) == 0) &&
                            (F == kINT4 || ((uintptr_t)op.z & 15) == 0);
            int t = 0, j = 0;
            for (int i = 0; i < nst; ++i, ++g) {
                const int r0 = rb + 16 * t;
                const int nrows = re - r0 < 16 ? re - r0 : 16;
                const bool last = j == NCH - 1;
                const int nsteps = last ? S - j * CS : CS;
                const uint32_t bytes = last ? (uint32_t)(rowbytes - (size_t)j * KC) : (uint32_t)KC;
                const uint32_t mbytes = meta_bulk ? (uint32_t)(2 * nrows * op.groups) : 0u;   // per metadata array
                // x is read right after the dependency wait, and its loads queue behind whatever this SM has in
                // flight: the producer streams `pre` stages, then waits until every consumer thread has issued its
                // first x loads before it fills the rest of the ring (the weights' latency then overlaps x staging).
                if (lane == 0 && live) {
                    if (g == pre) mbar_wait(xready, 0, 5);
                    if (g >= ST) live = mbar_wait(&empty[s], ph, 1);
                    if (!I4 && !live) *pstop = 1;
                }
                if (lane == 0 && live) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // consumers' reads before copies
                    const uint32_t wbytes = (tensor && nrows == 16) ? 16u * (uint32_t)RS : (uint32_t)nrows * bytes;
                    mbar_arrive_expect_tx(&full[s], wbytes + (F == kINT4A ? 2 : 1) * mbytes);
                    if (meta_bulk) {
                        uint8_t* mdst = meta + (size_t)s * MB + 112;
                        const size_t moff = (size_t)r0 * op.groups * 2;
                        bulk_copy_g2s(mdst, reinterpret_cast<const uint8_t*>(op.s) + moff, mbytes, &full[s]);
                        if constexpr (F == kINT4A)
                            bulk_copy_g2s(mdst + 32 * MR, reinterpret_cast<const uint8_t*>(op.z) + moff, mbytes,
                                          &full[s]);
                    }
                }
                __syncwarp();                                 // the slot is free and its byte count announced
                uint8_t* sdst = ring + (size_t)s * p.st_bytes;
                if (!live) {
                } else if (dense) {                                  // rows 8b .. 8b + 7 of the tile: one copy per block
                    if (lane < 2 && nrows > 8 * lane) {
                        const int nb = nrows - 8 * lane < 8 ? nrows - 8 * lane : 8;
                        bulk_copy_g2s_ef(sdst + (size_t)lane * (8 * RS + 64), op.W + (size_t)(r0 + 8 * lane) * rowbytes,
                                         (uint32_t)(nb * rowbytes), &full[s], wpol);
                    }
                } else if (tensor && nrows == 16) {           // a full tile's stage: one tiled copy of 16 rows
                    if (lane == 0) tensor_copy_g2s_ef(sdst, &p.tmap_w, (j * KC) >> 6, r0, &full[s], wpol);
                } else if (lane < nrows) {
                    bulk_copy_g2s_ef(sdst + (size_t)lane * RS,
                                     op.W + (size_t)(r0 + lane) * rowbytes + (size_t)j * KC, bytes, &full[s], wpol);
                }
                uint8_t* ms = meta + (size_t)s * MB;
                if (!live) {
                } else if constexpr (I4) {
                    uint16_t* msc = reinterpret_cast<uint16_t*>(ms + 112);
                    const uint16_t* sa = reinterpret_cast<const uint16_t*>(op.s);
                    const uint16_t* za = reinterpret_cast<const uint16_t*>(op.z);
                    if (NCH == 1) {
                        // whole rows per stage: the tile's scales (zeros) are one contiguous run of nrows x G halves
                        const long long e0 = (long long)r0 * op.groups;
                        const int n = nrows * op.groups;
                        if (!meta_bulk) {
                            const int nb = u16_blocks16(sa, e0, n);
                            for (int k = lane; k < nb; k += 32) u16_block_copy(msc, sa, e0, k);
                            if constexpr (F == kINT4A) {
                                const int nz = u16_blocks16(za, e0, n);
                                for (int k = lane; k < nz; k += 32) u16_block_copy(msc + 16 * MR, za, e0, k);
                            }
                        }
                    } else {
                        // rows x 16-byte blocks of this stage's scale (and zero) runs, spread over the lanes (a run of
                        // nsteps halves spans at most (nsteps + 21) / 8 blocks)
                        const int bpr = (nsteps + 21) >> 3;
                        for (int it = lane; it < 16 * bpr; it += 32) {
                            const int rr = it / bpr, k = it - rr * bpr;
                            if (rr < nrows) {
                                const long long e0 = (long long)(r0 + rr) * op.groups + (long long)j * CS;
                                if (k < u16_blocks16(sa, e0, nsteps)) u16_block_copy(msc + rr * MR, sa, e0, k);
                                if constexpr (F == kINT4A)
                                    if (k < u16_blocks16(za, e0, nsteps)) u16_block_copy(msc + (16 + rr) * MR, za, e0, k);
                            }
                        }
                    }
                }
                if constexpr (I4) {
                    live = __shfl_sync(0xffffffffu, live, 0); // lane 0's status (see above)
                    if (live) cp_async_arrive(&full[s]);
                    __syncwarp();                             // plain-load halves stored before the closing arrival
                    if (lane == 0 && live) mbar_arrive(&full[s]);
                } else {
                    if (lane != 0 && live) live = *pstop == 0;   // written before this stage's __syncwarp
                }
                if (++s == ST) { s = 0; if (g >= ST) ph ^= 1u; }    // waits from the second pass on: parity 0, 1, 0, ...
                if (++j == NCH) { j = 0; ++t; }
            }
        }
        if (lane == 0 && tma_aborted()) {
            // a wait gave up, so the consumers may not have waited for every stage: keep the CTA (and its shared
            // memory) alive for 200 us, long enough for this warp's copies in flight to land
            const uint64_t t0 = global_ns();
            while (global_ns() - t0 < 200000ull) __nanosleep(1000);
        }
        return;
    }

    if (warp == NC + 1) {
        // ------------------------------------------------------------ epilogue warp
        // Lane r < 16 owns row r of each tile: its row scale and bias are loaded before the wait for the tile's
        // partials (so their latency hides behind the tile's compute); then the NC partials are added in warp order
        // (deterministic), scaled, and stored; the buffer is handed back to the consumers. In layer mode, once all
        // of an op's tiles are stored the CTA counts itself in on the op's counter.
        grid_dependency_wait();                               // y is written only after the preceding grid is done
        const unsigned int tp_e = p.tp_world > 0 ? tp_enter(p, lane) : 0u;
        int b = 0;
        uint32_t bph = 0;
        for (int jo = 0; jo < nops; ++jo) {
            const GemvOp op = tma_op(p, jo);
            const int rb = tma_row_begin(p, op.N, blockIdx.x);
            const int re = tma_row_begin(p, op.N, blockIdx.x + 1);
            const int T = (re - rb + 15) >> 4;
            const float* xsc = xscale + 4 * (jo & 1);
            for (int t = 0; t < T; ++t) {
                const int row = rb + 16 * t + lane;
                const bool mine = lane < 16 && row < re;
                float rs = 1.f, rbias = 0.f;
                if (mine) {
                    if constexpr (F == kFP8) rs = ld_f32(reinterpret_cast<const float*>(op.s) + row);
                    if (op.bias) rbias = __uint_as_float((uint32_t)ld_u16(op.bias + row) << 16);
                }
                mbar_wait(&tdone[b], bph, 3);
                if constexpr (BAT) {
                    // 16 rows x XM x rows: lane pairs (row r, x row m); row scale first, then x row m's scale
                    const float* buf = part + (size_t)b * NC * 16 * 8;
                    for (int idx = lane; idx < 16 * XM; idx += 32) {
                        const int r = idx & 15, m = idx >> 4, rowb = rb + 16 * t + r;
                        if (rowb < re) {
                            float out = 0.f;
#pragma unroll
                            for (int w = 0; w < NC; ++w) out += buf[(w * 16 + r) * 8 + m];
                            if constexpr (F == kFP8)
                                out = out * ld_f32(reinterpret_cast<const float*>(op.s) + rowb) *
                                      __uint_as_float((uint32_t)(__float_as_int(xscale[4 * m]) + 127) << 23);
                            if (op.bias) out += __uint_as_float((uint32_t)ld_u16(op.bias + rowb) << 16);
                            op.y[(size_t)m * p.ldy + rowb] = __float2bfloat16_rn(out);
                        }
                    }
                } else {
                    float val = 0.f;
                    if (mine) {
                        const float* buf = part + (size_t)b * NC * 16;
                        float total = 0.f;
#pragma unroll
                        for (int w = 0; w < NC; ++w) total += buf[w * 16 + lane];
                        // row scale first, then the x scale (products only the row scale keeps finite stay finite)
                        float out = total;
                        if constexpr (F == kFP8)              // row scale, then 2^e (a normal power of two)
                            out = out * rs * __uint_as_float((uint32_t)(__float_as_int(xsc[0]) + 127) << 23);
                        if constexpr (I4 && DEC == 1)         // x was staged as x * 2^-e
                            out = out * __uint_as_float((uint32_t)(__float_as_int(xsc[0]) + 127) << 23);
                        if constexpr (I4 && DEC == 2)         // x was staged as integers x * 2^s
                            out = out * xsc[1];
                        val = out + rbias;
                    }
                    int orow = row;
                    if constexpr (ROPE) {                     // rotary pairs sit in adjacent lanes (even tile starts)
                        const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
                        if (mine && row < p.rope_rows) {
                            const int hd = p.rope_hd, jh = row % hd, i = jh >> 1;
                            float sn, cs;
                            sincosf(p.rope_pos * exp2f(-(float)(2 * i) / (float)hd * p.rope_log2_theta), &sn, &cs);
                            val = (jh & 1) ? fmaf(val, cs, partner * sn) : fmaf(val, cs, -(partner * sn));
                            orow = row - jh + i + (jh & 1) * (hd >> 1);
                        }
                    }
                    if (mine) {
                        const __nv_bfloat16 v = __float2bfloat16_rn(val);
                        if (p.tp_world == 0) {
                            op.y[orow] = v;
                        } else {
                            for (int r = 0; r < p.tp_world; ++r) p.tp_y[r][p.tp_off + row] = v;   // peer stores
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&pfree[b]);
                if (++b == NB) { b = 0; bph ^= 1u; }
            }
            if (p.nops > 0) {
                // this CTA's rows of op jo are stored: the warp barrier orders every lane's stores before lane 0's
                // release fence (cumulative), whose relaxed add then counts the CTA in without a round trip
                __syncwarp();
                if (lane == 0) {
                    asm volatile("fence.acq_rel.gpu;" ::: "memory");
                    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" :: "l"(&p.layer_done[jo]) : "memory");
                }
            }
        }
        if (p.tp_world > 0) tp_leave(p, lane, tp_e);          // this CTA's outputs are on every rank
        if (p.nops > 0) consumer_barrier(2, (NC + 1) * 32);    // this CTA's consumers are past their last wait
        if (p.nops > 0 && lane == 0) {
            // the last CTA through every op zeroes the counters for the next launch (every CTA's consumers have
            // passed all of their waits by then)
            const unsigned int fin = atomicAdd(&p.layer_done[nops], 1u);
            if (fin == gridDim.x - 1) {
                __threadfence();
                for (int jo = 0; jo <= nops; ++jo) atomicExch(&p.layer_done[jo], 0u);
                __threadfence();
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumer warps
    const int g = lane >> 2, c = lane & 3;
    // accumulator chains scaled by 1 (cvt decode, BF16) or 256 (FP8 ALU decode holds value / 256)
    constexpr float f0 = (F == kFP8 && DEC == 1) ? 256.f : 1.f;
    constexpr float f1 = (F == kFP8 && (DEC == 1 || DEC == 2)) ? 256.f : 1.f;
    TmaAcc<U> A;
    A.zero();
    float acc0 = 0.f, acc1 = 0.f;
    float acc4[4] = {0.f, 0.f, 0.f, 0.f};                     // batched INT4: rows g, g + 8 x columns 2c, 2c + 1
    int s = 0, b = 0, tg = 0;                                 // ring slot, partial buffer, tiles over all ops
    uint32_t ph = 0, bph = 0;
    bool seen = true;                                         // every `full` wait of this lane saw its phase complete
    for (int jo = 0; jo < nops; ++jo) {
        const GemvOp op = tma_op(p, jo);
        if (jo == 0) {
            grid_dependency_wait();
        } else {
            // every consumer warp is done with the previous op's x; then every CTA must have stored op jo - 1 (one
            // thread per CTA polls the counter; the barrier passes its acquire on to the others)
            consumer_barrier(1, NC * 32);
            if (tid == 0) wait_count(&p.layer_done[jo - 1], gridDim.x, 7);
            consumer_barrier(1, NC * 32);
        }
        const int NCH = op.nch, RS = op.rs, CS = op.kc >> 6;
        const bool blk = !p.tlayout && tma_blocked(NCH, op.kc, RS);
        const int m0 = tma_tile_row(g, blk), m1 = tma_tile_row(g + 8, blk);   // tile rows of MMA rows g, g + 8
        const int S = (op.nchunk + 3) >> 2;                   // 64-byte steps per row
        const int SF = op.nchunk >> 2;                        // steps whose four 16-byte chunks are all in the row
        const int Kp = tma_kx<F>(op.K);
        const int xps = x_plane_stride<F, DEC>(Kp);           // byte planes of x (FP8 DEC 3, INT4 DEC 2)
        const int rb = tma_row_begin(p, op.N, blockIdx.x);
        const int re = tma_row_begin(p, op.N, blockIdx.x + 1);
        const int nst = ((re - rb + 15) >> 4) * NCH;
        // op 0: every consumer thread tells the producer once its first x loads are issued (or at once without rows)
        const auto issued = [&]() { if (jo == 0) mbar_arrive_relaxed(xready); };
        if (nst > 0) {                                        // CTA-uniform: a CTA without rows of the op skips x
            if constexpr (BAT) {
                for (int m = 0; m < XM; ++m)                  // every x row: its own region, group sums and scale
                    stage_x<F, DEC, tma_gsum_words(DEC)>(
                        XSrc{op.x + (size_t)m * p.ldx, op.K, 0, Kp},
                        reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(xs) + (size_t)m * XROW), gsum + m * GR,
                        xscale + 4 * m, xscr, tid, NC * 32, [&]() { consumer_barrier(1, NC * 32); }, XAll(),
                        [&]() { if (m == 0) issued(); });
            } else {
                stage_x<F, DEC, tma_gsum_words(DEC)>(XSrc{op.x, op.K, op.act, Kp}, xs, gsum, xscale + 4 * (jo & 1),
                                                     xscr, tid, NC * 32, [&]() { consumer_barrier(1, NC * 32); },
                                                     XAll(), issued);
            }
            consumer_barrier(1, NC * 32);
        } else {
            issued();
        }
        if (jo == 0 && tid == 0) launch_dependents();
        const uint16_t* sa = reinterpret_cast<const uint16_t*>(op.s);
        const uint16_t* za = reinterpret_cast<const uint16_t*>(op.z);
        // batched: lanes of group g feed MMA column g with x row g (columns past the last row repeat it, unused)
        const uint16_t* xl = xs;
        const float *gl0 = gsum, *gl1 = gsum;
        if constexpr (BAT) {
            xl = reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(xs) +
                                                   (size_t)(g < XM ? g : XM - 1) * XROW);
            gl0 = gsum + (2 * c < XM ? 2 * c : XM - 1) * GR;
            gl1 = gsum + (2 * c + 1 < XM ? 2 * c + 1 : XM - 1) * GR;
        }
        int t = 0, j = 0;
        for (int i = 0; i < nst; ++i) {
            const int r0 = rb + 16 * t;
            const bool last = j == NCH - 1;
            // a wait that gave up leaves the warp out of step but in the loop (and in the named barriers of layer
            // mode), reading stages that may be in flight; its lane 0 then releases no slot, so the producer never
            // re-arms a `full` phase it cannot prove complete. Lane-local: no vote on the stage loop's path.
            seen = seen && mbar_wait(&full[s], ph, 2);
            const int nsteps = last ? S - j * CS : CS;
            const int sa0 = warp * nsteps / NC, sb0 = (warp + 1) * nsteps / NC;
            const uint8_t* st = ring + (size_t)s * p.st_bytes;
            const uint8_t* ms = meta + (size_t)s * MB;
            const uint8_t* r0p = st + tma_row_off(m0, RS, blk) + 16 * c;
            const uint8_t* r1p = st + tma_row_off(m1, RS, blk) + 16 * c;
            const uint16_t* msc = reinterpret_cast<const uint16_t*>(ms + 112);
            const uint16_t *sc0 = msc, *sc1 = msc, *zr0 = msc, *zr1 = msc;
            if constexpr (I4) {
                if (NCH == 1) {                               // the tile's run: row rr at rr x G (+ run parity)
                    const long long e0 = (long long)r0 * op.groups;
                    sc0 = msc + u16_off16(sa + e0) + m0 * op.groups;
                    sc1 = msc + u16_off16(sa + e0) + m1 * op.groups;
                    if constexpr (F == kINT4A) {
                        zr0 = msc + 16 * MR + u16_off16(za + e0) + m0 * op.groups;
                        zr1 = msc + 16 * MR + u16_off16(za + e0) + m1 * op.groups;
                    }
                } else {                                      // per-row runs: row rr at rr x MR (+ row parity)
                    const long long e0 = (long long)(r0 + m0) * op.groups + (long long)j * CS;
                    const long long e1 = (long long)(r0 + m1) * op.groups + (long long)j * CS;
                    sc0 = msc + m0 * MR + u16_off16(sa + e0);
                    sc1 = msc + m1 * MR + u16_off16(sa + e1);
                    if constexpr (F == kINT4A) {
                        zr0 = msc + (16 + m0) * MR + u16_off16(za + e0);
                        zr1 = msc + (16 + m1) * MR + u16_off16(za + e1);
                    }
                }
            }
            const int gb = j * CS;                            // global step of stage-local step 0
            const int sfull = SF - gb < sb0 ? SF - gb : sb0;  // steps below sfull are whole
            int sl = sa0;
            if constexpr (BAT && I4) {
#pragma unroll 1
                for (; sl + U <= sfull; sl += U)
                    tma_steps_i4_bat<F, U, false>(acc4, r0p, r1p, xl, gl0, gl1, sc0, sc1, zr0, zr1, sl, gb + sl, c,
                                                  op.nchunk);
                for (; sl < sb0; ++sl)
                    tma_steps_i4_bat<F, 1, false>(acc4, r0p, r1p, xl, gl0, gl1, sc0, sc1, zr0, zr1, sl, gb + sl, c,
                                                  op.nchunk);
            } else {
#pragma unroll 1                                      // a compact loop: instruction fetch stalls dominate INT4
                for (; sl + U <= sfull; sl += U)
                    tma_steps<F, DEC, U, false>(A, acc0, acc1, r0p, r1p, xl, gsum, sc0, sc1, zr0, zr1, sl, gb + sl, c,
                                                op.nchunk, xps);
                for (; sl < sfull; ++sl)
                    tma_steps<F, DEC, 1, false>(A, acc0, acc1, r0p, r1p, xl, gsum, sc0, sc1, zr0, zr1, sl, gb + sl, c,
                                                op.nchunk, xps);
                if constexpr (!I4)                            // INT4 rows are whole 64-byte steps (K % 128 == 0)
                    for (; sl < sb0; ++sl)                    // the ragged last step of the row
                        tma_steps<F, DEC, 1, true>(A, acc0, acc1, r0p, r1p, xl, gsum, sc0, sc1, zr0, zr1, sl, gb + sl,
                                                   c, op.nchunk, xps);
            }

            if (last) {
                // tile end: this warp's partial sums of rows g, g + 8 -> buffer b for the epilogue warp (batched:
                // rows g, g + 8 x columns 2c, 2c + 1)
                float s0 = 0.f, s1 = 0.f;
                float sb[4] = {0.f, 0.f, 0.f, 0.f};
                if constexpr (BAT && I4) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) { sb[e] = acc4[e]; acc4[e] = 0.f; }
                } else if constexpr (BAT) {
#pragma unroll
                    for (int u = 0; u < U; ++u)
#pragma unroll
                        for (int e = 0; e < 4; ++e) sb[e] += A.a[u][0][e] + A.a[u][1][e];
                    A.zero();
                } else if constexpr (I4) {
                    s0 = acc0; s1 = acc1;
                    if constexpr (DEC == 2) {                     // digits 0-1 (lane c = 0) + digit 2 (c = 1)
                        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
                        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
                    }
                    acc0 = acc1 = 0.f;
                } else {
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        if constexpr (F == kFP8 && DEC == 3) {    // lanes c = 0: columns 0 + 1 (tier 0); c = 1: 2 + 3
                            s0 += (A.a[u][0][0] + A.a[u][0][1]) + (A.a[u][1][0] + A.a[u][1][1]);
                            s1 += (A.a[u][0][2] + A.a[u][0][3]) + (A.a[u][1][2] + A.a[u][1][3]);
                        } else {
                            s0 += A.a[u][0][0] * f0 + A.a[u][1][0] * f1;
                            s1 += A.a[u][0][2] * f0 + A.a[u][1][2] * f1;
                        }
                    }
                    if constexpr (F == kFP8 && DEC == 3) {        // + 2^-16 tier 1 (exact scaling)
                        s0 = fmaf(__shfl_down_sync(0xffffffffu, s0, 1), 1.52587890625e-05f, s0);
                        s1 = fmaf(__shfl_down_sync(0xffffffffu, s1, 1), 1.52587890625e-05f, s1);
                    }
                    A.zero();
                }
                if (tg >= NB) mbar_wait(&pfree[b], bph ^ 1u, 4);   // the epilogue warp has read tile tg - NB
                ++tg;
                float* buf = part + (size_t)b * NC * 16 * PC;
                if constexpr (BAT) {
                    float* r0b = buf + (warp * 16 + m0) * 8 + 2 * c;
                    float* r1b = buf + (warp * 16 + m1) * 8 + 2 * c;
                    r0b[0] = sb[0]; r0b[1] = sb[1]; r1b[0] = sb[2]; r1b[1] = sb[3];
                } else if (c == 0) {
                    buf[warp * 16 + m0] = s0; buf[warp * 16 + m1] = s1;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&tdone[b]);         // release: this warp's partials of the tile
                if (++b == NB) { b = 0; bph ^= 1u; }
            }
            __syncwarp();
            if (lane == 0 && seen) mbar_arrive(&empty[s]);
            if (++s == ST) { s = 0; ph ^= 1u; }
            if (++j == NCH) { j = 0; ++t; }
        }
    }
    if (p.nops > 0) consumer_barrier(2, (NC + 1) * 32);        // no consumer waits on a counter any more
}

}  // namespace pb2
