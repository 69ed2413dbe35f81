// Tensor-core dot-product engine for the batch-1 decode GEMV on B200 (sm_100a).
//
// Why: at ~7 TB/s an INT4 GEMV delivers ~12 weights per SM sub-partition per clock and FP8 ~6. Dequantising each
// weight to fp32 and issuing an FFMA costs 3 to 8 issue slots per weight (measured with ncu on the CUDA-core kernel
// of gemv_kernel.cuh, and the reference's kernels recompiled for sm_100a stop at the same ~2.4 / ~4.3 TB/s), so the
// CUDA-core dot product cannot keep up with HBM3e. Here the dequantised weights go straight from registers into
// mma.sync.m16n8k16 (A = weights, B = x in column 0, fp32 accumulate): the tensor core does the multiply and the
// 4-lane reduction, and a lane spends about one issue slot per weight on conversion (INT4: one LOP3 per two weights;
// FP8: one cvt or a few bit operations per two weights; BF16: none). Weights still stream from HBM exactly once in
// 16-byte loads; there is no shared-memory staging of weights.
//
// Fragment mapping (PTX ISA, mma.m16n8k16, .f16/.bf16): lane = 4 g + c. A regs: a0 = (row g, k 2c..2c+1),
// a1 = (row g+8, same k), a2 = (row g, k 2c+8..2c+9), a3 = (row g+8, same k); B regs: b0 = (k 2c..2c+1, col g),
// b1 = (k 2c+8..2c+9, col g); D: d0 = (row g, col 2c), d2 = (row g+8, col 2c). Only output column 0 is used, so the
// lanes with c = 0 hold the results (d0 -> row g, d2 -> row g+8). Because the dot product is a sum over k, the MMA's
// k slots may hold ANY k of the row as long as A and B agree: lane (g, c) feeds its own 16-byte chunk of rows g and
// g+8 (the same k range for every g), and column 0 of B (lanes c = 0..3 of group 0) carries x for those k.
//
// One step = 64 bytes of each of the 16 rows of a tile (lane c loads bytes 16c..16c+15 of the step):
//   BF16  32 k per step, 2 MMAs (bf16). k slots of MMA h: (k0+4h, k0+4h+1) and (k0+4h+2, k0+4h+3), k0 = 32 s + 8 c.
//   FP8   64 k per step, 4 MMAs (f16). Weights: cvt.rn.f16x2.e4m3x2 (exact) or the bit decode below (value/256,
//         exact). x is staged as f16 scaled by 2^-e with e chosen per launch from max|x| (max|x| * 2^-e in
//         [2^14, 2^15)); y = ldexp(D * scale[row], e).
//   INT4  128 k per step = one quantisation group, 8 MMAs (bf16). Word i of the chunk holds k0+8i+j at nibble j;
//         (w >> 4j) & 0x000F000F | 0x43004300 is the bf16 pair (128 + n_{8i+j}, 128 + n_{8i+j+4}). x is staged with
//         each 8-block permuted to pairs (x0,x4),(x1,x5),(x2,x6),(x3,x7) so B loads match. Per group and row:
//         acc += s * (D - 136 * sum_group(x)) (+ z * sum_group(x) for the asymmetric format).
//
// Work split (stream-K inside the CTA): the grid is persistent and CTA c owns the contiguous rows [c N/G, (c+1) N/G),
// cut into 16-row tiles (the last one masked: its loads are clamped to the CTA's last row, its stores skipped). The
// CTA's T tiles x S steps form one linear index space that the NW warps split into equal contiguous ranges, so every
// warp streams the same number of bytes (+-1 step). A tile that lies inside one warp's range is finished by that warp
// alone (no barrier); only the tiles that straddle warp boundaries (at most NW - 1 per CTA) leave partial sums in
// shared memory, which are added in a fixed order once at the end (deterministic results).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include "gemv_kernel.cuh"

namespace pb2 {

template <int F> struct MmaStep;   // k per 64-byte step
template <> struct MmaStep<kBF16> { static constexpr int k = 32; };
template <> struct MmaStep<kFP8> { static constexpr int k = 64; };
template <> struct MmaStep<kINT4> { static constexpr int k = 128; };
template <> struct MmaStep<kINT4A> { static constexpr int k = 128; };

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D += A . B with e4m3 A (16 x 32) and B (32 x 8), fp32 accumulation (exact products).
__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two_bytes, __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}
// e4m3 bytes b0..b3 of w -> f16 pairs holding value/256 exactly (the e4m3 exponent and mantissa bits land on the low
// f16 exponent bits and the top mantissa bits, sign on the sign bit; subnormal codes land on f16 subnormals).
// (b0, b2): magnitudes shift by 7, signs by 8. (b1, b3): magnitudes shift right by 1, signs stay.
__device__ __forceinline__ uint32_t e4m3_pair02_div256(uint32_t w) {
    return ((w << 7) & 0x3F803F80u) | ((w << 8) & 0x80008000u);
}
__device__ __forceinline__ uint32_t e4m3_pair13_div256(uint32_t w) {
    return ((w >> 1) & 0x3F803F80u) | (w & 0x80008000u);
}
__device__ __forceinline__ uint32_t nib_pair_bf16(uint32_t w, int j) {   // (128 + n_j, 128 + n_{j+4}) as bf16x2
    return ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
}
// D += A . B with u8 A (16 x 32) and s8 B (32 x 8), exact int32 accumulation.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// f16 pairs straight from the nibbles: 0x6400 is 1024.0 and the f16 mantissa has 10 bits, so the low nibble of each
// half gives 1024 + n and the second nibble 1024 + 16 n, one LOP3 each.
__device__ __forceinline__ uint32_t nib_lo_f16(uint32_t w) { return (w & 0x000F000Fu) | 0x64006400u; }
__device__ __forceinline__ uint32_t nib_hi_f16(uint32_t w) { return (w & 0x00F000F0u) | 0x64006400u; }

template <int F>
__host__ __device__ constexpr int mma_kpad(int K) { return (K + MmaStep<F>::k - 1) / MmaStep<F>::k * MmaStep<F>::k; }

// Decodes that stage x as four byte planes (FP8 e4m3 terms, DEC 3; INT4 int8 digits, DEC 2): bytes from plane q to
// plane q + 1 for a staged length kp. The lanes of one quarter-warp read two planes at the same step offset, so
// consecutive planes start in different halves of the 32 banks (FP8 reads 16-byte pieces of 64-byte steps: planes
// 64 bytes apart modulo 128; INT4 reads 16-byte pieces 32 bytes apart in 128-byte steps: planes 16 bytes apart).
template <int F, int DEC>
__host__ __device__ constexpr int x_plane_stride(int kp) {
    return (F == kFP8 && DEC == 3) ? ((kp + 127) & ~127) + 64 : kp + 16;
}

// Shared memory: x [Kpad] 16-bit values, then (INT4) sum of x per 128-group [Kpad/128] floats, then the partial sums
// of straddling tiles [NW][2][16] floats, then two words (FP8: the exponent e and 2^-e).
template <int F, int NW>
__host__ __device__ constexpr size_t mma_smem_bytes(int K) {
    return (size_t)mma_kpad<F>(K) * 2 + ((F == kINT4 || F == kINT4A) ? (size_t)(mma_kpad<F>(K) / 128) * 4 : 0) +
           (size_t)2 * NW * 16 * 4 + 16;
}

// Visit the 16-byte blocks i = tid + k nthr < n (k = 0, 1, ...) of x with four blocks' loads in flight per thread
// (one dependent memory round per four blocks instead of one per block); blocks at or past K / 8 read as zeros.
// CACHE 1 keeps the first round's four blocks in `c`, CACHE 2 takes them from `c` instead of loading them again (a
// second pass over x then costs no memory round when K <= 32 nthr).
// x as the staging helpers see it: the vector, its length, and the transform applied on load (kActSiluMul: x holds
// [gate | up], 2K values, and the staged value is bf16(SiLU(gate) * up)).
// kx: the staged length (zero-filled past K; 0 = mma_kpad(K)).
struct XSrc {
    const __nv_bfloat16* x;
    int K;
    int act = 0;
    int kx = 0;
};
// Which 16-byte blocks of x a staging pass visits: count(n) blocks, the q-th being block idx(q); XAll visits all n.
struct XAll {
    __device__ __forceinline__ int count(int n) const { return n; }
    __device__ __forceinline__ int idx(int q) const { return q; }
};
// x is loaded at L2 (ld.global.cg): in a fused sequence of GEMVs it is the output of the previous one, written by
// other CTAs of the same grid, so the non-coherent read-only path must not serve it.
__device__ __forceinline__ uint4 ld_x16(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
// bf16(SiLU(g) * u) of two packed bf16 pairs, SiLU(g) = g / (1 + e^-g) in fp32 with the library expf.
__device__ __forceinline__ uint32_t silu_mul2(uint32_t g, uint32_t u) {
    const float g0 = __uint_as_float(g << 16), g1 = __uint_as_float(g & 0xFFFF0000u);
    const float u0 = __uint_as_float(u << 16), u1 = __uint_as_float(u & 0xFFFF0000u);
    const float a0 = g0 / (1.f + expf(-g0)) * u0, a1 = g1 / (1.f + expf(-g1)) * u1;
    const __nv_bfloat162 r = __floats2bfloat162_rn(a0, a1);
    return *reinterpret_cast<const uint32_t*>(&r);
}
// 16-byte block i of the staged x (i < K / 8); ACT: the SiLU(gate) * up transform (a compile-time choice, so the
// loads of a round issue back to back).
template <bool ACT>
__device__ __forceinline__ uint4 x_block(const uint4* x4, int nx, int i) {
    if constexpr (ACT) {
        const uint4 g = ld_x16(x4 + i), u = ld_x16(x4 + nx + i);
        return make_uint4(silu_mul2(g.x, u.x), silu_mul2(g.y, u.y), silu_mul2(g.z, u.z), silu_mul2(g.w, u.w));
    }
    return ld_x16(x4 + i);
}

// Called once by every thread as soon as its first round of x loads is issued (before their values are used): the
// TMA kernel's producer holds most of its weight copies until then, so the x loads do not queue behind them.
struct NoHook {
    __device__ __forceinline__ void operator()() const {}
};

// R blocks per thread per round (R loads in flight); CACHE 1 keeps the first round's blocks in c[0 .. R), CACHE 2 takes
// them from there. The map is taken by value: a stateful map (a cursor over its runs) restarts on every pass, and
// sees q in increasing order within a thread.
template <bool ACT, int CACHE, int R, typename Fn, typename Map, typename Hook>
__device__ __forceinline__ void x_blocks_t(const XSrc& p, int tid, int nthr, int n0, Fn& fn, uint4* c, Map map,
                                           const Hook& hook) {
    const uint4* x4 = reinterpret_cast<const uint4*>(p.x);
    const int nx = p.K / 8, n = map.count(n0);
    if (tid >= n) hook();                                 // no blocks for this thread
    for (int i0 = tid, r = 0; i0 < n; i0 += R * nthr, ++r) {
        uint4 v[R];
        int ii[R];
#pragma unroll
        for (int k = 0; k < R; ++k) {
            const int q = i0 + k * nthr;
            ii[k] = q < n ? map.idx(q) : nx;
            if (CACHE == 2 && r == 0) v[k] = c[k];
            else v[k] = ii[k] < nx ? x_block<ACT>(x4, nx, ii[k]) : make_uint4(0u, 0u, 0u, 0u);
            if (CACHE == 1 && r == 0) c[k] = v[k];
        }
        if (r == 0) hook();
#pragma unroll
        for (int k = 0; k < R; ++k)
            if (i0 + k * nthr < n) fn(ii[k], v[k]);
    }
}
template <int CACHE = 0, int R = 4, typename Fn, typename Map = XAll, typename Hook = NoHook>
__device__ __forceinline__ void x_blocks(const XSrc& p, int tid, int nthr, int n0, Fn fn, uint4* c = nullptr,
                                         Map map = Map(), const Hook& hook = Hook()) {
    if (p.act == kActSiluMul) x_blocks_t<true, CACHE, R>(p, tid, nthr, n0, fn, c, map, hook);
    else x_blocks_t<false, CACHE, R>(p, tid, nthr, n0, fn, c, map, hook);
}
// As x_blocks, but every thread calls fn(i, v) in every round (i may be >= the staged length; v is then zero), so fn
// may use warp shuffles; blocks q0 + tid of a round belong to consecutive lanes (with a Map, 16 consecutive q of a
// 16-aligned run map to one 128-group: runs are whole groups).
template <bool ACT, int CACHE, int R, typename Fn, typename Map, typename Hook>
__device__ __forceinline__ void x_blocks_all_t(const XSrc& p, int tid, int nthr, int n0, Fn& fn, uint4* c, Map map,
                                               const Hook& hook) {
    const uint4* x4 = reinterpret_cast<const uint4*>(p.x);
    const int nx = p.K / 8, n = map.count(n0);
    if (n <= 0) hook();
    for (int i0 = 0, r = 0; i0 < n; i0 += R * nthr, ++r) {
        uint4 v[R];
        int ii[R];
#pragma unroll
        for (int k = 0; k < R; ++k) {
            const int q = i0 + k * nthr + tid;
            ii[k] = q < n ? map.idx(q) : (1 << 30);
            if (CACHE == 2 && r == 0) v[k] = c[k];
            else v[k] = ii[k] < nx ? x_block<ACT>(x4, nx, ii[k]) : make_uint4(0u, 0u, 0u, 0u);
            if (CACHE == 1 && r == 0) c[k] = v[k];
        }
        if (r == 0) hook();
#pragma unroll
        for (int k = 0; k < R; ++k)
            if (i0 + k * nthr < n) fn(ii[k], v[k]);
    }
}
template <int CACHE = 0, int R = 4, typename Fn, typename Map = XAll, typename Hook = NoHook>
__device__ __forceinline__ void x_blocks_all(const XSrc& p, int tid, int nthr, int n0, Fn fn, uint4* c = nullptr,
                                             Map map = Map(), const Hook& hook = Hook()) {
    if (p.act == kActSiluMul) x_blocks_all_t<true, CACHE, R>(p, tid, nthr, n0, fn, c, map, hook);
    else x_blocks_all_t<false, CACHE, R>(p, tid, nthr, n0, fn, c, map, hook);
}

// Stage x for the tensor-core kernels (padded with zeros to Kpad): BF16 as is; FP8 as f16 scaled by 2^-e (e from the
// CTA-wide max|x|, written to xscale[0] as an int, 2^-e to xscale[1]) with the 4-block order the FP8 decoder DEC
// expects; INT4 with each 8-block permuted to pairs (x0,x4),(x1,x5),(x2,x6),(x3,x7) plus the sum of every 128-group.
// Called by `nthr` threads (thread index tid); `sync` is the barrier over exactly those threads; `scratch` holds
// nthr/32 floats. Ends with x visible to the caller only after the caller's own barrier.
// With a Map, only the mapped blocks are staged (and the max is taken over them). XR: blocks per thread per round.
template <int F, int DEC, int GST = 1, int XR = 4, typename Sync, typename Map = XAll, typename Hook = NoHook>
__device__ __forceinline__ void stage_x(const XSrc& p, uint16_t* xs, float* gsum, float* xscale, float* scratch, int tid,
                                        int nthr, Sync sync, const Map& map = Map(), const Hook& issued = Hook()) {
    // INT4 group sums are written GST words apart (the integer path needs 8 words per group)
    static_assert(!(F == kINT4 || F == kINT4A) || DEC != 2 || GST == 8, "integer INT4 staging needs 8 words per group");
    const int Kp = p.kx ? p.kx : mma_kpad<F>(p.K);
    if constexpr (F == kBF16) {
        x_blocks<0, XR>(p, tid, nthr, Kp / 8, [&](int i, uint4 v) { reinterpret_cast<uint4*>(xs)[i] = v; },   // K % 8 == 0
                        nullptr, map, issued);
        if (tid == 0) { xscale[0] = __int_as_float(0); xscale[1] = 1.f; }
    } else if constexpr (F == kFP8 && DEC == 3) {
        // v = x * 2^-e (max|x| * 2^-e in [128, 256)) as four e4m3 terms in two exponent tiers, one byte plane each
        // (bytes in natural order, plane q at xs + q x_plane_stride): hi0 = RN(v) keeps 4 significant bits and
        // lo0 = RN(v - hi0) the next 4, so hi0 + lo0 == v exactly for |v| >= 2^-2 (bf16 carries 8 significant bits).
        // Below that lo0 (or hi0) falls into the e4m3 subnormals and the rest r = v - hi0 - lo0 (|r| <= 2^-10, exact
        // in fp32) goes into tier 1 at 2^16 r: hi1 = RN(2^16 r), lo1 = RN(2^16 r - hi1). The kernel weighs tier 1 by
        // 2^-16, so x is reproduced exactly for every element within 2^25 of max|x| (an outlier channel of an LLM
        // activation leaves the ordinary elements exact), and smaller ones keep an error below 2^-33 of max|x|.
        float m = 0.f;
        uint4 xc[XR] = {};
        x_blocks<1, XR>(p, tid, nthr, p.K / 8, [&](int, uint4 v) {
            m = fmaxf(m, fmaxf(fmaxf(fmaxf(fabsf(bf_lo(v.x)), fabsf(bf_hi(v.x))), fmaxf(fabsf(bf_lo(v.y)), fabsf(bf_hi(v.y)))),
                               fmaxf(fmaxf(fabsf(bf_lo(v.z)), fabsf(bf_hi(v.z))), fmaxf(fabsf(bf_lo(v.w)), fabsf(bf_hi(v.w))))));
        }, xc, map, issued);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((tid & 31) == 0) scratch[tid >> 5] = m;
        sync();
        if (tid == 0) {
            float mm = 0.f;
            for (int w = 0; w < nthr / 32; ++w) mm = fmaxf(mm, scratch[w]);
            int e = 0;
            if (mm > 0.f && mm <= 3.40282347e38f) {
                const int ex = (int)((__float_as_uint(mm) >> 23) & 0xFF) - 127;
                e = (ex < -126 ? -126 : ex) - 7;
                e = e < -126 ? -126 : (e > 126 ? 126 : e);
            }
            xscale[0] = __int_as_float(e);
            xscale[1] = __uint_as_float((uint32_t)(127 - e) << 23);
        }
        sync();
        const float inv = xscale[1];
        uint8_t* x0 = reinterpret_cast<uint8_t*>(xs);
        const int ps = x_plane_stride<F, DEC>(Kp);
        x_blocks<2, XR>(p, tid, nthr, Kp / 8, [&](int i, uint4 v) {
            uint32_t w[4][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}, {0u, 0u}};
            if (8 * i < p.K) {
                const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 r = make_float2(bf_lo(vv[j]) * inv, bf_hi(vv[j]) * inv);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        // term q of the pair; every residual r - t is exact in fp32, and so is the tier step 2^16
                        const __nv_fp8x2_storage_t t = __nv_cvt_float2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
                        w[q][j >> 1] |= (uint32_t)t << (16 * (j & 1));
                        if (q < 3) {
                            const float2 tf = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(t, __NV_E4M3)));
                            r = make_float2(r.x - tf.x, r.y - tf.y);
                            if (q == 1) r = make_float2(r.x * 65536.f, r.y * 65536.f);
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) reinterpret_cast<uint2*>(x0 + (size_t)q * ps)[i] = make_uint2(w[q][0], w[q][1]);
        }, xc, map);
    } else if constexpr (F == kFP8) {
        // max |x| over the CTA, then x * 2^-e in f16 (exact while max|x| * 2^-e < 2^15 and values stay normal)
        float m = 0.f;
        uint4 xc[XR] = {};
        x_blocks<1, XR>(p, tid, nthr, p.K / 8, [&](int, uint4 v) {
            m = fmaxf(m, fmaxf(fmaxf(fmaxf(fabsf(bf_lo(v.x)), fabsf(bf_hi(v.x))), fmaxf(fabsf(bf_lo(v.y)), fabsf(bf_hi(v.y)))),
                               fmaxf(fmaxf(fabsf(bf_lo(v.z)), fabsf(bf_hi(v.z))), fmaxf(fabsf(bf_lo(v.w)), fabsf(bf_hi(v.w))))));
        }, xc, map, issued);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((tid & 31) == 0) scratch[tid >> 5] = m;
        sync();
        if (tid == 0) {
            float mm = 0.f;
            for (int w = 0; w < nthr / 32; ++w) mm = fmaxf(mm, scratch[w]);
            int e = 0;
            if (mm > 0.f && mm <= 3.40282347e38f) {             // finite and nonzero (NaN compares false)
                const int ex = (int)((__float_as_uint(mm) >> 23) & 0xFF) - 127;   // floor(log2) for normal mm
                e = (ex < -126 ? -126 : ex) - 14;           // max|x| * 2^-e in [2^14, 2^15)
                e = e < -126 ? -126 : (e > 126 ? 126 : e);  // 2^e and 2^-e both normal floats
            }
            xscale[0] = __int_as_float(e);                               // e (applied with ldexpf)
            xscale[1] = __uint_as_float((uint32_t)(127 - e) << 23);      // 2^-e
        }
        sync();
        const float inv = xscale[1];
        x_blocks<2, XR>(p, tid, nthr, Kp / 8, [&](int i, uint4 v) {
            uint4 o = make_uint4(0u, 0u, 0u, 0u);
            if (8 * i < p.K) {
                const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
                uint32_t oo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __half2 h = __floats2half2_rn(bf_lo(vv[j]) * inv, bf_hi(vv[j]) * inv);
                    oo[j] = *reinterpret_cast<const uint32_t*>(&h);
                }
                // words decoded on the ALU pair k (0,2) and (1,3) of each 4-block: store x in that order
                if (DEC == 1 || (DEC == 2 && (i & 1))) {
                    const uint32_t a0 = __byte_perm(oo[0], oo[1], 0x5410), a1 = __byte_perm(oo[0], oo[1], 0x7632);
                    const uint32_t a2 = __byte_perm(oo[2], oo[3], 0x5410), a3 = __byte_perm(oo[2], oo[3], 0x7632);
                    oo[0] = a0; oo[1] = a1; oo[2] = a2; oo[3] = a3;
                }
                o = make_uint4(oo[0], oo[1], oo[2], oo[3]);
            }
            reinterpret_cast<uint4*>(xs)[i] = o;
        }, xc, map);
    } else if constexpr (DEC == 2) {
        // INT4 for the integer MMA: v = x * 2^s rounded to an integer of magnitude < 2^30 (exact for every element
        // within 2^22 of max|x|, bf16 carrying 8 significant bits, so an outlier channel of an LLM activation leaves
        // the ordinary elements exact; smaller ones keep an error below 2^-31 max|x|), split into four signed
        // base-256 digits d0 + 256 d1 + 256^2 d2 + 256^3 d3 (each in [-128, 127]), each an int8 plane of Kpad bytes
        // at xs + d x_plane_stride with every 8-block stored as (x0,x2,x4,x6,x1,x3,x5,x7) (even k pair with the low
        // nibbles). Per 128-group g: sum(v) (float) at gsum[8g + 4] and the symmetric offsets 8 (S_0 + 256 S_1) and
        // 8 256^2 (S_2 + 256 S_3) (S_d = the group's sum of digit d; floats, exact) at gsum[8g + 5] and gsum[8g + 6].
        float m = 0.f;
        bool bad = false;
        uint4 xc[XR] = {};
        x_blocks<1, XR>(p, tid, nthr, p.K / 8, [&](int, uint4 v) {
            const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                bad |= ((vv[j] & 0x7F800000u) == 0x7F800000u) || ((vv[j] & 0x7F80u) == 0x7F80u);
                m = fmaxf(m, fmaxf(fabsf(bf_lo(vv[j])), fabsf(bf_hi(vv[j]))));
            }
        }, xc, map, issued);
        if (__any_sync(0xffffffffu, bad)) m = __int_as_float(0x7F800000);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((tid & 31) == 0) scratch[tid >> 5] = m;
        sync();
        if (tid == 0) {
            float mm = 0.f;
            for (int w = 0; w < nthr / 32; ++w) mm = fmaxf(mm, scratch[w]);
            int sh = 0;
            float inv = 1.f;
            if (!(mm <= 3.40282347e38f)) {
                inv = __int_as_float(0x7FC00000);                         // NaN or infinity in x
            } else if (mm > 0.f) {
                const int ex = (int)((__float_as_uint(mm) >> 23) & 0xFF) - 127;   // floor(log2) (subnormal: -127)
                sh = 29 - (ex < -126 ? -126 : ex);                        // max|x| * 2^sh in [2^29, 2^30)
                sh = sh > 126 ? 126 : sh;                                 // 2^-sh stays a normal float
                inv = __uint_as_float((uint32_t)(127 - sh) << 23);
            }
            xscale[0] = __int_as_float(sh);
            xscale[1] = inv;
        }
        sync();
        const int sh = __float_as_int(xscale[0]);
        // 2^sh as a product of two normal floats (|sh| <= 126)
        const float up = __uint_as_float((uint32_t)(127 + (sh > 0 ? sh / 2 : 0)) << 23);
        const float up2 = __uint_as_float((uint32_t)(127 + (sh > 0 ? sh - sh / 2 : sh)) << 23);
        uint8_t* planes = reinterpret_cast<uint8_t*>(xs);
        const int ps = x_plane_stride<F, DEC>(Kp);
        x_blocks_all<2, XR>(p, tid, nthr, Kp / 8, [&](int i, uint4 v) {
            // blocks past K / 8 arrive as zeros and stage as zero digits
            int s01 = 0, s23 = 0;                            // digit sums packed two per word: S_a + 65536 S_b
            if (i < Kp / 8) {
                const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
                uint32_t t[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float xf = (j & 1) ? bf_hi(vv[j >> 1]) : bf_lo(vv[j >> 1]);
                    // v = x 2^sh exactly (an integer, |v| < 2^30), and t = v + 0x80808080 lies in [0, 2^32): its bytes
                    // are b_d = d_d + 128, the balanced base-256 digits of v offset by 128 (one add per element)
                    t[j] = (uint32_t)__float2int_rn((xf * up) * up2) + 0x80808080u;
                }
                // 4 x 4 byte transposes (element words -> digit planes), evens then odds; b ^ 0x80 is d as an int8
                uint32_t pe[4], po[4];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t* out = h ? po : pe;
                    const uint32_t a = __byte_perm(t[h], t[h + 2], 0x5140), b = __byte_perm(t[h], t[h + 2], 0x7362);
                    const uint32_t c = __byte_perm(t[h + 4], t[h + 6], 0x5140), d = __byte_perm(t[h + 4], t[h + 6], 0x7362);
                    out[0] = __byte_perm(a, c, 0x5410) ^ 0x80808080u;
                    out[1] = __byte_perm(a, c, 0x7632) ^ 0x80808080u;
                    out[2] = __byte_perm(b, d, 0x5410) ^ 0x80808080u;
                    out[3] = __byte_perm(b, d, 0x7632) ^ 0x80808080u;
                }
                int sd[4];
#pragma unroll
                for (int d = 0; d < 4; ++d) {
                    sd[d] = __dp4a((int)pe[d], 0x01010101, __dp4a((int)po[d], 0x01010101, 0));   // |S_d| <= 1024
                    *reinterpret_cast<uint2*>(planes + (size_t)d * ps + 8 * (size_t)i) = make_uint2(pe[d], po[d]);
                }
                s01 = sd[0] + 65536 * sd[1];
                s23 = sd[2] + 65536 * sd[3];
            }
            // over the 16 lanes of a group: every sum stays within +-16384, so the packed halves add without loss
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                s01 += __shfl_xor_sync(0xffffffffu, s01, o);
                s23 += __shfl_xor_sync(0xffffffffu, s23, o);
            }
            if (i < Kp / 8 && (i & 15) == 0) {
                const int gg = i >> 4;
                const int S0 = (int)(short)(s01 & 0xFFFF), S1 = (s01 - S0) >> 16;
                const int S2 = (int)(short)(s23 & 0xFFFF), S3 = (s23 - S2) >> 16;
                const float lo = (float)S0 + 256.f * (float)S1, hi = (float)S2 + 256.f * (float)S3;   // exact
                gsum[8 * gg + 4] = fmaf(hi, 65536.f, lo);
                gsum[8 * gg + 5] = 8.f * lo;
                gsum[8 * gg + 6] = 524288.f * hi;
            }
        }, xc, map);
    } else if constexpr (DEC == 1) {
        // INT4 for the f16 nibble decode: x * 2^-e in f16 (max|x| * 2^-e in [2^13, 2^14)), 8-element blocks stored as
        // pairs (x0,x4),(x2,x6),(x1,x5),(x3,x7) (even k feed the "1024 + n" MMA, odd k the "1024 + 16 n" MMA); per
        // 128-group g: gsum[GST g] = 1032 S_even + 72 S_odd (the decode and symmetric offsets), gsum[GST g + 1] =
        // S_even + S_odd, over the f16 values the MMA sees.
        float m = 0.f;
        uint4 xc[XR] = {};
        x_blocks<1, XR>(p, tid, nthr, p.K / 8, [&](int, uint4 v) {
            m = fmaxf(m, fmaxf(fmaxf(fmaxf(fabsf(bf_lo(v.x)), fabsf(bf_hi(v.x))), fmaxf(fabsf(bf_lo(v.y)), fabsf(bf_hi(v.y)))),
                               fmaxf(fmaxf(fabsf(bf_lo(v.z)), fabsf(bf_hi(v.z))), fmaxf(fabsf(bf_lo(v.w)), fabsf(bf_hi(v.w))))));
        }, xc, map, issued);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((tid & 31) == 0) scratch[tid >> 5] = m;
        sync();
        if (tid == 0) {
            float mm = 0.f;
            for (int w = 0; w < nthr / 32; ++w) mm = fmaxf(mm, scratch[w]);
            int e = 0;
            if (mm > 0.f && mm <= 3.40282347e38f) {
                const int ex = (int)((__float_as_uint(mm) >> 23) & 0xFF) - 127;
                e = (ex < -126 ? -126 : ex) - 13;
                e = e < -126 ? -126 : (e > 126 ? 126 : e);
            }
            xscale[0] = __int_as_float(e);
            xscale[1] = __uint_as_float((uint32_t)(127 - e) << 23);
        }
        sync();
        const float inv = xscale[1];
        const int nb = p.K / 8;                                  // K % 128 == 0 -> nb % 16 == 0
        x_blocks_all<2, XR>(p, tid, nthr, nb, [&](int i, uint4 v) {
            float se = 0.f, so = 0.f;
            if (i < nb) {
                const __half2 h01 = __floats2half2_rn(bf_lo(v.x) * inv, bf_hi(v.x) * inv);
                const __half2 h23 = __floats2half2_rn(bf_lo(v.y) * inv, bf_hi(v.y) * inv);
                const __half2 h45 = __floats2half2_rn(bf_lo(v.z) * inv, bf_hi(v.z) * inv);
                const __half2 h67 = __floats2half2_rn(bf_lo(v.w) * inv, bf_hi(v.w) * inv);
                const uint32_t u01 = *reinterpret_cast<const uint32_t*>(&h01), u23 = *reinterpret_cast<const uint32_t*>(&h23);
                const uint32_t u45 = *reinterpret_cast<const uint32_t*>(&h45), u67 = *reinterpret_cast<const uint32_t*>(&h67);
                reinterpret_cast<uint4*>(xs)[i] = make_uint4(__byte_perm(u01, u45, 0x5410), __byte_perm(u23, u67, 0x5410),
                                                             __byte_perm(u01, u45, 0x7632), __byte_perm(u23, u67, 0x7632));
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                const float2 f45 = __half22float2(h45), f67 = __half22float2(h67);
                se = (f01.x + f23.x) + (f45.x + f67.x);
                so = (f01.y + f23.y) + (f45.y + f67.y);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {                    // 16-lane groups
                se += __shfl_xor_sync(0xffffffffu, se, o);
                so += __shfl_xor_sync(0xffffffffu, so, o);
            }
            if (i < nb && (i & 15) == 0) {
                gsum[GST * (i >> 4)] = 1032.f * se + 72.f * so;
                gsum[GST * (i >> 4) + 1] = se + so;
            }
        }, xc, map);
    } else {
        // 8-element blocks permuted to pairs (x0,x4),(x1,x5),(x2,x6),(x3,x7); sum of each 128-group (16 blocks)
        const int nb = p.K / 8;                                  // K % 128 == 0 -> nb % 16 == 0
        x_blocks_all<0, XR>(p, tid, nthr, nb, [&](int i, uint4 v) {
            float sum = 0.f;
            if (i < nb) {
                const uint32_t pr0 = (v.x & 0xFFFFu) | (v.z << 16);            // (x0, x4)
                const uint32_t pr1 = (v.x >> 16) | (v.z & 0xFFFF0000u);        // (x1, x5)
                const uint32_t pr2 = (v.y & 0xFFFFu) | (v.w << 16);            // (x2, x6)
                const uint32_t pr3 = (v.y >> 16) | (v.w & 0xFFFF0000u);        // (x3, x7)
                reinterpret_cast<uint4*>(xs)[i] = make_uint4(pr0, pr1, pr2, pr3);
                sum = bf_lo(v.x) + bf_hi(v.x) + bf_lo(v.y) + bf_hi(v.y) + bf_lo(v.z) + bf_hi(v.z) + bf_lo(v.w) +
                      bf_hi(v.w);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);   // 16-lane groups
            if (i < nb && (i & 15) == 0) gsum[GST * (i >> 4)] = sum;
        }, nullptr, map, issued);
        if (tid == 0) { xscale[0] = __int_as_float(0); xscale[1] = 1.f; }
    }
}

template <int U>
struct MmaFrag {
    uint4 w0[U], w1[U];        // 16-byte chunks of rows g and g+8 for U steps
    uint32_t m0[U], m1[U];     // INT4: scale bits (INT4A: scale | zero << 16) of rows g and g+8, group = step
    float rs0, rs1, rb0, rb1;  // epilogue data of rows g and g+8 (FP8 row scale, bias), loaded with a tile's step 0
};

// DEC (FP8 only): 0 = every word through cvt.rn.f16x2.e4m3x2; 1 = every word through the ALU bit decode (value/256);
// 2 = words 0,1 of each 16-byte chunk through cvt and words 2,3 through the ALU, which splits the decode between the
// two pipes (the hardware conversion does not run on the ALU pipe and saturates first when used alone).
template <int F, int NW, int U, int DEC = 0>
__global__ void __launch_bounds__(NW * 32) gemv_mma_kernel(const Params p) {
    constexpr bool I4 = (F == kINT4 || F == kINT4A);
    constexpr int SK = MmaStep<F>::k;
    extern __shared__ __align__(16) uint8_t smem[];
    const int Kp = mma_kpad<F>(p.K);
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
    float* gsum = reinterpret_cast<float*>(smem + (size_t)Kp * 2);
    float* part = reinterpret_cast<float*>(smem + (size_t)Kp * 2 + (I4 ? (size_t)(Kp / 128) * 4 : 0));
    float* xscale = part + 2 * NW * 16;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int rb = (int)((long long)blockIdx.x * p.N / gridDim.x);
    const int re = (int)((long long)(blockIdx.x + 1) * p.N / gridDim.x);
    const int T = (re - rb + 15) >> 4;                      // tiles of this CTA
    const int S = (p.nchunk + 3) >> 2;                      // 64-byte steps per row
    const int total = T * S;
    const int wb = (int)((long long)total * warp / NW), we = (int)((long long)total * (warp + 1) / NW);
    const bool ragged = (p.nchunk & 3) != 0;                // the last step of a row is partial
    const size_t rowbytes = (size_t)p.nchunk * 16;
    const int first_tile = wb / S;

    // iteration = (tile t, first step s, n steps): n <= U, never crossing a tile boundary or the end of the range
    auto it_n = [&](int cur) {
        const int s = cur % S;
        int n = S - s;
        if (n > U) n = U;
        if (n > we - cur) n = we - cur;
        return n;
    };

    auto load = [&](MmaFrag<U>& f, int cur) {
        const int t = cur / S, s = cur - t * S, n = it_n(cur);
        const int r0 = rb + t * 16 + g, r1 = r0 + 8;
        const int r0c = r0 < re ? r0 : re - 1, r1c = r1 < re ? r1 : re - 1;   // clamped: loads stay inside W
        const uint8_t* p0 = p.W + (size_t)r0c * rowbytes + (size_t)(4 * s + c) * 16;
        const uint8_t* p1 = p.W + (size_t)r1c * rowbytes + (size_t)(4 * s + c) * 16;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const bool ok = u < n && (!ragged || 4 * (s + u) + c < p.nchunk);
            f.w0[u] = ok ? ld_stream(p0 + 64 * u) : make_uint4(0u, 0u, 0u, 0u);
            f.w1[u] = ok ? ld_stream(p1 + 64 * u) : make_uint4(0u, 0u, 0u, 0u);
        }
        if constexpr (I4) {
            const uint16_t* sp0 = reinterpret_cast<const uint16_t*>(p.s) + (size_t)r0c * p.groups + s;
            const uint16_t* sp1 = reinterpret_cast<const uint16_t*>(p.s) + (size_t)r1c * p.groups + s;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                f.m0[u] = f.m1[u] = 0u;
                if (u < n) {
                    f.m0[u] = ld_u16(sp0 + u);
                    f.m1[u] = ld_u16(sp1 + u);
                    if constexpr (F == kINT4A) {
                        const uint16_t* zp0 = reinterpret_cast<const uint16_t*>(p.z) + (size_t)r0c * p.groups + s;
                        const uint16_t* zp1 = reinterpret_cast<const uint16_t*>(p.z) + (size_t)r1c * p.groups + s;
                        f.m0[u] |= (uint32_t)ld_u16(zp0 + u) << 16;
                        f.m1[u] |= (uint32_t)ld_u16(zp1 + u) << 16;
                    }
                }
            }
        }
        f.rs0 = f.rs1 = 1.f;
        f.rb0 = f.rb1 = 0.f;
        if (s == 0) {
            if constexpr (F == kFP8) {
                f.rs0 = ld_f32(reinterpret_cast<const float*>(p.s) + r0c);
                f.rs1 = ld_f32(reinterpret_cast<const float*>(p.s) + r1c);
            }
            if (p.bias) {
                f.rb0 = __uint_as_float((uint32_t)ld_u16(p.bias + r0c) << 16);
                f.rb1 = __uint_as_float((uint32_t)ld_u16(p.bias + r1c) << 16);
            }
        }
    };

    float D[U][4];                 // BF16/FP8: one accumulator per in-flight step (independent MMA chains)
    float E[U][4];                 // FP8 words decoded on the ALU (value/256), folded in with a factor 256
    float acc0 = 0.f, acc1 = 0.f;  // INT4: scaled per-group sums of rows g and g+8
    float rs0 = 1.f, rs1 = 1.f, rb0 = 0.f, rb1 = 0.f;
    int seg_s = -1;                // first step of the current tile segment (-1: none open)
#pragma unroll
    for (int u = 0; u < U; ++u) D[u][0] = D[u][1] = D[u][2] = D[u][3] = E[u][0] = E[u][1] = E[u][2] = E[u][3] = 0.f;

    auto epilogue = [&](float v, float rs, float rbias) {
        float out = v;
        if constexpr (F == kFP8) out = ldexpf(out * rs, __float_as_int(xscale[0]));   // row scale, then 2^e
        return __float2bfloat16_rn(out + rbias);
    };

    auto compute = [&](const MmaFrag<U>& f, int cur) {
        const int t = cur / S, s = cur - t * S, n = it_n(cur);
        if (seg_s < 0) {
            seg_s = s;
            rs0 = f.rs0; rs1 = f.rs1; rb0 = f.rb0; rb1 = f.rb1;
        }
        bool v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = u < n;              // warp-uniform
        const uint16_t* xb = xs + (size_t)s * SK + c * (SK / 4);
        if constexpr (F == kBF16) {
            uint4 xv[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                xv[u] = v[u] ? *reinterpret_cast<const uint4*>(xb + u * SK) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (v[u]) mma_bf16(D[u], f.w0[u].x, f.w1[u].x, f.w0[u].y, f.w1[u].y, xv[u].x, xv[u].y);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (v[u]) mma_bf16(D[u], f.w0[u].z, f.w1[u].z, f.w0[u].w, f.w1[u].w, xv[u].z, xv[u].w);
        } else if constexpr (F == kFP8) {
            uint32_t xv[U][8];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint4 xa = v[u] ? *reinterpret_cast<const uint4*>(xb + u * SK) : make_uint4(0u, 0u, 0u, 0u);
                const uint4 xc = v[u] ? *reinterpret_cast<const uint4*>(xb + u * SK + 8) : make_uint4(0u, 0u, 0u, 0u);
                xv[u][0] = xa.x; xv[u][1] = xa.y; xv[u][2] = xa.z; xv[u][3] = xa.w;
                xv[u][4] = xc.x; xv[u][5] = xc.y; xv[u][6] = xc.z; xv[u][7] = xc.w;
            }
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
                const bool alu = (DEC == 1) || (DEC == 2 && t4 >= 2);   // which decoder handles word t4
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (!v[u]) continue;
                    const uint32_t a = (&f.w0[u].x)[t4], bb = (&f.w1[u].x)[t4];
                    if (alu)
                        mma_f16(E[u], e4m3_pair02_div256(a), e4m3_pair02_div256(bb), e4m3_pair13_div256(a),
                                e4m3_pair13_div256(bb), xv[u][2 * t4], xv[u][2 * t4 + 1]);
                    else
                        mma_f16(D[u], e4m3x2_to_f16x2(a & 0xFFFFu), e4m3x2_to_f16x2(bb & 0xFFFFu),
                                e4m3x2_to_f16x2(a >> 16), e4m3x2_to_f16x2(bb >> 16), xv[u][2 * t4], xv[u][2 * t4 + 1]);
                }
            }
        } else {
            float d[U][4];
#pragma unroll
            for (int u = 0; u < U; ++u) d[u][0] = d[u][1] = d[u][2] = d[u][3] = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 xq[U];
#pragma unroll
                for (int u = 0; u < U; ++u)      // permuted pairs of 8-block i
                    xq[u] = v[u] ? *reinterpret_cast<const uint4*>(xb + u * SK + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (!v[u]) continue;
                    const uint32_t a = (&f.w0[u].x)[i], bb = (&f.w1[u].x)[i];
                    mma_bf16(d[u], nib_pair_bf16(a, 0), nib_pair_bf16(bb, 0), nib_pair_bf16(a, 1),
                             nib_pair_bf16(bb, 1), xq[u].x, xq[u].y);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (!v[u]) continue;
                    const uint32_t a = (&f.w0[u].x)[i], bb = (&f.w1[u].x)[i];
                    mma_bf16(d[u], nib_pair_bf16(a, 2), nib_pair_bf16(bb, 2), nib_pair_bf16(a, 3),
                             nib_pair_bf16(bb, 3), xq[u].z, xq[u].w);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (!v[u]) continue;
                const float sx = gsum[s + u];
                const float off = -136.f * sx;
                if constexpr (F == kINT4) {
                    acc0 = fmaf(__half2float(__ushort_as_half((unsigned short)(f.m0[u] & 0xFFFFu))), d[u][0] + off, acc0);
                    acc1 = fmaf(__half2float(__ushort_as_half((unsigned short)(f.m1[u] & 0xFFFFu))), d[u][2] + off, acc1);
                } else {
                    acc0 = fmaf(bf_lo(f.m0[u]), d[u][0] + off, acc0);
                    acc0 = fmaf(bf_hi(f.m0[u]), sx, acc0);
                    acc1 = fmaf(bf_lo(f.m1[u]), d[u][2] + off, acc1);
                    acc1 = fmaf(bf_hi(f.m1[u]), sx, acc1);
                }
            }
        }
        // end of this warp's segment of tile t: finish the tile, or leave a partial sum for the cleanup pass
        if (s + n == S || cur + n == we) {
            float s0, s1;
            if constexpr (I4) {
                s0 = acc0; s1 = acc1;
                acc0 = acc1 = 0.f;
            } else {
                s0 = 0.f; s1 = 0.f;
#pragma unroll
                for (int u = 0; u < U; ++u) { s0 += D[u][0]; s1 += D[u][2]; }
                if constexpr (F == kFP8 && DEC != 0) {
                    float e0 = 0.f, e1 = 0.f;
#pragma unroll
                    for (int u = 0; u < U; ++u) { e0 += E[u][0]; e1 += E[u][2]; }
                    s0 = fmaf(256.f, e0, s0);
                    s1 = fmaf(256.f, e1, s1);
                }
#pragma unroll
                for (int u = 0; u < U; ++u)
                    D[u][0] = D[u][1] = D[u][2] = D[u][3] = E[u][0] = E[u][1] = E[u][2] = E[u][3] = 0.f;
            }
            const bool whole = seg_s == 0 && s + n == S;
            if (c == 0) {
                const int r0 = rb + t * 16 + g, r1 = r0 + 8;
                if (whole) {
                    if (r0 < re) p.y[r0] = epilogue(s0, rs0, rb0);
                    if (r1 < re) p.y[r1] = epilogue(s1, rs1, rb1);
                } else {
                    float* slot = part + ((size_t)warp * 2 + (t == first_tile ? 0 : 1)) * 16;
                    slot[g] = s0;
                    slot[g + 8] = s1;
                }
            }
            seg_s = -1;
        }
    };

    MmaFrag<U> fa, fb;
    if (wb < we) load(fa, wb);                  // weights and their metadata: independent of the previous kernel

    grid_dependency_wait();

    stage_x<F, DEC>(XSrc{p.x, p.K}, xs, gsum, xscale, part, tid, NW * 32, []() { __syncthreads(); });
    __syncthreads();
    launch_dependents();

    for (int cur = wb; cur < we;) {
        const int nxt = cur + it_n(cur);
        if (nxt < we) load(fb, nxt);
        compute(fa, cur);
        cur = nxt;
        if (cur >= we) break;
        const int nxt2 = cur + it_n(cur);
        if (nxt2 < we) load(fa, nxt2);
        compute(fb, cur);
        cur = nxt2;
    }

    // Tiles that straddle warp boundaries: add the partial sums of every warp that touched them, in warp order.
    __syncthreads();
    for (int j = tid; j < (NW - 1) * 16; j += NW * 32) {
        const int w = 1 + j / 16, r = j % 16;                 // boundary between warps w-1 and w
        const int bw = (int)((long long)total * w / NW);
        if (bw % S == 0 || bw >= total) continue;             // the boundary does not cut a tile
        const int t = bw / S;
        const int bprev = (int)((long long)total * (w - 1) / NW);
        if (bprev > t * S) continue;                          // an earlier boundary inside this tile handles it
        float sum = 0.f;
        for (int v2 = w - 1; v2 < NW; ++v2) {
            const int vb = (int)((long long)total * v2 / NW), ve = (int)((long long)total * (v2 + 1) / NW);
            if (vb >= (t + 1) * S) break;
            if (ve <= t * S || vb >= ve) continue;
            sum += part[((size_t)v2 * 2 + (t == vb / S ? 0 : 1)) * 16 + r];
        }
        const int row = rb + t * 16 + r;
        if (row < re) {
            float rs = 1.f, rbias = 0.f;
            if constexpr (F == kFP8) rs = ld_f32(reinterpret_cast<const float*>(p.s) + row);
            if (p.bias) rbias = __uint_as_float((uint32_t)ld_u16(p.bias + row) << 16);
            p.y[row] = epilogue(sum, rs, rbias);
        }
    }
}

}  // namespace pb2
