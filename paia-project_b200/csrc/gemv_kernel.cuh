// Batch-1 decode GEMV for B200 (sm_100a): y[N] = dequant(W)[N,K] . x[K] (+ bias), bf16 in and out, fp32 accumulate.
//
// One kernel template serves the four weight formats of the drop-in path (Bejaine/PAIA-Project
// src/paia_gemv/gemv_bf16.cuh:97-134, gemv_fp8.cuh:84-113, gemv_int4.cuh:88-122, plus the asymmetric INT4 format of
// paia-bench/bench/ops/lib_quant.py:159-167). The work is HBM-bound (1 to 4 flops per weight byte), so there are no
// tensor cores: every weight byte is read exactly once with 16-byte streaming loads and dequantised in registers.
//
// B200 design (148 SMs, ~7 TB/s of HBM3e: about 45 KB must be in flight per SM, and INT4 delivers ~14 weights per SM
// sub-partition per clock at full bandwidth, so the dequantisation must cost less than ~2 issue slots per weight):
//   * Persistent grid. The launcher sizes the grid to the number of CTAs that are resident at once (a multiple of
//     the SM count) and gives CTA c the contiguous rows [c*N/G, (c+1)*N/G): every SM streams the same number of rows.
//   * Warps split K. A CTA of NW warps is NR row slots x KS K-slices (NW = NR*KS). A row tile is NR*R rows; the KS warps
//     of a slot each stream a contiguous 1/KS of every row of the slot (16 B per lane per step, 512 B per warp step),
//     and their partial sums meet in shared memory. KS is chosen at launch from K and from the rows per CTA, so short
//     rows (INT4, K=4096: 2 KiB) and few rows per SM both keep all lanes busy.
//   * Register double buffering. Each lane holds R rows x U steps of 16-byte weight chunks for the current iteration
//     while the next iteration's R*U chunks are already in flight, so 2*R*U*16 B per lane are outstanding.
//   * x staged once per CTA in shared memory (bf16, plus the per-chunk sum of x for INT4), read with 16-byte LDS.
//   * Programmatic dependent launch (PDL). The first iteration's weights, scales and bias are loaded BEFORE
//     griddepcontrol.wait; x is read, and y written, only after it. Launched with programmatic stream serialisation,
//     a GEMV therefore streams its weights while the kernel before it (which produces x) finishes, and it triggers
//     its own dependents as soon as x is staged. This requires that W, scales, zeros and bias are not written by the
//     kernel immediately before on the same stream; x may be.
//   * Dequantisation (what each format costs per weight):
//       BF16  MATH 0: shift/mask to fp32 + FFMA.  MATH 1: fma.rn.f32.bf16 (mixed-precision FMA, sm_100) on the packed
//             halves directly; both give identical results (the bf16 x bf16 product is exact in fp32).
//       FP8   cvt.rn.f16x2.e4m3x2 (exact) -> fp32 -> FFMA; the per-row fp32 scale is applied once in the epilogue.
//       INT4  one LOP3 turns two nibbles into the bf16 pair (128 + n_a, 128 + n_b) (0x4300 is 128.0 and the nibble
//             is the low mantissa bits), fma.rn.f32.bf16 multiplies them by x with fp32 accumulation, and the offset
//             is folded per 32-weight chunk: sum((n - 8) x) = sum((128 + n) x) - 136 * sum(x). The per-chunk sum of x is
//             computed once per CTA while x is staged. MATH 0 uses the reference-style PRMT into an fp32 mantissa
//             ((128 + n)/256) and FFMA instead; the two give bit-identical chunk sums up to the 2^-8 factor.
//       INT4A as INT4, then s * chunk + z * sum(x) per group chunk (w = (q - 8) s + z).
//
// Requirements (checked by the C ABI): rows are 16-byte multiples (K % 8 bf16, K % 16 fp8, K % 128 int4), W and x
// 16-byte aligned, K small enough for x to fit in shared memory (K <= 98304).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace pb2 {

enum : int { kBF16 = 0, kFP8 = 1, kINT4 = 2, kINT4A = 3 };

// Transform applied to x while it is staged (layer mode): none, or SiLU(gate) * up with x = [gate | up], 2K values,
// each product rounded to bf16 (the activation between a fused gate_up projection and the down projection).
enum : int { kActNone = 0, kActSiluMul = 1 };

// One GEMV of a fused sequence (TMA kernels' layer mode): operands and shape, and its stage geometry: nch stages per
// 16-row tile, kc row bytes per stage, rs shared-memory row stride.
struct GemvOp {
    const uint8_t* W;
    const void* s;
    const void* z;
    const __nv_bfloat16* x;
    const __nv_bfloat16* bias;
    __nv_bfloat16* y;
    int N, K, nchunk, groups, nch, act, kc, rs;
};
constexpr int kMaxOps = 6;             // ops carried in the kernel parameters
// Tensor-parallel counter block of one rank (uint32 words): epoch, then per-source arrival and ready counts.
// TMA kernels: weight stages streamed before the producer waits for the consumers to issue their x loads (so the x
// loads, on the critical path after the dependency wait, do not queue behind a whole ring of copies). Measured within
// one build through the launch knob (the same binary, so no code-layout effects): FP8 gate_up 20.8 -> 20.3 us, qkv
// 7.29 -> 7.15, INT4 asym lm_head 52.3 -> 51.8, o 5.7 -> 5.5; ties elsewhere.
constexpr int kTmaPreAuto = 1;
constexpr int kTpEpoch = 0, kTpReaders = 4, kTpComplete = 5, kTpArrive = 8, kTpReady = 16, kTpCounterWords = 32;
constexpr int kMaxPlanOps = 4096;       // ops of a plan (device-memory op table)

struct Params {
    const uint8_t* W;              // [N][rowbytes]
    const void* s;                 // FP8: float[N]; INT4: half[N][G]; INT4A: bf16[N][G]; else unused
    const void* z;                 // INT4A: bf16[N][G]
    const __nv_bfloat16* x;        // [K]
    const __nv_bfloat16* bias;     // [N] or nullptr
    __nv_bfloat16* y;              // [N]
    int N, K;
    int nchunk;                    // 16-byte chunks per row
    int ks_log2;                   // log2(KS): warps that share a row
    int groups;                    // K / 128 (INT4 formats)
    int kc, nch, rs, st_bytes;     // TMA kernels: bytes per row per stage, stages per tile, smem row stride, stage size
    // Batched TMA kernels (x holds xm rows, 1..8, ldx elements apart; y rows ldy elements apart): each x row rides in
    // its own MMA column, so the weights stream once for all rows.
    int xm, ldx, ldy;
    int cs_slot;                   // TMA kernels: 64-byte steps a stage slot holds per row
    int mr;                        // TMA kernels: halves per row of a stage's metadata slot
    int ring;                      // TMA kernels: stages in the shared-memory ring
    int pre;                       // TMA kernels: stages streamed before x is staged (0 = the whole ring)
    // TMA kernels, single GEMV, on request (tensor_on; measured slower than the per-row bulk copies on every decode
    // shape, so off by default): W as a 3-D tiled tensor (64 bytes x 64-byte pieces of a row x rows) whose 16-row box
    // lands a whole stage of a full tile in one copy, in the same layout as the per-row copies (row r at r * rs).
    // tmap_ok: the map was encoded (else per-row copies). tlayout: the stage layout is the one the tensor copy lands
    // (no blocked 8-row layout), whichever copies fill it.
    int tensor_on, tlayout, tmap_ok;
    CUtensorMap tmap_w;
    // Row-sharded tensor parallelism (TMA kernels; tp_world = 0: off). Rank tp_rank computes rows [0, N) of its shard
    // and stores each output to every rank's full-size y (peer memory over NVLink) at tp_off + row. tp_flag[r] is
    // rank r's counter block (kTpCounterWords uint32): [kTpEpoch] calls completed on r, [kTpArrive + s] CTAs of rank
    // s that finished their stores into r, [kTpReady + s] calls rank s has started (its readers of the previous y are
    // done). CTA 0 of each launch waits for every rank's CTAs before the grid ends, so y is complete when the kernel
    // is; no rank stores into a peer's y before that peer has started the same call.
    // tp_defer: the deferred form - the kernel only stores (after the start handshake); paia_gemv_tp_exchange publishes
    // and waits later. Every CTA counts itself in on [kTpReaders] once it has read the epoch, and in this form CTA 0
    // advances the epoch only after all of them have.
    int tp_world, tp_off, tp_rank, tp_defer;
    // Rotary embedding fused into the epilogue (single GEMV, rope_rows > 0): rows [0, rope_rows) are q and k heads of
    // rope_hd rows each, stored pair-interleaved (row 2i + h of a head holds dimension i + h rope_hd / 2); the epilogue
    // rotates each pair by pos * theta^(-2i / rope_hd) and stores dimension d of the head at its natural place. CTA
    // row ranges then start on even rows, so a pair never straddles two tiles.
    int rope_rows, rope_hd;
    float rope_pos, rope_log2_theta;
    __nv_bfloat16* tp_y[8];
    unsigned int* tp_flag[8];
    // Layer mode (TMA kernels; nops = 0: off, the single GEMV above). One persistent cooperative launch runs ops
    // 0..nops-1 in order, each op's x being any earlier op's y: the weights of every op stream without a break, and
    // the consumers of op j wait until every CTA has written op j-1 (layer_done[j-1] == grid size). layer_done holds
    // nops + 1 zeroed counters; the last CTA to finish zeroes them again for the next launch.
    // Ops come from `ops` (nops <= kMaxOps) or, for longer sequences (a whole token's GEMVs), from op_table in device
    // memory; host_ops is the host copy the launch geometry is computed from (host only; ops when null).
    int nops;
    unsigned int* layer_done;
    GemvOp ops[kMaxOps];
    const GemvOp* op_table;
    GemvOp* host_ops;
};

template <int F> struct Elems;     // weights per 16-byte chunk
template <> struct Elems<kBF16> { static constexpr int v = 8; };
template <> struct Elems<kFP8> { static constexpr int v = 16; };
template <> struct Elems<kINT4> { static constexpr int v = 32; };
template <> struct Elems<kINT4A> { static constexpr int v = 32; };

// ------------------------------------------------------------------ PTX helpers

// Weights are read once: bypass L1 allocation, read-only path.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint16_t ld_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ float ld_f32(const void* p) {
    float r;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}
// x and y are touched only after this returns (no-op unless launched with programmatic stream serialisation).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// Mixed-precision FMA (PTX ISA 8.6, sm_100): d = a.half(i) * b.half(j) + c with bf16 a, b and fp32 c, d.
#define PB2_FMA_BF16(NAME, SELA, SELB)                                                                      \
    __device__ __forceinline__ float NAME(uint32_t a, uint32_t b, float c) {                                 \
        float d;                                                                                             \
        asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"          \
            "fma.rn.f32.bf16 %0, " SELA ", " SELB ", %3;\n\t}"                                               \
            : "=f"(d) : "r"(a), "r"(b), "f"(c));                                                             \
        return d;                                                                                            \
    }
PB2_FMA_BF16(fma_ll, "al", "bl")
PB2_FMA_BF16(fma_hh, "ah", "bh")
PB2_FMA_BF16(fma_hl, "ah", "bl")
PB2_FMA_BF16(fma_lh, "al", "bh")
#undef PB2_FMA_BF16

// ------------------------------------------------------------------ per-chunk dot products
// Each takes the 16-byte weight chunk w, the chunk's x values (already in registers) and returns acc + w . x.

// BF16: 8 weights, x = one uint4 of 8 bf16 (xf: the same 8 values in fp32, shared by the R rows).
template <int MATH>
__device__ __forceinline__ float dot_bf16(const uint4 w, const uint4 xv, const float (&xf)[8], float acc) {
    if constexpr (MATH == 0) {
        acc = fmaf(bf_lo(w.x), xf[0], acc); acc = fmaf(bf_hi(w.x), xf[1], acc);
        acc = fmaf(bf_lo(w.y), xf[2], acc); acc = fmaf(bf_hi(w.y), xf[3], acc);
        acc = fmaf(bf_lo(w.z), xf[4], acc); acc = fmaf(bf_hi(w.z), xf[5], acc);
        acc = fmaf(bf_lo(w.w), xf[6], acc); acc = fmaf(bf_hi(w.w), xf[7], acc);
    } else {
        acc = fma_ll(w.x, xv.x, acc); acc = fma_hh(w.x, xv.x, acc);
        acc = fma_ll(w.y, xv.y, acc); acc = fma_hh(w.y, xv.y, acc);
        acc = fma_ll(w.z, xv.z, acc); acc = fma_hh(w.z, xv.z, acc);
        acc = fma_ll(w.w, xv.w, acc); acc = fma_hh(w.w, xv.w, acc);
    }
    return acc;
}

// FP8 e4m3: 16 weights; xf = the chunk's 16 x values in fp32. Returns acc + sum(e4m3(w) * x) (scale applied later).
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two_bytes) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two_bytes, __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
__device__ __forceinline__ float dot_fp8(const uint4 w, const float (&xf)[16], float acc) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 a = e4m3x2_to_float2(ws[i] & 0xFFFFu);
        const float2 b = e4m3x2_to_float2(ws[i] >> 16);
        acc = fmaf(a.x, xf[4 * i + 0], acc);
        acc = fmaf(a.y, xf[4 * i + 1], acc);
        acc = fmaf(b.x, xf[4 * i + 2], acc);
        acc = fmaf(b.y, xf[4 * i + 3], acc);
    }
    return acc;
}

// INT4: 32 nibbles (word i holds k = 8i..8i+7, nibble j of a word is k = 8i+j). Returns
//   MATH 1: t + sum((128 + n_k) * x_k)        with bf16 (128 + n) pairs and mixed-precision FMA
//   MATH 0: t + sum((128 + n_k) / 256 * x_k)  with fp32 (128 + n)/256 from one PRMT per weight
// xv[i] = the 8 bf16 x values of word i (uint4), xf = all 32 x values in fp32 (MATH 0 only).
template <int MATH>
__device__ __forceinline__ float dot_int4(const uint4 w, const uint4 (&xv)[4], const float* xf, float t) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    if constexpr (MATH == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = ws[i];
            // pair (n_j, n_{j+4}) of word i, as bf16 (128 + n): low half k = 8i+j, high half k = 8i+j+4
            const uint32_t p0 = (v & 0x000F000Fu) | 0x43004300u;
            const uint32_t p1 = ((v >> 4) & 0x000F000Fu) | 0x43004300u;
            const uint32_t p2 = ((v >> 8) & 0x000F000Fu) | 0x43004300u;
            const uint32_t p3 = ((v >> 12) & 0x000F000Fu) | 0x43004300u;
            // x word layout: xv[i].x = (x[8i], x[8i+1]), .y = (x[8i+2], x[8i+3]), .z = (x[8i+4], x[8i+5]), .w = ...
            t = fma_ll(p0, xv[i].x, t);      // n0 * x0
            t = fma_hl(p0, xv[i].z, t);      // n4 * x4
            t = fma_lh(p1, xv[i].x, t);      // n1 * x1
            t = fma_hh(p1, xv[i].z, t);      // n5 * x5
            t = fma_ll(p2, xv[i].y, t);      // n2 * x2
            t = fma_hl(p2, xv[i].w, t);      // n6 * x6
            t = fma_lh(p3, xv[i].y, t);      // n3 * x3
            t = fma_hh(p3, xv[i].w, t);      // n7 * x7
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t ev = ws[i] & 0x0F0F0F0Fu, od = (ws[i] >> 4) & 0x0F0F0F0Fu;
            // byte j of ev is k = 8i+2j, of od k = 8i+2j+1; [0x3F, n, 0, 0] is the fp32 0.5 + n/256
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                t = fmaf(__uint_as_float(__byte_perm(ev, 0x3F000000u, 0x7044u | (j << 8))), xf[8 * i + 2 * j], t);
                t = fmaf(__uint_as_float(__byte_perm(od, 0x3F000000u, 0x7044u | (j << 8))), xf[8 * i + 2 * j + 1], t);
            }
        }
    }
    return t;
}

// ------------------------------------------------------------------ the kernel

template <int F, int R, int U>
struct Frag {
    uint4 w[R][U];
    uint32_t m[R][U];    // INT4: fp16 scale bits | INT4A: bf16 scale | (bf16 zero << 16)
    float rs[R];         // FP8 row scale
    float rb[R];         // bias (0 when none)
};

// Shared memory: x as bf16 [K] (16-byte aligned), then (INT4 formats) sum of x per 32-chunk [K/32] floats, then the
// cross-warp reduction buffer [2][NW][R] floats.
template <int F, int NW, int R>
__host__ __device__ constexpr size_t smem_bytes(int K) {
    return (size_t)K * 2 + ((F == kINT4 || F == kINT4A) ? (size_t)(K / 32) * 4 : 0) + (size_t)2 * NW * R * 4;
}

template <int F, int NW, int R, int U, int MATH>
__global__ void __launch_bounds__(NW * 32, 1) gemv_kernel(const Params p) {
    constexpr int E = Elems<F>::v;
    constexpr bool I4 = (F == kINT4 || F == kINT4A);
    extern __shared__ __align__(16) uint8_t smem[];
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);
    float* xsum = reinterpret_cast<float*>(smem + (size_t)p.K * 2);
    float* red = reinterpret_cast<float*>(smem + (size_t)p.K * 2 + (I4 ? (size_t)(p.K / 32) * 4 : 0));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ksl = p.ks_log2, KS = 1 << ksl;
    const int rslot = warp >> ksl, kslot = warp & (KS - 1);
    const int NR = NW >> ksl;
    const int rb = (int)((long long)blockIdx.x * p.N / gridDim.x);
    const int re = (int)((long long)(blockIdx.x + 1) * p.N / gridDim.x);
    const int tile_rows = NR * R;
    const int ntiles = (re - rb + tile_rows - 1) / tile_rows;
    const int cb = (int)(((long long)p.nchunk * kslot) >> ksl);
    const int ce = (int)(((long long)p.nchunk * (kslot + 1)) >> ksl);
    const int nsteps = (ce - cb + 31) >> 5;
    const int nbatch = nsteps > U ? (nsteps + U - 1) / U : 1;
    const int nit = ntiles * nbatch;
    const size_t rowbytes = (size_t)p.nchunk * 16;

    auto load = [&](Frag<F, R, U>& f, int t, int b) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = rb + t * tile_rows + rslot * R + r;
            const bool rv = row < re;
            const uint8_t* wrow = p.W + (size_t)row * rowbytes;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = cb + ((b * U + u) << 5) + lane;
                const bool cv = rv && c < ce;
                f.w[r][u] = cv ? ld_stream(wrow + (size_t)c * 16) : make_uint4(0u, 0u, 0u, 0u);
                if constexpr (F == kINT4) {
                    f.m[r][u] = cv ? (uint32_t)ld_u16(reinterpret_cast<const __half*>(p.s) +
                                                      (size_t)row * p.groups + (c >> 2)) : 0u;
                } else if constexpr (F == kINT4A) {
                    const size_t gi = (size_t)row * p.groups + (c >> 2);
                    f.m[r][u] = cv ? ((uint32_t)ld_u16(reinterpret_cast<const __nv_bfloat16*>(p.s) + gi) |
                                      ((uint32_t)ld_u16(reinterpret_cast<const __nv_bfloat16*>(p.z) + gi) << 16)) : 0u;
                }
            }
            if (b == 0) {
                if constexpr (F == kFP8) f.rs[r] = rv ? ld_f32(reinterpret_cast<const float*>(p.s) + row) : 0.f;
                f.rb[r] = (rv && p.bias) ? __uint_as_float((uint32_t)ld_u16(p.bias + row) << 16) : 0.f;
            }
        }
    };

    float acc[R];
    float cur_rs[R], cur_rb[R];
#pragma unroll
    for (int r = 0; r < R; ++r) { acc[r] = 0.f; cur_rs[r] = 0.f; cur_rb[r] = 0.f; }

    auto compute = [&](const Frag<F, R, U>& f, int t, int b) {
        if (b == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) { acc[r] = 0.f; cur_rs[r] = f.rs[r]; cur_rb[r] = f.rb[r]; }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = cb + ((b * U + u) << 5) + lane;
            if (c < ce) {
                const uint4* xp = reinterpret_cast<const uint4*>(xs + (size_t)c * E);
                if constexpr (F == kBF16) {
                    const uint4 xv = xp[0];
                    float xf[8];
                    if constexpr (MATH == 0) {
                        xf[0] = bf_lo(xv.x); xf[1] = bf_hi(xv.x); xf[2] = bf_lo(xv.y); xf[3] = bf_hi(xv.y);
                        xf[4] = bf_lo(xv.z); xf[5] = bf_hi(xv.z); xf[6] = bf_lo(xv.w); xf[7] = bf_hi(xv.w);
                    }
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r] = dot_bf16<MATH>(f.w[r][u], xv, xf, acc[r]);
                } else if constexpr (F == kFP8) {
                    const uint4 xa = xp[0], xb = xp[1];
                    const float xf[16] = {bf_lo(xa.x), bf_hi(xa.x), bf_lo(xa.y), bf_hi(xa.y),
                                          bf_lo(xa.z), bf_hi(xa.z), bf_lo(xa.w), bf_hi(xa.w),
                                          bf_lo(xb.x), bf_hi(xb.x), bf_lo(xb.y), bf_hi(xb.y),
                                          bf_lo(xb.z), bf_hi(xb.z), bf_lo(xb.w), bf_hi(xb.w)};
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r] = dot_fp8(f.w[r][u], xf, acc[r]);
                } else {
                    const uint4 xv[4] = {xp[0], xp[1], xp[2], xp[3]};
                    float xf[MATH == 0 ? 32 : 1];
                    if constexpr (MATH == 0) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            xf[8 * i + 0] = bf_lo(xv[i].x); xf[8 * i + 1] = bf_hi(xv[i].x);
                            xf[8 * i + 2] = bf_lo(xv[i].y); xf[8 * i + 3] = bf_hi(xv[i].y);
                            xf[8 * i + 4] = bf_lo(xv[i].z); xf[8 * i + 5] = bf_hi(xv[i].z);
                            xf[8 * i + 6] = bf_lo(xv[i].w); xf[8 * i + 7] = bf_hi(xv[i].w);
                        }
                    }
                    const float sx = xsum[c];
                    const float off = (MATH == 1) ? -136.f * sx : -0.53125f * sx;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float tch = dot_int4<MATH>(f.w[r][u], xv, xf, off);
                        if constexpr (F == kINT4) {
                            float s = __half2float(__ushort_as_half((unsigned short)(f.m[r][u] & 0xFFFFu)));
                            if constexpr (MATH == 0) s *= 256.f;
                            acc[r] = fmaf(s, tch, acc[r]);
                        } else {
                            float s = bf_lo(f.m[r][u]);
                            const float zz = bf_hi(f.m[r][u]);
                            if constexpr (MATH == 0) s *= 256.f;
                            acc[r] = fmaf(s, tch, acc[r]);
                            acc[r] = fmaf(zz, sx, acc[r]);
                        }
                    }
                }
            }
        }
        if (b == nbatch - 1) {
            // Multi-value butterfly: R partial sums per lane -> after the xor steps lane l holds the warp total of
            // row (l >> (5 - log2 R)); (R - 1) + (5 - log2 R) shuffles instead of 5 R.
            float v[R];
#pragma unroll
            for (int r = 0; r < R; ++r) v[r] = acc[r];
#pragma unroll
            for (int m = R, off = 16; m > 1; m >>= 1, off >>= 1) {
                const bool upper = (lane & off) != 0;
#pragma unroll
                for (int i = 0; i < m / 2; ++i) {
                    const float send = upper ? v[i] : v[i + m / 2];
                    const float keep = upper ? v[i + m / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            float s = v[0];
            constexpr int rl = (R == 1) ? 0 : (R == 2) ? 1 : (R == 4) ? 2 : 3;
#pragma unroll
            for (int off = 16 >> rl; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            const int rr = lane >> (5 - rl);                  // row of this lane's sum
            const bool leader = (lane & ((32 >> rl) - 1)) == 0;
            const int row = rb + t * tile_rows + rslot * R + rr;
            float total = s;
            bool store = leader;
            if (KS > 1) {
                float* buf = red + (size_t)(t & 1) * NW * R;
                if (leader) buf[warp * R + rr] = s;
                asm volatile("bar.sync %0, %1;" :: "r"(1 + rslot), "r"(KS * 32) : "memory");
                store = leader && kslot == 0;
                if (store) {
                    total = 0.f;
                    for (int k = 0; k < KS; ++k) total += buf[(rslot * KS + k) * R + rr];
                }
            }
            if (store && row < re) {
                float rs_v = 1.f, rb_v = 0.f;
#pragma unroll
                for (int r = 0; r < R; ++r) if (r == rr) { rs_v = cur_rs[r]; rb_v = cur_rb[r]; }
                float out = total;
                if constexpr (F == kFP8) out = out * rs_v;
                out = out + rb_v;
                p.y[row] = __float2bfloat16_rn(out);
            }
        }
    };

    Frag<F, R, U> fa, fb;
    if (nit > 0) load(fa, 0, 0);            // weights (and their metadata) only: independent of the previous kernel

    grid_dependency_wait();

    // Stage x (and, for INT4, the sum of each 32-element chunk of x) in shared memory.
    if constexpr (I4) {
        const int nc = p.K >> 5;
        for (int c = tid; c < nc; c += NW * 32) {
            const uint4* src = reinterpret_cast<const uint4*>(p.x + (size_t)c * 32);
            uint4 v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __ldg(src + i);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                reinterpret_cast<uint4*>(xs + (size_t)c * 32)[i] = v[i];
                sum += bf_lo(v[i].x) + bf_hi(v[i].x) + bf_lo(v[i].y) + bf_hi(v[i].y) +
                       bf_lo(v[i].z) + bf_hi(v[i].z) + bf_lo(v[i].w) + bf_hi(v[i].w);
            }
            xsum[c] = sum;
        }
    } else {
        const int n16 = p.K >> 3;
        for (int i = tid; i < n16; i += NW * 32)
            reinterpret_cast<uint4*>(xs)[i] = __ldg(reinterpret_cast<const uint4*>(p.x) + i);
    }
    __syncthreads();
    launch_dependents();

    int t = 0, b = 0;
    for (int it = 0; it < nit;) {
        int t1 = t, b1 = b + 1;
        if (b1 == nbatch) { b1 = 0; ++t1; }
        if (it + 1 < nit) load(fb, t1, b1);
        compute(fa, t, b);
        ++it; t = t1; b = b1;
        if (it >= nit) break;
        int t2 = t, b2 = b + 1;
        if (b2 == nbatch) { b2 = 0; ++t2; }
        if (it + 1 < nit) load(fa, t2, b2);
        compute(fb, t, b);
        ++it; t = t2; b = b2;
    }
}

}  // namespace pb2
