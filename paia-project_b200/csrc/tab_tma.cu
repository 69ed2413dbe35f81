// TMA-fed tensor-core kernel instances (gemv_tma.cuh). math 5 = default weight decode of the format, and for FP8
// math 6 = ALU bit decode, math 7 = split cvt/ALU decode, math 8 = e4m3 weights straight into e4m3 mma against x
// split into four e4m3 terms in two exponent tiers; for INT4 math 6 = f16 nibble decode (1024 + n / 1024 + 16 n),
// math 7 = u8 nibbles against x as int8 digits in an integer MMA (exact group sums). Tuple knobs: W = consumer warps
// (plus one producer warp), U = 64-byte steps per consumer iteration. The ring depth and the shared-memory share are
// launch options.
#include "gemv_launch.cuh"
#include "gemv_tma.cuh"

namespace pb2 {

#define PB2_TMA(F, NC, U, H, M, DEC) {0, U, NC, 0, H, M, &gemv_tma_kernel<F, NC, U, DEC>, nullptr, &tma_prep<F, NC, DEC>},
#define PB2_TMA_H(F, NC, U, M, DEC) PB2_TMA(F, NC, U, 0, M, DEC) PB2_TMA(F, NC, U, 1, M, DEC)
#define PB2_TMA_U(F, NC, M, DEC) PB2_TMA_H(F, NC, 2, M, DEC) PB2_TMA_H(F, NC, 4, M, DEC)
#define PB2_TMA_NC(F, M, DEC) PB2_TMA_U(F, 4, M, DEC) PB2_TMA_U(F, 8, M, DEC) PB2_TMA_U(F, 16, M, DEC)
static const Variant kBf16[] = {PB2_TMA_NC(kBF16, 5, 0)};
static const Variant kFp8[] = {PB2_TMA_NC(kFP8, 5, 0)};
static const Variant kFp8Alu[] = {PB2_TMA_NC(kFP8, 6, 1)};
static const Variant kFp8Split[] = {PB2_TMA_NC(kFP8, 7, 2)};
static const Variant kFp8Mma8[] = {PB2_TMA_NC(kFP8, 8, 3)};
static const Variant kInt4[] = {PB2_TMA_NC(kINT4, 5, 0)};
static const Variant kInt4a[] = {PB2_TMA_NC(kINT4A, 5, 0)};
static const Variant kInt4F16[] = {PB2_TMA_NC(kINT4, 6, 1)};
static const Variant kInt4aF16[] = {PB2_TMA_NC(kINT4A, 6, 1)};
static const Variant kInt4I8[] = {PB2_TMA_NC(kINT4, 7, 2)};
static const Variant kInt4aI8[] = {PB2_TMA_NC(kINT4A, 7, 2)};
// batched x (math 9): x rows in the MMA columns, per-column decodes (BF16, FP8 cvt to f16, INT4 bf16 128 + n)
#define PB2_TMA_BAT(F) {0, 2, 8, 0, 1, 9, &gemv_tma_kernel<F, 8, 2, 0, true>, nullptr, &tma_prep<F, 8, 0, true>},
static const Variant kBat[4] = {PB2_TMA_BAT(kBF16) PB2_TMA_BAT(kFP8) PB2_TMA_BAT(kINT4) PB2_TMA_BAT(kINT4A)};
#undef PB2_TMA_BAT
#undef PB2_TMA_NC
#undef PB2_TMA_U
#undef PB2_TMA_H
#undef PB2_TMA

// The TMA-fed kernel as public variants of every format's table (after the reference's tuple grid): R = 0 marks them
// (no reference tuple has R = 0), U = steps per consumer iteration {2, 4}, W = consumer warps {4, 8, 16}, S = 0,
// H = PDL {0, 1}; the format's default decode (BF16 5, FP8 8, INT4 / INT4A 7), the ring as deep as fits. A tuned
// table (src/tuned/<platform>.json) can name them per shape through the unchanged op adapters.
#define PB2_TP(F, NC, U, H, M, DEC) {0, U, NC, 0, H, M, &gemv_tma_kernel<F, NC, U, DEC>, nullptr, &tma_prep<F, NC, DEC>},
#define PB2_TP_H(F, NC, U, M, DEC) PB2_TP(F, NC, U, 0, M, DEC) PB2_TP(F, NC, U, 1, M, DEC)
#define PB2_TP_U(F, NC, M, DEC) PB2_TP_H(F, NC, 2, M, DEC) PB2_TP_H(F, NC, 4, M, DEC)
#define PB2_TP_NC(F, M, DEC) PB2_TP_U(F, 4, M, DEC) PB2_TP_U(F, 8, M, DEC) PB2_TP_U(F, 16, M, DEC)
static const Variant kPubBf16[] = {PB2_TP_NC(kBF16, 5, 0)};
static const Variant kPubFp8[] = {PB2_TP_NC(kFP8, 8, 3)};
static const Variant kPubInt4[] = {PB2_TP_NC(kINT4, 7, 2)};
static const Variant kPubInt4a[] = {PB2_TP_NC(kINT4A, 7, 2)};
#undef PB2_TP_NC
#undef PB2_TP_U
#undef PB2_TP_H
#undef PB2_TP

// The rotary-epilogue instances (paia_gemv_rope): W = 8, U = 2, PDL on, per format its default decode and the
// fallback one. Only these carry the rotary code, so the other instances' epilogue stays as lean as before.
#define PB2_ROPE(F, M, DEC) {0, 2, 8, 0, 1, M, &gemv_tma_kernel<F, 8, 2, DEC, false, true>, nullptr, &tma_prep<F, 8, DEC>},
static const Variant kRope[] = {PB2_ROPE(kBF16, 5, 0) PB2_ROPE(kFP8, 8, 3) PB2_ROPE(kFP8, 5, 0)
                                PB2_ROPE(kINT4, 7, 2) PB2_ROPE(kINT4, 5, 0) PB2_ROPE(kINT4A, 7, 2) PB2_ROPE(kINT4A, 5, 0)};
static const int kRopeFmt[] = {kBF16, kFP8, kFP8, kINT4, kINT4, kINT4A, kINT4A};
#undef PB2_ROPE

#define PB2_N(t) (int)(sizeof(t) / sizeof(t[0]))
const Variant* tma_rope(int fmt, int math) {
    for (int i = 0; i < PB2_N(kRope); ++i)
        if (kRopeFmt[i] == fmt && kRope[i].math == math) return &kRope[i];
    return nullptr;
}
const Variant* tma_public(int fmt, int* n) {
    switch (fmt) {
        case kBF16: *n = PB2_N(kPubBf16); return kPubBf16;
        case kFP8: *n = PB2_N(kPubFp8); return kPubFp8;
        case kINT4: *n = PB2_N(kPubInt4); return kPubInt4;
        case kINT4A: *n = PB2_N(kPubInt4a); return kPubInt4a;
        default: *n = 0; return nullptr;
    }
}
const Variant* tma_instances(int fmt, int math, int* n) {
    *n = 0;
    if (math == 9) {
        if (fmt < 0 || fmt > 3) return nullptr;
        *n = 1;
        return &kBat[fmt];
    }
    if (fmt == kFP8) {
        if (math == 5) { *n = PB2_N(kFp8); return kFp8; }
        if (math == 6) { *n = PB2_N(kFp8Alu); return kFp8Alu; }
        if (math == 7) { *n = PB2_N(kFp8Split); return kFp8Split; }
        if (math == 8) { *n = PB2_N(kFp8Mma8); return kFp8Mma8; }
        return nullptr;
    }
    if (math == 6) {
        if (fmt == kINT4) { *n = PB2_N(kInt4F16); return kInt4F16; }
        if (fmt == kINT4A) { *n = PB2_N(kInt4aF16); return kInt4aF16; }
        return nullptr;
    }
    if (math == 7) {
        if (fmt == kINT4) { *n = PB2_N(kInt4I8); return kInt4I8; }
        if (fmt == kINT4A) { *n = PB2_N(kInt4aI8); return kInt4aI8; }
        return nullptr;
    }
    if (math != 5) return nullptr;
    switch (fmt) {
        case kBF16: *n = PB2_N(kBf16); return kBf16;
        case kINT4: *n = PB2_N(kInt4); return kInt4;
        case kINT4A: *n = PB2_N(kInt4a); return kInt4a;
        default: return nullptr;
    }
}
#undef PB2_N

int launch_tp_exchange(unsigned int* const* flag_all, int world, int rank, cudaStream_t st) {
    TpExchangeArgs a{};
    for (int r = 0; r < world; ++r) a.flag[r] = flag_all[r];
    a.world = world;
    a.rank = rank;
    tp_exchange_kernel<<<1, 32, 0, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
}

// Error word of the bounded waits (1 producer gave up on a free stage, 2 consumer on a full stage, 3 epilogue on a
// tile's partials, 4 consumer on a free partial buffer, 5 producer on the staged x, 6 tensor-parallel arrivals of
// every rank's CTAs, 7 consumer on the previous op of a layer launch, 8 tensor-parallel start of the other ranks).
int tma_device_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tma_error, sizeof(int)) != cudaSuccess) { (void)cudaGetLastError(); return -1; }
    if (clear && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_tma_error, &zero, sizeof(int));
    }
    return v;
}
}  // namespace pb2
