// Tensor-core (mma.sync) kernel instances of every format (gemv_mma.cuh), registered with math = 2.
// Tuple knobs: U = 64-byte steps per lane in flight (x2 with double buffering), W = warps per CTA; R is unused
// (a tile is always 16 rows) and reported as 1.
#include "gemv_launch.cuh"
#include "gemv_mma.cuh"

namespace pb2 {
template <int F, int NW>
size_t mma_smem_of(int K) { return mma_smem_bytes<F, NW>(K); }

#define PB2_MMA(F, W, U, H) {1, U, W, 0, H, 2, &gemv_mma_kernel<F, W, U, 0>, &mma_smem_of<F, W>},
#define PB2_MMA_H(F, W, U) PB2_MMA(F, W, U, 0) PB2_MMA(F, W, U, 1)
#define PB2_MMA_U(F, W) PB2_MMA_H(F, W, 1) PB2_MMA_H(F, W, 2) PB2_MMA_H(F, W, 4)
#define PB2_MMA_W(F) PB2_MMA_U(F, 4) PB2_MMA_U(F, 8) PB2_MMA_U(F, 16)
static const Variant kBf16[] = {PB2_MMA_W(kBF16)};
static const Variant kFp8[] = {PB2_MMA_W(kFP8)};
// FP8 with the ALU decode (math 3) and the split cvt/ALU decode (math 4)
#undef PB2_MMA
#define PB2_MMA(F, W, U, H) {1, U, W, 0, H, 3, &gemv_mma_kernel<F, W, U, 1>, &mma_smem_of<F, W>},
static const Variant kFp8Alu[] = {PB2_MMA_W(kFP8)};
#undef PB2_MMA
#define PB2_MMA(F, W, U, H) {1, U, W, 0, H, 4, &gemv_mma_kernel<F, W, U, 2>, &mma_smem_of<F, W>},
static const Variant kFp8Split[] = {PB2_MMA_W(kFP8)};
#undef PB2_MMA
#define PB2_MMA(F, W, U, H) {1, U, W, 0, H, 2, &gemv_mma_kernel<F, W, U, 0>, &mma_smem_of<F, W>},
static const Variant kInt4[] = {PB2_MMA_W(kINT4)};
static const Variant kInt4a[] = {PB2_MMA_W(kINT4A)};
#undef PB2_MMA_W
#undef PB2_MMA_U
#undef PB2_MMA_H
#undef PB2_MMA

const Variant* mma_instances(int fmt, int math, int* n) {
    if (fmt == kFP8 && math == 3) { *n = (int)(sizeof(kFp8Alu) / sizeof(kFp8Alu[0])); return kFp8Alu; }
    if (fmt == kFP8 && math == 4) { *n = (int)(sizeof(kFp8Split) / sizeof(kFp8Split[0])); return kFp8Split; }
    if (math != 2) { *n = 0; return nullptr; }
    switch (fmt) {
        case kBF16: *n = (int)(sizeof(kBf16) / sizeof(kBf16[0])); return kBf16;
        case kFP8: *n = (int)(sizeof(kFp8) / sizeof(kFp8[0])); return kFp8;
        case kINT4: *n = (int)(sizeof(kInt4) / sizeof(kInt4[0])); return kInt4;
        case kINT4A: *n = (int)(sizeof(kInt4a) / sizeof(kInt4a[0])); return kInt4a;
        default: *n = 0; return nullptr;
    }
}
}  // namespace pb2
