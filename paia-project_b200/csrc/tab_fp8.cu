// FP8 W8A16 variant table: every (R, U, W, H) tuple of the reference's FP8 table (src/paia_gemv/gemv_quant.cu:30-38:
// R {1,2,4} x U {1,2,4} x H {0,1} x W {4,8}), each mapped to a B200 kernel instance (S is reported as 0).
#include "gemv_launch.cuh"

namespace pb2 {
#define PB2_FP8(W, R, U, H) {R, U, W, 0, H, 0, &gemv_kernel<kFP8, W, R, U, 0>, &smem_of<kFP8, W, R>},
#define PB2_FP8_H(W, R, U) PB2_FP8(W, R, U, 0) PB2_FP8(W, R, U, 1)
#define PB2_FP8_U(W, R) PB2_FP8_H(W, R, 1) PB2_FP8_H(W, R, 2) PB2_FP8_H(W, R, 4)
#define PB2_FP8_R(W) PB2_FP8_U(W, 1) PB2_FP8_U(W, 2) PB2_FP8_U(W, 4)
static const Variant kTable[] = {PB2_FP8_R(4) PB2_FP8_R(8)};
#undef PB2_FP8_R
#undef PB2_FP8_U
#undef PB2_FP8_H
#undef PB2_FP8

const Variant* table_fp8(int* n) { *n = (int)(sizeof(kTable) / sizeof(kTable[0])); return kTable; }
}  // namespace pb2
