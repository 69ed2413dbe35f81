// BF16 variant table: every (R, U, W, S, H) tuple of the reference's BF16 table (src/paia_gemv/gemv_bf16.cu:22-31:
// R {1,2,4} x U {1,2,4,8} x S {0,1} x H {0,1} x W {4,8}), each mapped to a B200 kernel instance.
// S selects the FMA path (0: fp32 conversion + FFMA, 1: mixed-precision bf16 FMA); H selects PDL launch.
#include "gemv_launch.cuh"

namespace pb2 {
#define PB2_BF16(W, R, U, S, H) {R, U, W, S, H, S, &gemv_kernel<kBF16, W, R, U, S>, &smem_of<kBF16, W, R>},
#define PB2_BF16_SH(W, R, U) PB2_BF16(W, R, U, 0, 0) PB2_BF16(W, R, U, 0, 1) PB2_BF16(W, R, U, 1, 0) PB2_BF16(W, R, U, 1, 1)
#define PB2_BF16_U(W, R) PB2_BF16_SH(W, R, 1) PB2_BF16_SH(W, R, 2) PB2_BF16_SH(W, R, 4) PB2_BF16_SH(W, R, 8)
#define PB2_BF16_R(W) PB2_BF16_U(W, 1) PB2_BF16_U(W, 2) PB2_BF16_U(W, 4)
static const Variant kTable[] = {PB2_BF16_R(4) PB2_BF16_R(8)};
#undef PB2_BF16_R
#undef PB2_BF16_U
#undef PB2_BF16_SH
#undef PB2_BF16

const Variant* table_bf16(int* n) { *n = (int)(sizeof(kTable) / sizeof(kTable[0])); return kTable; }
}  // namespace pb2
