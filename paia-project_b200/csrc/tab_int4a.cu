// Asymmetric INT4 W4A16 g128 (bf16 scale and zero) variant table. It has no reference kernel; it reuses the INT4
// tuple space (R {1,2,4,8} x U {1,2,4} x H {0,1} x W {4,8}) so the same tuned tuples apply to both INT4 formats.
// The table's instances use the mixed-precision bf16 FMA path (math 1); the PRMT/fp32 path (math 0) is compiled as
// extra instances reachable through paia_gemv_launch_ex for comparison.
#include "gemv_launch.cuh"

namespace pb2 {
#define PB2_I4(W, R, U, H, M) {R, U, W, 0, H, M, &gemv_kernel<kINT4A, W, R, U, M>, &smem_of<kINT4A, W, R>},
#define PB2_I4_H(W, R, U, M) PB2_I4(W, R, U, 0, M) PB2_I4(W, R, U, 1, M)
#define PB2_I4_U(W, R, M) PB2_I4_H(W, R, 1, M) PB2_I4_H(W, R, 2, M) PB2_I4_H(W, R, 4, M)
#define PB2_I4_R(W, M) PB2_I4_U(W, 1, M) PB2_I4_U(W, 2, M) PB2_I4_U(W, 4, M) PB2_I4_U(W, 8, M)
static const Variant kTable[] = {PB2_I4_R(4, 1) PB2_I4_R(8, 1)};
static const Variant kExtra[] = {PB2_I4_R(4, 0) PB2_I4_R(8, 0)};
#undef PB2_I4_R
#undef PB2_I4_U
#undef PB2_I4_H
#undef PB2_I4

const Variant* table_int4a(int* n) { *n = (int)(sizeof(kTable) / sizeof(kTable[0])); return kTable; }
const Variant* extra_int4a(int* n) { *n = (int)(sizeof(kExtra) / sizeof(kExtra[0])); return kExtra; }
}  // namespace pb2
