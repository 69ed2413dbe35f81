// The INT4 control kernels kept for drop-in compatibility (they are measured, never tuned):
//   * naive  (K1 semantics, src/paia_gemv/gemv_int4.cuh:124-152): one row per warp, one 4-byte load of 8 nibbles per
//     lane per iteration, the group scale re-read from global every iteration, a shift/mask/convert per weight.
//   * dequant-to-bf16 (stage 1 of the unfused control, gemv_int4.cuh:154-174, gemv_quant.cu:88-97): writes the
//     dequantised weights (bf16 RNE of (n - 8) * fp16 scale) into a caller-owned scratch matrix [N][K], which the
//     BF16 GEMV then reads back.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace pb2 {

__global__ void __launch_bounds__(128) int4_naive_kernel(const uint8_t* __restrict__ Wq, const __half* __restrict__ sc,
                                                         const __nv_bfloat16* __restrict__ x,
                                                         __nv_bfloat16* __restrict__ y, int N, int K) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= N) return;
    const uint32_t* wr = reinterpret_cast<const uint32_t*>(Wq + (size_t)row * (size_t)(K / 2));
    const __half* sr = sc + (size_t)row * (size_t)(K / 128);
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(x);
    float acc = 0.f;
#pragma unroll 1
    for (int k0 = lane * 8; k0 < K; k0 += 32 * 8) {
        const uint32_t w = wr[k0 / 8];
        const float s = __half2float(sr[k0 / 128]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int n = (int)((w >> (4 * j)) & 0xFu) - 8;
            const uint32_t xp = xw[(k0 + j) / 2];
            const float xv = __uint_as_float((j & 1) ? (xp & 0xFFFF0000u) : (xp << 16));
            acc = fmaf((float)n * s, xv, acc);
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = __float2bfloat16_rn(acc);
}

// 8 weights (one 32-bit word of nibbles) per thread and iteration, grid-stride over the whole matrix.
__global__ void __launch_bounds__(256) int4_dequant_bf16_kernel(const uint8_t* __restrict__ Wq,
                                                                const __half* __restrict__ sc,
                                                                __nv_bfloat16* __restrict__ out, size_t words, int K) {
    const size_t words_per_row = (size_t)K / 8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t w = reinterpret_cast<const uint32_t*>(Wq)[i];
        const size_t row = i / words_per_row;
        const int k = (int)(i - row * words_per_row) * 8;
        const float s = __half2float(sc[row * (size_t)(K / 128) + k / 128]);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = (float)((int)((w >> (8 * j)) & 0xFu) - 8) * s;
            const float b = (float)((int)((w >> (8 * j + 4)) & 0xFu) - 8) * s;
            const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
            o[j] = *reinterpret_cast<const uint32_t*>(&v);
        }
        reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

int launch_int4_naive(const void* Wq, const void* sc, const void* x, void* y, int N, int K, cudaStream_t st) {
    int4_naive_kernel<<<dim3((N + 3) / 4), dim3(128), 0, st>>>((const uint8_t*)Wq, (const __half*)sc,
                                                               (const __nv_bfloat16*)x, (__nv_bfloat16*)y, N, K);
    return (int)cudaGetLastError();
}

int launch_int4_dequant(const void* Wq, const void* sc, void* out, int N, int K, cudaStream_t st) {
    const size_t words = (size_t)N * (size_t)K / 8;
    int4_dequant_bf16_kernel<<<dim3(148 * 8), dim3(256), 0, st>>>((const uint8_t*)Wq, (const __half*)sc,
                                                                   (__nv_bfloat16*)out, words, K);
    return (int)cudaGetLastError();
}

}  // namespace pb2
