// Thin C-ABI shim over the reference's own host format library (TEST INFRASTRUCTURE ONLY).
// It includes Bejaine/PAIA-Project src/paia_gemv/quant_host.h from the read-only reference checkout (the include
// path is given by oracle/Makefile) and exports its functions unchanged, so the tests can compare the oracle in
// oracle/gemv_oracle.c with the reference bit for bit. Built only into oracle/_ref/, never into the product.
#include <cstdint>
#include "quant_host.h"

extern "C" {
float ref_e4m3_decode(uint8_t b) { return paia_host::e4m3_decode(b); }
uint8_t ref_e4m3_encode(float x) { return paia_host::e4m3_encode(x); }
uint16_t ref_f32_to_f16(float f) { return paia_host::f32_to_f16_bits(f); }
float ref_f16_to_f32(uint16_t h) { return paia_host::f16_bits_to_f32(h); }
void ref_quantize_fp8_rowwise(const float* W, int N, int K, uint8_t* q, float* scale) {
    paia_host::quantize_fp8_rowwise(W, N, K, q, scale);
}
void ref_quantize_int4_g128(const float* W, int N, int K, uint8_t* packed, uint16_t* scales) {
    paia_host::quantize_int4_g128(W, N, K, packed, scales);
}
float ref_dequant_fp8(const uint8_t* q, const float* scale, int K, int n, int k) {
    return paia_host::dequant_fp8(q, scale, K, n, k);
}
float ref_dequant_int4(const uint8_t* packed, const uint16_t* scales, int K, int n, int k) {
    return paia_host::dequant_int4(packed, scales, K, n, k);
}
}
