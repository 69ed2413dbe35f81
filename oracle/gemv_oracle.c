/*
 * CPU oracle for the batch-1 decode GEMV family (TEST INFRASTRUCTURE ONLY).
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load it. It restates, in plain C, the reference's number formats and its dequantise-then-matmul definition of
 * the result:
 *
 *   formats   Bejaine/PAIA-Project src/paia_gemv/quant_host.h:18-111 (e4m3 decode/encode, fp16 bits, symmetric INT4
 *             g128 quantiser) and src/paia_gemv/quant.py:8-38 (the torch quantisers and dequantisers that mirror it);
 *             the asymmetric INT4 g128 convention of paia-bench/bench/ops/lib_quant.py:159-167 (quantiser) and
 *             :223-233 (dequantiser), packed like the symmetric format (byte j = weight 2j low nibble, 2j+1 high).
 *   result    y[n] = bf16_RNE( sum_k fp64(dequant(W)[n,k]) * fp64(x[k]) + bias[n] ), the fp32-dequantise-then-matmul
 *             reference of paia-bench/bench/ops/ours_quant.py:69-71 and src/tests/gemv_bf16_check.cu:85-90, carried
 *             in fp64 so that the only rounding left is the final one to bf16.
 *
 * Pinned against the reference itself: tests/golden/ holds vectors produced by the reference's own quant.py and
 * lib_quant.py, and oracle/_ref/ (built by oracle/Makefile from quant_host.h where it lies) is compared bit for bit.
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fPIC -shared (oracle/Makefile). -ffp-contract=off keeps every fp32
 * operation a separately rounded IEEE operation, as torch and the reference's C++ perform them.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---------------------------------------------------------------- e4m3 ("fn": bias 7, no inf, S.1111.111 = NaN) */

/* quant_host.h:18-23. Subnormal codes (e == 0) are m * 2^-9; normal codes are (8 + m) * 2^(e - 10). */
float orc_e4m3_decode(uint8_t b) {
    const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    if (e == 15 && m == 7) return NAN;
    const float v = (e == 0) ? ldexpf((float)m, -9) : ldexpf((float)(8 + m), e - 10);
    return s ? -v : v;
}

/* quant_host.h:26-40: nearest code, ties to the even code, magnitude clamped to 448, sign from signbit (so -0.0 and
 * negative NaN keep the sign bit). The reference searches a table; this computes the same code directly: on a grid of
 * equally spaced codes, "nearest, ties to the even code" is round-half-even of the position on the grid, and the
 * parity of the code is the parity of its mantissa. A NaN input yields code 0 with its sign, as the reference's table
 * search does (every comparison with NaN is false). */
uint8_t orc_e4m3_encode(float x) {
    const uint8_t sign = signbit(x) ? 0x80 : 0;
    const float a = fabsf(x);
    if (isnan(a)) return sign;
    if (!(a < 448.f)) return sign | 0x7E;
    int code;
    if (a < 0.015625f) {                      /* below 2^-6: subnormal grid, step 2^-9 (code 8 is 2^-6 itself) */
        code = (int)nearbyintf(a * 512.f);
    } else {
        int e;
        const float fr = frexpf(a, &e);       /* a = fr * 2^e, fr in [0.5, 1): a = (1 + f) * 2^(e-1) */
        const int q = (int)nearbyintf((2.f * fr - 1.f) * 8.f);   /* mantissa on the 1/8 grid; 8 carries */
        code = ((e - 1 + 7) << 3) + q;
    }
    if (code > 0x7E) code = 0x7E;
    return sign | (uint8_t)code;
}

/* ---------------------------------------------------------------- fp16 / bf16 bit conversions */

/* f32 -> f16 bits, round to nearest even, subnormals, overflow to inf, NaN kept quiet (quant_host.h:42-62). */
uint16_t orc_f32_to_f16(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    const int e = (int)(ax >> 23) - 127;      /* unbiased exponent */
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    if (e >= -14) {                           /* normal half range: keep 10 mantissa bits, RNE on the other 13 */
        uint32_t r = ((uint32_t)(e + 15) << 10) | ((ax >> 13) & 0x3FFu);
        const uint32_t rem = ax & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;   /* a carry into the exponent is still right */
        return (uint16_t)(sign | r);
    }
    if (e < -25) return (uint16_t)sign;       /* below half of the smallest subnormal */
    /* subnormal half: value = m24 * 2^(e-23), quantum 2^-24 -> shift the 24-bit significand right by (-1 - e) */
    const uint32_t m24 = (ax & 0x7FFFFFu) | 0x800000u;
    const int shift = -1 - e;                 /* 14 .. 24 */
    uint32_t r = m24 >> shift;
    const uint32_t rem = m24 & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
}

/* f16 bits -> f32 (exact). */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const int e = (h >> 10) & 0x1F;
    const uint32_t m = h & 0x3FFu;
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    if (e == 0) {
        const float v = ldexpf((float)m, -24);
        return sign ? -v : v;
    }
    return u2f(sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13));
}

/* f32 -> bf16 bits, round to nearest even (torch's .to(torch.bfloat16) on finite values); NaN stays a quiet NaN. */
uint16_t orc_f32_to_bf16(float f) {
    const uint32_t u = f2u(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* f64 -> bf16 bits with a single round-to-nearest-even (no double rounding through f32). */
uint16_t orc_f64_to_bf16(double v) {
    if (isnan(v)) return 0x7FC0;
    const uint16_t sign = signbit(v) ? 0x8000 : 0;
    const double a = fabs(v);
    if (a == 0.0) return sign;
    if (isinf(a)) return sign | 0x7F80;
    int e;
    (void)frexp(a, &e);                        /* a in [2^(e-1), 2^e) */
    int qexp = e - 8;                          /* bf16 keeps 8 significant bits */
    if (qexp < -133) qexp = -133;              /* subnormal quantum 2^-133 */
    const double r = ldexp(nearbyint(ldexp(a, -qexp)), qexp);
    if (r >= 0x1.0p128) return sign | 0x7F80;  /* rounds past the largest finite bf16 */
    const uint32_t u = f2u((float)r);          /* exact: r has <= 8 significant bits */
    return (uint16_t)(sign | (u >> 16));
}

/* ---------------------------------------------------------------- quantisers (formats of the drop-in path) */

/* FP8 W8A16, per output row: scale = amax / 448 (1 when the row is all zero), q = e4m3(w / scale).
 * quant_host.h:74-82, quant.py:8-13. */
void orc_quantize_fp8_rowwise(const float* W, int N, int K, uint8_t* q, float* scale) {
    for (int n = 0; n < N; ++n) {
        const float* w = W + (size_t)n * K;
        float amax = 0.f;
        for (int k = 0; k < K; ++k) { const float a = fabsf(w[k]); if (a > amax) amax = a; }
        const float s = amax > 0.f ? amax / 448.f : 1.f;
        scale[n] = s;
        for (int k = 0; k < K; ++k) q[(size_t)n * K + k] = orc_e4m3_encode(w[k] / s);
    }
}

/* INT4 W4A16 symmetric, group 128 along K: fp16 scale = fp16(amax / 7) (1 when amax == 0, and a zero fp16 scale
 * divides as 1), n = clamp(rint(w / scale), -7, 7) + 8, byte j = n[2j] | n[2j+1] << 4.
 * quant_host.h:88-106, quant.py:20-31. */
void orc_quantize_int4_g128(const float* W, int N, int K, uint8_t* packed, uint16_t* scales) {
    const int G = K / 128;
    for (int n = 0; n < N; ++n) {
        for (int g = 0; g < G; ++g) {
            const float* w = W + (size_t)n * K + (size_t)g * 128;
            float amax = 0.f;
            for (int i = 0; i < 128; ++i) { const float a = fabsf(w[i]); if (a > amax) amax = a; }
            const uint16_t sb = orc_f32_to_f16(amax > 0.f ? amax / 7.f : 1.f);
            scales[(size_t)n * G + g] = sb;
            float sf = orc_f16_to_f32(sb);
            if (!(sf > 0.f)) sf = 1.f;
            for (int i = 0; i < 128; i += 2) {
                int q0 = (int)nearbyintf(w[i] / sf), q1 = (int)nearbyintf(w[i + 1] / sf);
                q0 = (q0 < -7 ? -7 : q0 > 7 ? 7 : q0) + 8;
                q1 = (q1 < -7 ? -7 : q1 > 7 ? 7 : q1) + 8;
                packed[(size_t)n * (K / 2) + (size_t)(g * 128 + i) / 2] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
}

/* INT4 W4A16 asymmetric, group 128 along K (lib_quant.py:159-167): scale = max(max - min, 1e-6) / 15,
 * q = clamp(rint((w - min) / scale), 0, 15), zero = min + 8 * scale, all in fp32; the kernel reads scale and zero
 * rounded to bf16 (lib_quant.py:209, :227), stored as two [N, K/128] arrays. Packing as the symmetric format. */
void orc_quantize_int4_asym(const float* W, int N, int K, uint8_t* packed, uint16_t* scale_bf16, uint16_t* zero_bf16) {
    const int G = K / 128;
    for (int n = 0; n < N; ++n) {
        for (int g = 0; g < G; ++g) {
            const float* w = W + (size_t)n * K + (size_t)g * 128;
            float mn = w[0], mx = w[0];
            for (int i = 1; i < 128; ++i) { if (w[i] < mn) mn = w[i]; if (w[i] > mx) mx = w[i]; }
            float d = mx - mn;
            if (d < 1e-6f) d = 1e-6f;
            const float s = d / 15.f;
            const float z = mn + 8.f * s;
            scale_bf16[(size_t)n * G + g] = orc_f32_to_bf16(s);
            zero_bf16[(size_t)n * G + g] = orc_f32_to_bf16(z);
            for (int i = 0; i < 128; i += 2) {
                int q0 = (int)nearbyintf((w[i] - mn) / s), q1 = (int)nearbyintf((w[i + 1] - mn) / s);
                q0 = q0 < 0 ? 0 : q0 > 15 ? 15 : q0;
                q1 = q1 < 0 ? 0 : q1 > 15 ? 15 : q1;
                packed[(size_t)n * (K / 2) + (size_t)(g * 128 + i) / 2] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
}

/* ---------------------------------------------------------------- dequantisers (one weight, fp32) */

static inline int nib(const uint8_t* packed, int K, int n, int k) {
    const uint8_t b = packed[(size_t)n * (K / 2) + k / 2];
    return (k & 1) ? (b >> 4) : (b & 0xF);
}
/* quant_host.h:83-85 / quant.py:16-17: e4m3(q) * scale in fp32. */
float orc_dequant_fp8(const uint8_t* q, const float* scale, int K, int n, int k) {
    return orc_e4m3_decode(q[(size_t)n * K + k]) * scale[n];
}
/* quant_host.h:107-111 / quant.py:34-38: (nibble - 8) * fp16 scale (exact in fp32). */
float orc_dequant_int4(const uint8_t* packed, const uint16_t* scales, int K, int n, int k) {
    return (float)(nib(packed, K, n, k) - 8) * orc_f16_to_f32(scales[(size_t)n * (K / 128) + k / 128]);
}
/* lib_quant.py:227-231: (q - 8) * bf16(scale) + bf16(zero) in fp32. */
float orc_dequant_int4_asym(const uint8_t* packed, const uint16_t* s, const uint16_t* z, int K, int n, int k) {
    const size_t gi = (size_t)n * (K / 128) + k / 128;
    const float p = (float)(nib(packed, K, n, k) - 8) * orc_bf16_to_f32(s[gi]);
    return p + orc_bf16_to_f32(z[gi]);
}

/* ---------------------------------------------------------------- GEMV oracles
 * Rows [r0, r1) of y = dequant(W) @ x (+ bias). yd (may be NULL) receives the fp64 sums, yb (may be NULL) the bf16
 * bits; both are indexed by the absolute row. bias (may be NULL) is bf16 bits [N]. x is bf16 bits [K]. */

static void finish(double acc, const uint16_t* bias, int n, double* yd, uint16_t* yb) {
    if (bias) acc += (double)orc_bf16_to_f32(bias[n]);
    if (yd) yd[n] = acc;
    if (yb) yb[n] = orc_f64_to_bf16(acc);
}

void orc_gemv_bf16(const uint16_t* W, const uint16_t* x, const uint16_t* bias, int N, int K, int r0, int r1,
                   double* yd, uint16_t* yb) {
    (void)N;
    for (int n = r0; n < r1; ++n) {
        double acc = 0.0;
        const uint16_t* w = W + (size_t)n * K;
        for (int k = 0; k < K; ++k) acc += (double)orc_bf16_to_f32(w[k]) * (double)orc_bf16_to_f32(x[k]);
        finish(acc, bias, n, yd, yb);
    }
}

void orc_gemv_fp8(const uint8_t* q, const float* scale, const uint16_t* x, const uint16_t* bias, int N, int K,
                  int r0, int r1, double* yd, uint16_t* yb) {
    (void)N;
    for (int n = r0; n < r1; ++n) {
        double acc = 0.0;
        for (int k = 0; k < K; ++k) acc += (double)orc_dequant_fp8(q, scale, K, n, k) * (double)orc_bf16_to_f32(x[k]);
        finish(acc, bias, n, yd, yb);
    }
}

void orc_gemv_int4(const uint8_t* packed, const uint16_t* scales, const uint16_t* x, const uint16_t* bias, int N,
                   int K, int r0, int r1, double* yd, uint16_t* yb) {
    (void)N;
    for (int n = r0; n < r1; ++n) {
        double acc = 0.0;
        for (int k = 0; k < K; ++k)
            acc += (double)orc_dequant_int4(packed, scales, K, n, k) * (double)orc_bf16_to_f32(x[k]);
        finish(acc, bias, n, yd, yb);
    }
}

void orc_gemv_int4_asym(const uint8_t* packed, const uint16_t* s, const uint16_t* z, const uint16_t* x,
                        const uint16_t* bias, int N, int K, int r0, int r1, double* yd, uint16_t* yb) {
    (void)N;
    for (int n = r0; n < r1; ++n) {
        double acc = 0.0;
        for (int k = 0; k < K; ++k)
            acc += (double)orc_dequant_int4_asym(packed, s, z, K, n, k) * (double)orc_bf16_to_f32(x[k]);
        finish(acc, bias, n, yd, yb);
    }
}

/* Dequantise to bf16 (the unfused control's stage 1, gemv_int4.cuh:154-174: bf16 RNE of (nibble - 8) * scale). */
void orc_dequant_int4_to_bf16(const uint8_t* packed, const uint16_t* scales, int N, int K, uint16_t* out) {
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k)
            out[(size_t)n * K + k] = orc_f32_to_bf16(orc_dequant_int4(packed, scales, K, n, k));
}

/* ---------------------------------------------------------------- batch helpers for the Python wrapper */
void orc_e4m3_encode_n(const float* x, uint8_t* out, size_t n) { for (size_t i = 0; i < n; ++i) out[i] = orc_e4m3_encode(x[i]); }
void orc_e4m3_decode_n(const uint8_t* b, float* out, size_t n) { for (size_t i = 0; i < n; ++i) out[i] = orc_e4m3_decode(b[i]); }
void orc_f32_to_f16_n(const float* x, uint16_t* out, size_t n) { for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(x[i]); }
void orc_f16_to_f32_n(const uint16_t* h, float* out, size_t n) { for (size_t i = 0; i < n; ++i) out[i] = orc_f16_to_f32(h[i]); }
void orc_f32_to_bf16_n(const float* x, uint16_t* out, size_t n) { for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(x[i]); }
void orc_f64_to_bf16_n(const double* x, uint16_t* out, size_t n) { for (size_t i = 0; i < n; ++i) out[i] = orc_f64_to_bf16(x[i]); }
