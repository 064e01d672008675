/*
 * nvfp4_oracle.c -- CPU restatement of the reference NVFP4 quantizer.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels
 * in the fp4-gemm-blackwell_b200 package; the product never links, loads or
 * calls it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may use it.
 *
 * Every function restates one piece of VincentKaufmann/fp4-gemm-blackwell,
 * file fp4_gemm_lib.cu, in plain C with IEEE fp32 arithmetic:
 *
 *   oracle_e2m1_code      fp4_gemm_lib.cu:107-124  (d_float_to_fp4)
 *   oracle_ue4m3_encode   fp4_gemm_lib.cu:128-164  (d_float_to_ue4m3)
 *   oracle_ue4m3_decode   fp4_gemm_lib.cu:167-177  (d_ue4m3_to_float)
 *   oracle_sf_index       fp4_gemm_lib.cu:198-237  (compute_sf_index)
 *   oracle_quantize       fp4_gemm_lib.cu:241-286  (quantize_bf16_to_fp4_kernel)
 *                         plus the zero padding of fp4_gemm.py:296-309, 350-362
 *   oracle_dequantize     the inverse map used by the GEMM tolerance oracle
 *
 * Parity is pinned: tests/test_oracle.py checks these functions against the
 * golden vectors in tests/golden/, which tests/golden/make_golden.py produced
 * by running the reference's own quantizer source (compiled for the host by
 * build_ref() in oracle/build.py into oracle/_ref/).
 *
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fno-fast-math -fopenmp -fPIC -shared
 * (build_oracle() in oracle/build.py).  Contraction must stay off so that every product
 * and difference is rounded exactly as the device code rounds it.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define SF_VEC 16

/* E2M1 magnitudes in code order (fp4_gemm_lib.cu:107). */
static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* Nearest E2M1 code by a linear scan that only moves on a strictly smaller
 * distance, so ties keep the lower code; the sign nibble is set for any
 * value < 0 (fp4_gemm_lib.cu:110-124).  NaN and +-Inf give magnitude code 0. */
uint8_t oracle_e2m1_code(float v) {
    float a = fabsf(v);
    uint8_t sign = (v < 0.0f) ? 0x8 : 0x0;
    uint8_t code = 0;
    float best = a;
    for (int i = 1; i < 8; ++i) {
        float d = fabsf(a - kE2M1[i]);
        if (d < best) {
            best = d;
            code = (uint8_t)i;
        }
    }
    return (uint8_t)(sign | code);
}

/* UE4M3 encode (fp4_gemm_lib.cu:128-164): clamp to [2^-9, 480]; exponent
 * rebiased by +7; subnormal mantissa truncated; normal mantissa rounded half
 * up with carry into the exponent; exponents >= 15 before rounding give 0x7F. */
uint8_t oracle_ue4m3_encode(float val) {
    val = fmaxf(val, 1.953125e-3f);
    val = fminf(val, 480.0f);
    uint32_t u = f32_bits(val);
    int e = (int)((u >> 23) & 0xFF) - 127;
    int m = (int)(u & 0x7FFFFF);
    int ue = e + 7;
    if (ue <= 0) {
        int shift = 1 - ue;
        int mant = (0x800000 | m) >> (20 + shift);
        if (mant > 7) mant = 7;
        return (uint8_t)mant;
    }
    if (ue >= 15) return 0x7F;
    int mant = (m + (1 << 19)) >> 20;
    if (mant >= 8) {
        mant = 0;
        ue += 1;
        if (ue >= 16) return 0xFF;
    }
    return (uint8_t)((ue << 3) | mant);
}

/* UE4M3 decode (fp4_gemm_lib.cu:167-177). */
float oracle_ue4m3_decode(uint8_t raw) {
    int e = (raw >> 3) & 0xF;
    int m = raw & 0x7;
    if (e == 0) return ldexpf((float)m, -9);
    return ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

/* Byte offset of scale (row r, 16-element block kb) in the 128x4 interleaved
 * scale layout (fp4_gemm_lib.cu:198-237).  nsb = K / 16. */
long oracle_sf_index(long r, long kb, long nsb) {
    long r0 = r % 32, r1 = (r / 32) % 4, r2 = r / 128;
    long k1 = kb % 4, k2 = kb / 4;
    return r0 * 16 + r1 * 4 + r2 * 512 * (nsb / 4) + k1 + k2 * 512;
}

/* One 16-element block (fp4_gemm_lib.cu:257-285): absmax -> absmax/6 ->
 * clamp -> UE4M3 -> 1/decode -> per-element nearest E2M1, even element in the
 * low nibble. */
static void quantize_block(const float* x, uint8_t* fp4_out, uint8_t* sf_out) {
    float amax = 0.0f;
    for (int i = 0; i < SF_VEC; ++i) amax = fmaxf(amax, fabsf(x[i]));
    float s = amax / 6.0f;
    if (s < 1.953125e-3f) s = 1.953125e-3f;
    uint8_t sraw = oracle_ue4m3_encode(s);
    float inv = 1.0f / oracle_ue4m3_decode(sraw);
    *sf_out = sraw;
    for (int i = 0; i < SF_VEC; i += 2) {
        uint8_t lo = oracle_e2m1_code(x[i] * inv);
        uint8_t hi = oracle_e2m1_code(x[i + 1] * inv);
        fp4_out[i / 2] = (uint8_t)((hi << 4) | lo);
    }
}

/* Quantize a BF16 matrix [rows, cols] (row stride ld elements) into the packed
 * FP4 buffer [rows_pad, k_pad/2] and the interleaved scale buffer
 * (rows_pad * k_pad / 16 bytes).  Elements outside [rows, cols) read as zero,
 * which is exactly the reference's torch.zeros padding to multiples of 128
 * (fp4_gemm.py:146-160, 296-309, 350-362).  rows_pad and k_pad must be
 * multiples of 128.  Returns 0, or -1 on a bad shape. */
int oracle_quantize(const uint16_t* src, long rows, long cols, long ld,
                    long rows_pad, long k_pad, uint8_t* fp4, uint8_t* sf) {
    if (rows_pad % 128 || k_pad % 128 || rows > rows_pad || cols > k_pad || ld < cols) return -1;
    long nsb = k_pad / SF_VEC;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows_pad; ++r) {
        float x[SF_VEC];
        for (long kb = 0; kb < nsb; ++kb) {
            for (int i = 0; i < SF_VEC; ++i) {
                long c = kb * SF_VEC + i;
                x[i] = (r < rows && c < cols) ? bf16_to_f32(src[r * ld + c]) : 0.0f;
            }
            quantize_block(x, fp4 + r * (k_pad / 2) + kb * 8, sf + oracle_sf_index(r, kb, nsb));
        }
    }
    return 0;
}

/* Dequantize packed FP4 + interleaved scales back to fp32 [rows, k_pad]:
 * value = sign * E2M1(code) * UE4M3(scale).  This is the operand the
 * reference GEMM multiplies (fp4_gemm_lib.cu:547-561). */
int oracle_dequantize(const uint8_t* fp4, const uint8_t* sf, long rows, long k_pad, float* out) {
    if (rows % 128 || k_pad % 128) return -1;
    long nsb = k_pad / SF_VEC;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        for (long kb = 0; kb < nsb; ++kb) {
            float s = oracle_ue4m3_decode(sf[oracle_sf_index(r, kb, nsb)]);
            for (int i = 0; i < SF_VEC; ++i) {
                long c = kb * SF_VEC + i;
                uint8_t byte = fp4[r * (k_pad / 2) + c / 2];
                uint8_t nib = (c & 1) ? (byte >> 4) : (byte & 0xF);
                float mag = kE2M1[nib & 7];
                out[r * k_pad + c] = ((nib & 8) ? -mag : mag) * s;
            }
        }
    }
    return 0;
}

/* Bits of the fp32 value x (exported so tests can check the host float model). */
uint32_t oracle_f32_bits(float x) { return f32_bits(x); }
