// nvfp4_codec.cuh -- NVFP4 element / scale codecs shared by host and device.
//
// Semantics follow the reference quantizer of VincentKaufmann/fp4-gemm-blackwell
// exactly (bytes must match), not IEEE round-to-nearest-even:
//   * E2M1: nearest of {0,.5,1,1.5,2,3,4,6} by a scan that only moves on a
//     strictly smaller fp32 distance -> ties keep the lower code; sign nibble
//     for any value < 0; NaN/Inf -> magnitude 0      (fp4_gemm_lib.cu:107-124)
//   * UE4M3: clamp [2^-9, 480], subnormal mantissa truncated, normal mantissa
//     rounded half up with carry, pre-rounding exponent >= 15 -> 0x7F
//                                                    (fp4_gemm_lib.cu:128-164)
//   * scale layout: 512-byte atoms of 128 rows x 4 blocks
//                                                    (fp4_gemm_lib.cu:198-237)
#pragma once
#include <cstdint>
#include <cstring>

#ifndef FP4B_HD
#define FP4B_HD __host__ __device__ __forceinline__
#endif

namespace fp4b {

constexpr int kSfVec = 16;                  // elements per scale factor
constexpr float kScaleMin = 1.953125e-3f;   // 2^-9, smallest UE4M3 subnormal
constexpr float kScaleMax = 480.0f;         // largest UE4M3 value
// Blocks whose |x|max (as bf16 bits) is below this (2^30) take the GPU
// quantizer's fast path, which reads the scale byte from a table over these
// bit patterns; larger, infinite and NaN blocks take the literal path.
constexpr uint32_t kFastAbsmaxBf16Limit = 0x4E80u;

FP4B_HD uint32_t f32_bits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
#endif
}

FP4B_HD float bits_f32(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    std::memcpy(&f, &u, 4);
    return f;
#endif
}

FP4B_HD float fmax_ieee(float a, float b) {  // fmaxf: a NaN operand yields the other
#ifdef __CUDA_ARCH__
    return fmaxf(a, b);
#else
    return (a != a) ? b : ((b != b) ? a : (a > b ? a : b));
#endif
}

FP4B_HD float fmin_ieee(float a, float b) {
#ifdef __CUDA_ARCH__
    return fminf(a, b);
#else
    return (a != a) ? b : ((b != b) ? a : (a < b ? a : b));
#endif
}

// Literal nearest-value scan; the exact definition the fast table is derived from.
FP4B_HD uint8_t e2m1_scan(float v) {
    const float vals[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    float a = bits_f32(f32_bits(v) & 0x7FFFFFFFu);
    uint8_t sign = (v < 0.0f) ? 0x8 : 0x0;
    uint8_t code = 0;
    float best = a;
#pragma unroll
    for (int i = 1; i < 8; ++i) {
        float d = bits_f32(f32_bits(a - vals[i]) & 0x7FFFFFFFu);
        if (d < best) {
            best = d;
            code = (uint8_t)i;
        }
    }
    return (uint8_t)(sign | code);
}

FP4B_HD uint8_t ue4m3_encode(float val) {
    val = fmax_ieee(val, kScaleMin);
    val = fmin_ieee(val, kScaleMax);
    const uint32_t u = f32_bits(val);
    const int e = (int)((u >> 23) & 0xFF) - 127;
    const int m = (int)(u & 0x7FFFFF);
    int ue = e + 7;
    if (ue <= 0) {
        int mant = (0x800000 | m) >> (20 + (1 - ue));
        return (uint8_t)(mant < 7 ? mant : 7);
    }
    if (ue >= 15) return 0x7F;
    int mant = (m + (1 << 19)) >> 20;
    if (mant >= 8) {
        mant = 0;
        ++ue;
        if (ue >= 16) return 0xFF;
    }
    return (uint8_t)((ue << 3) | mant);
}

// Exact UE4M3 value: m * 2^-9 (subnormal) or (8 + m) * 2^(e-10).
FP4B_HD float ue4m3_decode(uint8_t raw) {
    const uint32_t e = (raw >> 3) & 0xF, m = raw & 0x7;
    if (e == 0) return (float)m * 0.001953125f;
    return bits_f32(((e + 120u) << 23) | (m << 20));
}

// Byte offset of (row r, block kb) in the interleaved scale buffer; nsb = K/16.
FP4B_HD uint32_t sf_offset(uint32_t r, uint32_t kb, uint32_t nsb) {
    return (((r & 31u) << 4) | (((r >> 5) & 3u) << 2) | (kb & 3u)) + (((kb >> 2) + (r >> 7) * (nsb >> 2)) << 9);
}

}  // namespace fp4b
