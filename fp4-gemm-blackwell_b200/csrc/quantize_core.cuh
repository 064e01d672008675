// quantize_core.cuh -- device code of the BF16 -> NVFP4 quantizer shared by
// the standalone quantize kernel (quantize.cu) and the GEMM kernel that
// quantizes its activations itself (gemm_sm100.cu).  The arithmetic is
// described in quantize.cu.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "nvfp4_codec.cuh"

namespace fp4b {
namespace qcore {


// |x|max (bf16 bits) below 6 * 2^-9 gives absmax/6 < 2^-9: the scale clamps to 0x01.
constexpr uint32_t kScaleClampBf16 = 0x3C40u;
constexpr int kScaleTableSize = (int)(kFastAbsmaxBf16Limit - kScaleClampBf16);  // 4672

struct QuantTables {
    uint8_t sbyte[kScaleTableSize];  // scale byte for |x|max bits kScaleClampBf16 + i
    float rcp[128];                  // RN(1 / ue4m3_decode(byte))
};
static_assert(kScaleTableSize % 16 == 0, "tables are copied in 16-byte pieces");

struct QuantParams {
    const uint16_t* src;
    uint8_t* fp4;
    uint8_t* sf;
    uint32_t rows, cols, ld;
    uint32_t nsb;      // 16-element blocks per padded row
    uint32_t total;    // rows_pad * nsb
    uint32_t div_mul;  // fast division by nsb: q = (umulhi(n, div_mul) + n) >> div_shift
    uint32_t div_shift;
    uint32_t vec_ok;   // 16-byte aligned rows
    // Stored blocks of a row (cols / 16 when cols % 16 == 0) with fast division,
    // for the staged kernel, whose spans walk the rows' stored blocks.
    uint32_t cpb, cpb_mul, cpb_shift;
};

// Shared-memory copies of the tables (copy_tables fills them).
struct SmemTables {
    const uint8_t* sbyte;
    const float* rcp;
};

// Bytes of shared memory copy_tables needs (16-byte aligned start).
constexpr int kSmemTableBytes = kScaleTableSize + 128 * 4;

// Threads [0, nthreads) of the caller copy the tables from global memory into
// `smem` (kSmemTableBytes, 16-byte aligned); the caller synchronizes after.
__device__ __forceinline__ SmemTables copy_tables(const QuantTables* g, uint8_t* smem, int tid, int nthreads) {
    const uint4* src = reinterpret_cast<const uint4*>(g);
    uint4* dst = reinterpret_cast<uint4*>(smem);
    static_assert(sizeof(QuantTables) == kSmemTableBytes, "table layout");
    for (int i = tid; i < kSmemTableBytes / 16; i += nthreads) dst[i] = __ldg(src + i);
    return SmemTables{smem, reinterpret_cast<const float*>(smem + kScaleTableSize)};
}

// Round-up multiplier for exact unsigned division of n < 2^31 by d >= 1.
inline void make_fast_div(uint32_t d, uint32_t* mul, uint32_t* shift) {
    uint32_t s = 0;
    while ((1ull << s) < d) ++s;
    *shift = s;
    *mul = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
}

// E2M1 rounding.  The reference scans {0, .5, 1, 1.5, 2, 3, 4, 6} for the
// nearest value with a strict <, so a tie keeps the lower magnitude, and sets
// the sign for any v < 0 (fp4_gemm_lib.cu:110-124).  The hardware conversion
// (cvt.rn.satfinite.e2m1x2.f32) rounds to nearest even, which differs only on
// ties (0.75, 1.75 and 3.5 go up) and on -0.  So it is applied to a stand-in
// for v = RN(x * inv) that is never a tie and rounds like v under the
// reference's rule:
//   * v' = RN(x * inv + 2^-149), two elements per fma.rn.f32x2.  For the
//     fast path's inputs this has the reference's code: a zero becomes 2^-149
//     (code 0, as the reference gives for +0 and -0); every non-zero product
//     has |x * inv| >= 2^-142, keeps its sign and, when it is not exactly
//     halfway between two floats, rounds to v; the products that are exactly
//     halfway (23,720 of all BF16 x and scale reciprocals) move by one ulp
//     without changing the nearest E2M1 value (checked exhaustively in
//     tests/test_fast_path_model.py);
//   * with b the bits of v' (never 0), (b - 1) | 1 is b itself when b is odd
//     (not a tie: ties have at least 21 trailing zero bits) and otherwise the
//     float one ulp closer to zero, which has the same nearest value as v'
//     unless v' is a tie, where it has the lower one; the sign is unchanged.
constexpr unsigned long long kTinyPair = 0x0000000100000001ull;  // (2^-149, 2^-149)

__device__ __forceinline__ unsigned long long scaled_pair(uint32_t w, unsigned long long inv2) {
    // w holds two BF16 values, the even element in the low half.
    const unsigned long long x2 = ((unsigned long long)(w & 0xFFFF0000u) << 32) | (unsigned long long)(w << 16);
    unsigned long long v2;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(v2) : "l"(x2), "l"(inv2), "l"(kTinyPair));
    return v2;
}

__device__ __forceinline__ float stand_in_bits(uint32_t b) { return __uint_as_float((b - 1u) | 1u); }

// Eight elements (four packed BF16 pairs, low element first) -> one word of
// eight E2M1 codes, element 2i in the low nibble of byte i.
__device__ __forceinline__ uint32_t pack8_e2m1(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, float inv) {
    const unsigned long long inv2 =
        ((unsigned long long)__float_as_uint(inv) << 32) | (unsigned long long)__float_as_uint(inv);
    const unsigned long long v0 = scaled_pair(w0, inv2), v1 = scaled_pair(w1, inv2);
    const unsigned long long v2 = scaled_pair(w2, inv2), v3 = scaled_pair(w3, inv2);
    uint32_t out;
    asm("{\n"
        ".reg .b8 b0, b1, b2, b3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
        "mov.b32 %0, {b0, b1, b2, b3};\n"
        "}"
        : "=r"(out)
        : "f"(stand_in_bits((uint32_t)v0)), "f"(stand_in_bits((uint32_t)(v0 >> 32))),
          "f"(stand_in_bits((uint32_t)v1)), "f"(stand_in_bits((uint32_t)(v1 >> 32))),
          "f"(stand_in_bits((uint32_t)v2)), "f"(stand_in_bits((uint32_t)(v2 >> 32))),
          "f"(stand_in_bits((uint32_t)v3)), "f"(stand_in_bits((uint32_t)(v3 >> 32))));
    return out;
}

// Element load with zero padding outside [rows, cols).
__device__ __forceinline__ uint32_t load_pair(const uint16_t* src, uint32_t ld, uint32_t rows, uint32_t cols,
                                              uint32_t r, uint32_t c) {
    uint32_t lo = 0, hi = 0;
    if (r < rows) {
        const uint16_t* row = src + (size_t)r * ld;
        if (c < cols) lo = row[c];
        if (c + 1 < cols) hi = row[c + 1];
    }
    return lo | (hi << 16);
}

struct BlockOut {
    uint32_t sbyte, out0, out1;
};

// Literal path for blocks holding NaN, Inf or |x| >= 2^30 (fp4_gemm_lib.cu:257-285).
// Rare, so it reloads its 16 elements instead of keeping them live, and
// returns its result by value (no stack traffic on the fast path).
static __device__ __noinline__ BlockOut quantize_block_exact(const uint16_t* src, uint32_t ld, uint32_t rows,
                                                      uint32_t cols, uint32_t r, uint32_t c0) {
    float amax = 0.0f;
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = load_pair(src, ld, rows, cols, r, c0 + 2 * i);
        amax = fmaxf(amax, fabsf(__uint_as_float(w << 16)));
        amax = fmaxf(amax, fabsf(__uint_as_float(w & 0xFFFF0000u)));
    }
    float s = __fdiv_rn(amax, 6.0f);
    if (s < kScaleMin) s = kScaleMin;
    const uint8_t b = ue4m3_encode(s);
    const float inv = __fdiv_rn(1.0f, ue4m3_decode(b));
    uint32_t o0 = 0u, o1 = 0u;
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = load_pair(src, ld, rows, cols, r, c0 + 2 * i);
        const uint32_t lo = e2m1_scan(__fmul_rn(__uint_as_float(w << 16), inv));
        const uint32_t hi = e2m1_scan(__fmul_rn(__uint_as_float(w & 0xFFFF0000u), inv));
        const uint32_t byte = (lo | (hi << 4)) << (8 * (i & 3));
        if (i < 4) o0 |= byte; else o1 |= byte;
    }
    return BlockOut{b, o0, o1};
}

// Per half: max(|a|, |b|) as bf16 (a NaN operand gives NaN); the sign bit of
// the result is not used.
__device__ __forceinline__ uint32_t max_abs_bf16x2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

constexpr int kThreads = 256;

// Scale byte of a block from its |x|max (bf16 bits < kFastAbsmaxBf16Limit);
// below 6 * 2^-9 the reference clamps the scale to 2^-9 (byte 0x01).
__device__ __forceinline__ uint32_t scale_byte(uint32_t amax_bits, const uint8_t* s_sbyte) {
    return amax_bits < kScaleClampBf16 ? 0x01u : (uint32_t)s_sbyte[amax_bits - kScaleClampBf16];
}

__device__ __forceinline__ void load_block(const QuantParams& p, uint32_t idx, uint32_t end, uint32_t (&w)[8],
                                           uint32_t& r, uint32_t& kb) {
    const bool valid = idx < end;
    r = (__umulhi(idx, p.div_mul) + idx) >> p.div_shift;
    kb = idx - r * p.nsb;
    const uint32_t c0 = kb * kSfVec;
    if (valid && p.vec_ok && r < p.rows && c0 + kSfVec <= p.cols) {
        const uint4* g = reinterpret_cast<const uint4*>(p.src + (size_t)r * p.ld + c0);
        const uint4 v0 = __ldcs(g);
        const uint4 v1 = __ldcs(g + 1);
        w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
        w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
    } else {
        // Ragged edge, padding rows/columns or unaligned rows: element loads, zeros outside.
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = valid ? load_pair(p.src, p.ld, p.rows, p.cols, r, c0 + 2 * i) : 0u;
    }
}

__device__ __forceinline__ void quantize_and_store(const QuantParams& p, uint32_t idx, uint32_t end,
                                                   const uint32_t (&w)[8],
                                                   uint32_t r, uint32_t kb, uint32_t lane, const SmemTables& tab) {
    const uint32_t m01 = max_abs_bf16x2(w[0], w[1]), m23 = max_abs_bf16x2(w[2], w[3]);
    const uint32_t m45 = max_abs_bf16x2(w[4], w[5]), m67 = max_abs_bf16x2(w[6], w[7]);
    const uint32_t mx = max_abs_bf16x2(max_abs_bf16x2(m01, m23), max_abs_bf16x2(m45, m67));
    const uint32_t amax_bits = max(mx & 0x7FFFu, (mx >> 16) & 0x7FFFu);

    uint32_t sbyte, out0, out1;
    if (amax_bits < kFastAbsmaxBf16Limit) {
        sbyte = scale_byte(amax_bits, tab.sbyte);
        const float inv = tab.rcp[sbyte];
        out0 = pack8_e2m1(w[0], w[1], w[2], w[3], inv);
        out1 = pack8_e2m1(w[4], w[5], w[6], w[7], inv);
    } else {
        const BlockOut o = quantize_block_exact(p.src, p.ld, p.rows, p.cols, r, kb * kSfVec);
        sbyte = o.sbyte;
        out0 = o.out0;
        out1 = o.out1;
    }
    const bool valid = idx < end;
    if (valid) *reinterpret_cast<uint2*>(p.fp4 + (size_t)idx * 8) = make_uint2(out0, out1);

    // Scales of 4 consecutive blocks of one row are 4 consecutive bytes.
    uint32_t sw = sbyte << (8 * (lane & 3u));
    sw |= __shfl_xor_sync(0xffffffffu, sw, 1);
    sw |= __shfl_xor_sync(0xffffffffu, sw, 2);
    if (valid && (lane & 3u) == 0) *reinterpret_cast<uint32_t*>(p.sf + sf_offset(r, kb, p.nsb)) = sw;
}


}  // namespace qcore

// Device address of the quantizer tables on the current device, uploaded on
// first use (defined in quantize.cu).
const qcore::QuantTables* quant_tables_device();

struct QuantizeArgs;
// Kernel parameters of a checked quantize call (defined in quantize.cu).
qcore::QuantParams make_quant_params(const QuantizeArgs& a);

}  // namespace fp4b
