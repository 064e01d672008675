// quantize.cu -- BF16 -> NVFP4 (E2M1 + UE4M3 per 16 elements) for sm_100a.
//
// Replaces quantize_bf16_to_fp4_kernel (fp4_gemm_lib.cu:241-286) with the
// same bytes out:
//   * one thread per 16-element block, flattened (row, block) index so a warp
//     reads 1 KB of contiguous BF16 with two 16-byte loads per thread;
//   * |x|max as an integer max over the bf16 bit patterns (exact for finite
//     values); absmax/6 rounded to nearest from a 128-entry table of
//     RN((128 + m) / 6) scaled by the exponent (exact for normal results);
//     UE4M3 encode; reciprocal table;
//   * E2M1 rounding by a 2048-entry shared-memory table indexed by
//     (bits(x*inv) - 1) >> 21, which reproduces the reference's strict-<
//     nearest-value scan (ties to the lower code, sign for any value < 0)
//     for every |x*inv| < 2^23; blocks that could leave that range (|x|max >=
//     2^30, Inf, NaN) take a literal scan instead;
//   * packed codes written as one 8-byte store per thread, scales gathered
//     over 4 lanes into one 4-byte store into the 128x4 interleaved layout.
// HBM-bound: 2 + 0.5 + 1/16 bytes per element.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"

namespace fp4b {

namespace {

struct QuantTables {
    uint8_t e2m1[kE2M1TableSize];  // code by fp32 bit slot
    float rcp[128];                // 1 / ue4m3_decode(byte), IEEE round-to-nearest
    uint32_t div6[128];            // bits of RN((128 + m) / 6) for a bf16 mantissa m
};

// |x|max (bf16 bits) below 6 * 2^-9 gives absmax/6 < 2^-9: the scale clamps to 0x01.
constexpr uint32_t kScaleClampBf16 = 0x3C40u;

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
};

// Device copy of the tables, written once per device (host_tables() -> here).
// Read with coalesced loads at CTA start; passing them as kernel parameters
// instead cost several microseconds per CTA (divergent constant-bank reads).
__device__ QuantTables g_qtab;
std::mutex g_qtab_mu;
bool g_qtab_ready[64];

// Tables built on the host from the same codec definitions as the device code.
const QuantTables& host_tables() {
    static const QuantTables t = [] {
        QuantTables q{};
        for (uint32_t i = 0; i < (uint32_t)kE2M1TableSize; ++i) q.e2m1[i] = e2m1_table_entry(i);
        for (int b = 0; b < 128; ++b) q.rcp[b] = 1.0f / ue4m3_decode((uint8_t)b);
        for (int m = 0; m < 128; ++m) q.div6[m] = f32_bits((float)(128 + m) / 6.0f);
        return q;
    }();
    return t;
}

// Round-up multiplier for exact unsigned division of n < 2^31 by d >= 1.
void make_fast_div(uint32_t d, uint32_t* mul, uint32_t* shift) {
    uint32_t s = 0;
    while ((1ull << s) < d) ++s;
    *shift = s;
    *mul = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
}

__device__ __forceinline__ uint32_t e2m1_fast(float x, float inv, const uint8_t* tab) {
    const float v = __fmul_rn(x, inv);
    return tab[(__float_as_uint(v) - 1u) >> 21];
}

// Two packed BF16 -> byte of two E2M1 codes (low element in the low nibble).
__device__ __forceinline__ uint32_t pack_pair_fast(uint32_t w, float inv, const uint8_t* tab) {
    const uint32_t lo = e2m1_fast(__uint_as_float(w << 16), inv, tab);
    const uint32_t hi = e2m1_fast(__uint_as_float(w & 0xFFFF0000u), inv, tab);
    return lo | (hi << 4);
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

// Literal path for blocks holding NaN, Inf or |x| >= 2^30 (fp4_gemm_lib.cu:257-285).
// Rare, so it reloads its 16 elements instead of keeping them live.
__device__ __noinline__ void quantize_block_exact(const uint16_t* src, uint32_t ld, uint32_t rows, uint32_t cols,
                                                  uint32_t r, uint32_t c0, const float* rcp, uint32_t* sbyte,
                                                  uint32_t* out0, uint32_t* out1) {
    float amax = 0.0f;
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = load_pair(src, ld, rows, cols, r, c0 + 2 * i);
        amax = fmaxf(amax, fabsf(__uint_as_float(w << 16)));
        amax = fmaxf(amax, fabsf(__uint_as_float(w & 0xFFFF0000u)));
    }
    float s = __fdiv_rn(amax, 6.0f);
    if (s < kScaleMin) s = kScaleMin;
    const uint8_t b = ue4m3_encode(s);
    const float inv = rcp[b];
    uint32_t o0 = 0u, o1 = 0u;
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = load_pair(src, ld, rows, cols, r, c0 + 2 * i);
        const uint32_t lo = e2m1_scan(__fmul_rn(__uint_as_float(w << 16), inv));
        const uint32_t hi = e2m1_scan(__fmul_rn(__uint_as_float(w & 0xFFFF0000u), inv));
        const uint32_t byte = (lo | (hi << 4)) << (8 * (i & 3));
        if (i < 4) o0 |= byte; else o1 |= byte;
    }
    *sbyte = b;
    *out0 = o0;
    *out1 = o1;
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

constexpr int kThreads = 256;
constexpr int kBlocksPerThread = 2;  // 16-element blocks per thread per loop trip

// Scale byte of a block from its |x|max (bf16 bits < kFastAbsmaxBf16Limit):
// RN(absmax / 6) = RN((128 + m) / 6) * 2^(E - 134) exactly while the result is
// a normal fp32, which it is whenever absmax / 6 >= 2^-9; below that the
// reference clamps to 2^-9 (byte 0x01).
__device__ __forceinline__ uint32_t scale_byte(uint32_t amax_bits, const uint32_t* div6) {
    if (amax_bits < kScaleClampBf16) return 0x01u;
    const uint32_t s_bits = div6[amax_bits & 0x7Fu] + (((amax_bits >> 7) - 134u) << 23);
    return ue4m3_encode(__uint_as_float(s_bits));
}

__device__ __forceinline__ void load_block(const QuantParams& p, uint32_t idx, uint32_t (&w)[8], uint32_t& r,
                                           uint32_t& kb) {
    const bool valid = idx < p.total;
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

__device__ __forceinline__ void quantize_and_store(const QuantParams& p, uint32_t idx, const uint32_t (&w)[8],
                                                   uint32_t r, uint32_t kb, uint32_t lane, const uint8_t* s_e2m1,
                                                   const float* s_rcp, const uint32_t* s_div6) {
    uint32_t mx = w[0] & 0x7FFF7FFFu;
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = max_u16x2(mx, w[i] & 0x7FFF7FFFu);
    const uint32_t amax_bits = max(mx & 0xFFFFu, mx >> 16);

    uint32_t sbyte, out0 = 0, out1 = 0;
    if (amax_bits < kFastAbsmaxBf16Limit) {
        sbyte = scale_byte(amax_bits, s_div6);
        const float inv = s_rcp[sbyte];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out0 |= pack_pair_fast(w[i], inv, s_e2m1) << (8 * i);
            out1 |= pack_pair_fast(w[i + 4], inv, s_e2m1) << (8 * i);
        }
    } else {
        quantize_block_exact(p.src, p.ld, p.rows, p.cols, r, kb * kSfVec, s_rcp, &sbyte, &out0, &out1);
    }
    const bool valid = idx < p.total;
    if (valid) *reinterpret_cast<uint2*>(p.fp4 + (size_t)idx * 8) = make_uint2(out0, out1);

    // Scales of 4 consecutive blocks of one row are 4 consecutive bytes.
    uint32_t sw = sbyte << (8 * (lane & 3u));
    sw |= __shfl_xor_sync(0xffffffffu, sw, 1);
    sw |= __shfl_xor_sync(0xffffffffu, sw, 2);
    if (valid && (lane & 3u) == 0) *reinterpret_cast<uint32_t*>(p.sf + sf_offset(r, kb, p.nsb)) = sw;
}

__global__ void __launch_bounds__(kThreads) nvfp4_quantize_kernel(const __grid_constant__ QuantParams p) {
    __shared__ __align__(16) uint8_t s_e2m1[kE2M1TableSize];
    __shared__ float s_rcp[128];
    __shared__ uint32_t s_div6[128];
    {
        const uint4* src = reinterpret_cast<const uint4*>(g_qtab.e2m1);
        uint4* dst = reinterpret_cast<uint4*>(s_e2m1);
        for (int i = threadIdx.x; i < kE2M1TableSize / 16; i += kThreads) dst[i] = __ldg(src + i);
        if (threadIdx.x < 128) {
            s_rcp[threadIdx.x] = __ldg(&g_qtab.rcp[threadIdx.x]);
            s_div6[threadIdx.x] = __ldg(&g_qtab.div6[threadIdx.x]);
        }
    }
    __syncthreads();

    const uint32_t lane = threadIdx.x & 31u;
    constexpr uint32_t kSpan = kThreads * kBlocksPerThread;
    const uint32_t stride = gridDim.x * kSpan;
    for (uint32_t base = blockIdx.x * kSpan; base < p.total; base += stride) {
        // Both loads are issued before either block is processed.
        const uint32_t i0 = base + threadIdx.x, i1 = i0 + kThreads;
        uint32_t w0[8], w1[8], r0, kb0, r1, kb1;
        load_block(p, i0, w0, r0, kb0);
        load_block(p, i1, w1, r1, kb1);
        quantize_and_store(p, i0, w0, r0, kb0, lane, s_e2m1, s_rcp, s_div6);
        quantize_and_store(p, i1, w1, r1, kb1, lane, s_e2m1, s_rcp, s_div6);
    }
}

}  // namespace

const char* quantize_check(const QuantizeArgs& a) {
    if (!a.src || !a.fp4 || !a.sf) return "null pointer";
    if (a.rows < 0 || a.cols < 0) return "negative size";
    if (a.rows_pad <= 0 || a.k_pad <= 0 || a.rows_pad % 128 || a.k_pad % 128)
        return "padded rows and K must be positive multiples of 128";
    if (a.rows > a.rows_pad || a.cols > a.k_pad) return "matrix larger than its padded shape";
    if (a.ld < a.cols) return "row stride smaller than the row length";
    if ((reinterpret_cast<uintptr_t>(a.fp4) & 7) || (reinterpret_cast<uintptr_t>(a.sf) & 3))
        return "output buffers must be 8-byte (fp4) and 4-byte (scales) aligned";
    if (a.rows_pad * (a.k_pad / kSfVec) >= (1l << 31) || a.ld >= (1l << 31))
        return "matrix too large for one launch (rows*K/16 must stay below 2^31)";
    return nullptr;
}

cudaError_t quantize_launch(const QuantizeArgs& a, cudaStream_t stream) {
    QuantParams p{};
    p.src = static_cast<const uint16_t*>(a.src);
    p.fp4 = a.fp4;
    p.sf = a.sf;
    p.rows = (uint32_t)a.rows;
    p.cols = (uint32_t)a.cols;
    p.ld = (uint32_t)a.ld;
    p.nsb = (uint32_t)(a.k_pad / kSfVec);
    p.total = (uint32_t)(a.rows_pad * p.nsb);
    make_fast_div(p.nsb, &p.div_mul, &p.div_shift);
    p.vec_ok = ((reinterpret_cast<uintptr_t>(a.src) & 15) == 0 && (a.ld % 8) == 0) ? 1u : 0u;

    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    {
        // First use on this device: copy the tables (synchronous, not an allocation).
        std::lock_guard<std::mutex> lk(g_qtab_mu);
        if (!g_qtab_ready[dev & 63]) {
            const cudaError_t e = cudaMemcpyToSymbol(g_qtab, &host_tables(), sizeof(QuantTables));
            if (e != cudaSuccess) return e;
            g_qtab_ready[dev & 63] = true;
        }
    }
    const uint32_t span = kThreads * kBlocksPerThread;
    const uint32_t need = (p.total + span - 1) / span;
    const uint32_t cap = (uint32_t)sms * 8u;
    const uint32_t grid = need < cap ? need : cap;
    nvfp4_quantize_kernel<<<grid, kThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace fp4b
