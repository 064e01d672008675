// quantize.cu -- BF16 -> NVFP4 (E2M1 + UE4M3 per 16 elements) for sm_100a.
//
// Replaces quantize_bf16_to_fp4_kernel (fp4_gemm_lib.cu:241-286) with the
// same bytes out:
//   * one thread per 16-element block, flattened (row, block) index so a warp
//     reads 1 KB of contiguous BF16 with two 16-byte loads per thread;
//   * |x|max by bf16x2 max of magnitudes with NaN propagation (a NaN or Inf
//     sends the block to the literal path); the scale byte
//     ue4m3(max(|x|max / 6, 2^-9)) from a table over the fast-path |x|max
//     bit patterns, built on the host with IEEE division; reciprocal table;
//   * E2M1 rounding by a 2048-entry shared-memory table indexed by the fp32
//     bit slot of 32*x*inv (e2m1_banked_index), which reproduces the
//     reference's strict-< nearest-value scan (ties to the lower code, sign
//     for any value < 0) for every |x*inv| < 2^23 with the lookups of a warp
//     on distinct banks; blocks that could leave that range (|x|max >= 2^30,
//     Inf, NaN) take a literal scan instead;
//   * packed codes written as one 8-byte store per thread, scales gathered
//     over 4 lanes into one 4-byte store into the 128x4 interleaved layout.
// HBM-bound: 2 + 0.5 + 1/16 bytes per element.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"
#include "ptx_sm100.cuh"

namespace fp4b {

namespace {

// |x|max (bf16 bits) below 6 * 2^-9 gives absmax/6 < 2^-9: the scale clamps to 0x01.
constexpr uint32_t kScaleClampBf16 = 0x3C40u;
constexpr int kScaleTableSize = (int)(kFastAbsmaxBf16Limit - kScaleClampBf16);  // 4672

struct QuantTables {
    uint8_t e2m1[kE2M1TableSize];    // code by bank-spread fp32 bit slot of 32v (e2m1_banked_entry)
    uint8_t sbyte[kScaleTableSize];  // scale byte for |x|max bits kScaleClampBf16 + i
    float rcp32[128];                // 32 * RN(1 / ue4m3_decode(byte)) (exact power-of-two factor)
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
        for (uint32_t i = 0; i < (uint32_t)kE2M1TableSize; ++i) q.e2m1[i] = e2m1_banked_entry(i);
        for (int i = 0; i < kScaleTableSize; ++i) {
            // The reference: scale = absmax / 6 in fp32, clamped to [2^-9, 480], UE4M3.
            const float amax = bits_f32((kScaleClampBf16 + (uint32_t)i) << 16);
            q.sbyte[i] = ue4m3_encode(amax / 6.0f);
        }
        for (int b = 0; b < 128; ++b) q.rcp32[b] = 32.0f * (1.0f / ue4m3_decode((uint8_t)b));
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

// inv32 = 32 * RN(1 / scale): RN(x * inv32) = 32 * RN(x * RN(1 / scale)) whenever
// the latter is a normal float; when it is not, |v| < 2^-126 and both give
// code 0 with the same sign (no BF16 x underflows to zero here).
__device__ __forceinline__ uint32_t e2m1_fast(float x, float inv32, const uint8_t* tab) {
    return tab[e2m1_banked_index(__float_as_uint(__fmul_rn(x, inv32)))];
}

// Two packed BF16 -> byte of two E2M1 codes (low element in the low nibble).
__device__ __forceinline__ uint32_t pack_pair_fast(uint32_t w, float inv32, const uint8_t* tab) {
    const uint32_t lo = e2m1_fast(__uint_as_float(w << 16), inv32, tab);
    const uint32_t hi = e2m1_fast(__uint_as_float(w & 0xFFFF0000u), inv32, tab);
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

struct BlockOut {
    uint32_t sbyte, out0, out1;
};

// Literal path for blocks holding NaN, Inf or |x| >= 2^30 (fp4_gemm_lib.cu:257-285).
// Rare, so it reloads its 16 elements instead of keeping them live, and
// returns its result by value (no stack traffic on the fast path).
__device__ __noinline__ BlockOut quantize_block_exact(const uint16_t* src, uint32_t ld, uint32_t rows,
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
constexpr int kBlocksPerThread = 2;  // 16-element blocks per thread per loop trip

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
                                                   uint32_t r, uint32_t kb, uint32_t lane, const uint8_t* s_e2m1,
                                                   const uint8_t* s_sbyte, const float* s_rcp32) {
    const uint32_t m01 = max_abs_bf16x2(w[0], w[1]), m23 = max_abs_bf16x2(w[2], w[3]);
    const uint32_t m45 = max_abs_bf16x2(w[4], w[5]), m67 = max_abs_bf16x2(w[6], w[7]);
    const uint32_t mx = max_abs_bf16x2(max_abs_bf16x2(m01, m23), max_abs_bf16x2(m45, m67));
    const uint32_t amax_bits = max(mx & 0x7FFFu, (mx >> 16) & 0x7FFFu);

    uint32_t sbyte, out0 = 0, out1 = 0;
    if (amax_bits < kFastAbsmaxBf16Limit) {
        sbyte = scale_byte(amax_bits, s_sbyte);
        const float inv32 = s_rcp32[sbyte];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out0 |= pack_pair_fast(w[i], inv32, s_e2m1) << (8 * i);
            out1 |= pack_pair_fast(w[i + 4], inv32, s_e2m1) << (8 * i);
        }
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

// Grid-stride over spans of 512 blocks (one thread per block, two blocks per
// thread per span), so the CTAs running at one time read neighbouring memory.
// The first loads go out before the tables are copied to shared memory, so
// their latencies overlap.
__global__ void __launch_bounds__(kThreads) nvfp4_quantize_kernel(const __grid_constant__ QuantParams p) {
    __shared__ __align__(16) uint8_t s_e2m1[kE2M1TableSize];
    __shared__ __align__(16) uint8_t s_sbyte[kScaleTableSize];
    __shared__ float s_rcp32[128];

    constexpr uint32_t kSpan = kThreads * kBlocksPerThread;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t end = p.total;
    const uint32_t stride = gridDim.x * kSpan;
    uint32_t base = blockIdx.x * kSpan;
    uint32_t w0[8], w1[8], r0, kb0, r1, kb1;
    load_block(p, base + threadIdx.x, end, w0, r0, kb0);
    load_block(p, base + threadIdx.x + kThreads, end, w1, r1, kb1);
    {
        const uint4* src = reinterpret_cast<const uint4*>(g_qtab.e2m1);
        uint4* dst = reinterpret_cast<uint4*>(s_e2m1);
        for (int i = threadIdx.x; i < kE2M1TableSize / 16; i += kThreads) dst[i] = __ldg(src + i);
        const uint4* srcs = reinterpret_cast<const uint4*>(g_qtab.sbyte);
        uint4* dsts = reinterpret_cast<uint4*>(s_sbyte);
        for (int i = threadIdx.x; i < kScaleTableSize / 16; i += kThreads) dsts[i] = __ldg(srcs + i);
        if (threadIdx.x < 128) s_rcp32[threadIdx.x] = __ldg(&g_qtab.rcp32[threadIdx.x]);
    }
    __syncthreads();
    // A GEMM launched behind this kernel may start setting up (it waits for
    // this grid to complete before reading the quantized activations).
    ptx::launch_dependents();

    for (;;) {
        quantize_and_store(p, base + threadIdx.x, end, w0, r0, kb0, lane, s_e2m1, s_sbyte, s_rcp32);
        quantize_and_store(p, base + threadIdx.x + kThreads, end, w1, r1, kb1, lane, s_e2m1, s_sbyte, s_rcp32);
        base += stride;
        if (base >= end) break;
        load_block(p, base + threadIdx.x, end, w0, r0, kb0);
        load_block(p, base + threadIdx.x + kThreads, end, w1, r1, kb1);
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
    // Up to FP4B_QUANT_CTAS_PER_SM (default 16) CTAs per SM, grid-stride beyond.
    static int per_sm = [] {
        const char* e = getenv("FP4B_QUANT_CTAS_PER_SM");
        const int v = e ? atoi(e) : 16;
        return v > 0 ? v : 16;
    }();
    const uint32_t span = kThreads * kBlocksPerThread;
    const uint64_t need = (p.total + span - 1) / span;
    const uint64_t cap = (uint64_t)sms * (uint64_t)per_sm;
    const uint64_t grid = need < cap ? need : cap;
    nvfp4_quantize_kernel<<<(uint32_t)grid, kThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace fp4b
