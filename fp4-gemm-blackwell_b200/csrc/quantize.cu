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
#include "quantize_core.cuh"

namespace fp4b {

namespace {

using namespace qcore;

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

// Grid-stride over spans of 512 blocks (one thread per block, two blocks per
// thread per span), so the CTAs running at one time read neighbouring memory.
// The first loads go out before the tables are copied to shared memory, so
// their latencies overlap.
__global__ void __launch_bounds__(kThreads) nvfp4_quantize_kernel(const __grid_constant__ QuantParams p) {
    __shared__ __align__(16) uint8_t s_tables[kSmemTableBytes];

    constexpr uint32_t kSpan = kThreads * kBlocksPerThread;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t end = p.total;
    const uint32_t stride = gridDim.x * kSpan;
    uint32_t base = blockIdx.x * kSpan;
    uint32_t w0[8], w1[8], r0, kb0, r1, kb1;
    load_block(p, base + threadIdx.x, end, w0, r0, kb0);
    load_block(p, base + threadIdx.x + kThreads, end, w1, r1, kb1);
    const SmemTables tab = copy_tables(&g_qtab, s_tables, threadIdx.x, kThreads);
    __syncthreads();
    // A GEMM launched behind this kernel may start setting up (it waits for
    // this grid to complete before reading the quantized activations).
    ptx::launch_dependents();

    for (;;) {
        quantize_and_store(p, base + threadIdx.x, end, w0, r0, kb0, lane, tab);
        quantize_and_store(p, base + threadIdx.x + kThreads, end, w1, r1, kb1, lane, tab);
        base += stride;
        if (base >= end) break;
        load_block(p, base + threadIdx.x, end, w0, r0, kb0);
        load_block(p, base + threadIdx.x + kThreads, end, w1, r1, kb1);
    }
}

}  // namespace

const qcore::QuantTables* quant_tables_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_qtab_mu);
    if (!g_qtab_ready[dev & 63]) {
        // First use on this device: copy the tables (synchronous, not an allocation).
        if (cudaMemcpyToSymbol(g_qtab, &host_tables(), sizeof(qcore::QuantTables)) != cudaSuccess) return nullptr;
        g_qtab_ready[dev & 63] = true;
    }
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qtab) != cudaSuccess) return nullptr;
    return static_cast<const qcore::QuantTables*>(p);
}

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

qcore::QuantParams make_quant_params(const QuantizeArgs& a) {
    qcore::QuantParams p{};
    p.src = static_cast<const uint16_t*>(a.src);
    p.fp4 = a.fp4;
    p.sf = a.sf;
    p.rows = (uint32_t)a.rows;
    p.cols = (uint32_t)a.cols;
    p.ld = (uint32_t)a.ld;
    p.nsb = (uint32_t)(a.k_pad / kSfVec);
    p.total = (uint32_t)(a.rows_pad * p.nsb);
    qcore::make_fast_div(p.nsb, &p.div_mul, &p.div_shift);
    p.vec_ok = ((reinterpret_cast<uintptr_t>(a.src) & 15) == 0 && (a.ld % 8) == 0) ? 1u : 0u;
    return p;
}

cudaError_t quantize_launch(const QuantizeArgs& a, cudaStream_t stream) {
    const QuantParams p = make_quant_params(a);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (!quant_tables_device()) return cudaErrorInvalidValue;
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
