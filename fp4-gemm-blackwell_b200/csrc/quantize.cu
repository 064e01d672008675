// quantize.cu -- BF16 -> NVFP4 (E2M1 + UE4M3 per 16 elements) for sm_100a.
//
// Replaces quantize_bf16_to_fp4_kernel (fp4_gemm_lib.cu:241-286) with the
// same bytes out:
//   * one thread per 16-element block, flattened (row, block) index so a warp
//     reads 1 KB of contiguous BF16 with two 16-byte loads per thread; a
//     persistent grid with the next block's loads in flight;
//   * |x|max by bf16x2 max of magnitudes with NaN propagation (a NaN or Inf
//     sends the block to the literal path); the scale byte
//     ue4m3(max(|x|max / 6, 2^-9)) from a table over the fast-path |x|max
//     bit patterns, built on the host with IEEE division; reciprocal table;
//   * E2M1 rounding by the hardware conversion (cvt.rn.satfinite.e2m1x2)
//     applied to a stand-in for each scaled value that is never a tie and
//     rounds to the reference's code (pack8_e2m1 in quantize_core.cuh), so
//     the reference's strict-< nearest-value scan (ties to the lower code,
//     sign for any value < 0) is reproduced bit for bit; blocks with
//     |x|max >= 2^30, Inf or NaN take a literal scan instead;
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
        for (int i = 0; i < kScaleTableSize; ++i) {
            // The reference: scale = absmax / 6 in fp32, clamped to [2^-9, 480], UE4M3.
            const float amax = bits_f32((kScaleClampBf16 + (uint32_t)i) << 16);
            q.sbyte[i] = ue4m3_encode(amax / 6.0f);
        }
        for (int b = 0; b < 128; ++b) q.rcp[b] = 1.0f / ue4m3_decode((uint8_t)b);
        return q;
    }();
    return t;
}

// Persistent grid (as many CTAs as fit on the device at once): thread i
// quantizes blocks i, i + T, i + 2T, ... (T threads in the grid), so a warp
// reads 1 KB of contiguous BF16 per block and all resident threads together
// read one contiguous stretch.  The loads of a thread's next block are in
// flight while it quantizes the current one (two register sets used in turn),
// and the first loads go out before the tables are copied to shared memory.
// Launched with programmatic stream serialization behind a GEMM that may
// still read this kernel's output buffers: nothing in global memory is read
// or written before grid_dependency_wait.
__global__ void __launch_bounds__(kThreads, 6) nvfp4_quantize_kernel(const __grid_constant__ QuantParams p) {
    __shared__ __align__(16) uint8_t s_tables[kSmemTableBytes];

    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t end = p.total;
    const uint32_t stride = gridDim.x * kThreads;
    uint32_t idx = blockIdx.x * kThreads + threadIdx.x;
    uint32_t wa[8], wb[8], ra, kba, rb = 0, kbb = 0;
    ptx::grid_dependency_wait();
    load_block(p, idx, end, wa, ra, kba);
    const SmemTables tab = copy_tables(&g_qtab, s_tables, threadIdx.x, kThreads);
    __syncthreads();
    // A GEMM launched behind this kernel may start setting up (it waits for
    // this grid to complete before reading the quantized activations).
    ptx::launch_dependents();

    // Whether the warp's first lane has a block at idx + stride: warp-uniform,
    // as the scale bytes are gathered with shuffles.
    for (;;) {
        const bool more_b = idx - lane + stride < end;
        if (more_b) load_block(p, idx + stride, end, wb, rb, kbb);
        quantize_and_store(p, idx, end, wa, ra, kba, lane, tab);
        if (!more_b) break;
        idx += stride;
        const bool more_a = idx - lane + stride < end;
        if (more_a) load_block(p, idx + stride, end, wa, ra, kba);
        quantize_and_store(p, idx, end, wb, rb, kbb, lane, tab);
        if (!more_a) break;
        idx += stride;
    }
}

// Staged variant for inputs whose rows are stored back to back (ld == cols, a
// multiple of 64, 16-byte aligned): the stored blocks of rows [0, rows) are one
// contiguous array of 32-byte blocks, so span j (BPC x 256 of them) is one 1-D
// bulk copy; a stored block (r, kb) goes to block kb of padded row r.  The
// blocks that are not stored (the K padding of each row, when cols < K_pad,
// and the padding rows) are zeros, written after the spans.
// A producer warp streams the spans of this CTA (j = CTA, CTA + G, ...) into a
// ring of STAGES shared-memory stages with cp.async.bulk; eight consumer warps
// quantize BPC blocks per thread from shared memory and release the stage.
// BPC = 1: 8 KB spans, 4 stages, 5 CTAs per SM (160 KB in flight per SM);
// BPC = 2: 16 KB spans, 2 stages, 4 CTAs per SM (128 KB in flight), which
// halves the per-span work (barriers, index arithmetic) per block but leaves
// fewer spans per CTA, so it is used from 4 Mi blocks up.  Blocks of the
// padding rows are zeros.
constexpr int kStagedWarps = 8;
constexpr int kStagedThreads = (kStagedWarps + 1) * 32;
constexpr int kErrQuantStageTimeout = 5;  // device error word: a quantizer ring wait gave up
constexpr uint64_t kQuantDrainNs = 200000;  // after a timeout, let issued copies land
constexpr uint32_t kTwoBlocksFrom = 1u << 22;  // blocks of a launch from which BPC = 2

template <int BPC, int STAGES, int MIN_CTAS>
__global__ void __launch_bounds__(kStagedThreads, MIN_CTAS)
    nvfp4_quantize_staged_kernel(const __grid_constant__ QuantParams p, int* err) {
    constexpr int kSpanBlocks = kStagedWarps * 32 * BPC;
    constexpr int kSpanBytes = kSpanBlocks * 32;
    constexpr int kStagedStages = STAGES;
    __shared__ __align__(128) uint8_t s_stage[kStagedStages][kSpanBytes];
    __shared__ __align__(16) uint8_t s_tables[kSmemTableBytes];
    __shared__ __align__(8) uint64_t full[kStagedStages], empty[kStagedStages];
    __shared__ int s_abort;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t dense = p.rows * p.cpb;  // blocks stored in memory
    const uint32_t nspans = (dense + kSpanBlocks - 1) / kSpanBlocks;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStagedStages; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], kStagedWarps);
        }
        s_abort = 0;
        ptx::fence_mbar_init();
    }
    const SmemTables tab = copy_tables(&g_qtab, s_tables, threadIdx.x, kStagedThreads);
    __syncthreads();
    // The input may be the output of the kernel before this one, and that
    // kernel may still read the buffers this one writes.
    ptx::grid_dependency_wait();
    ptx::launch_dependents();

    bool timed_out = false;
    if (warp == kStagedWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t k = 0;
            for (uint32_t span = blockIdx.x; span < nspans; span += gridDim.x, ++k) {
                const uint32_t s = k % kStagedStages;
                if (k >= kStagedStages && !ptx::mbar_wait(&empty[s], ((k / kStagedStages) - 1) & 1)) {
                    timed_out = true;
                    break;
                }
                if (*reinterpret_cast<volatile int*>(&s_abort)) break;
                const uint32_t b0 = span * kSpanBlocks;
                const uint32_t nb = dense > b0 ? min((uint32_t)kSpanBlocks, dense - b0) : 0u;
                if (nb > 0) {
                    ptx::mbar_arrive_expect_tx(&full[s], nb * 32u);
                    ptx::bulk_load(s_stage[s], p.src + (size_t)b0 * kSfVec, nb * 32u, &full[s]);
                } else {
                    ptx::mbar_arrive(&full[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        uint32_t k = 0;
        for (uint32_t span = blockIdx.x; span < nspans; span += gridDim.x, ++k) {
            const uint32_t s = k % kStagedStages;
            const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (k / kStagedStages) & 1));
            if (!ok || *reinterpret_cast<volatile int*>(&s_abort)) {
                timed_out = !ok;
                break;
            }
            uint32_t w[BPC][8], idx[BPC], r[BPC], kb[BPC], end[BPC];
#pragma unroll
            for (int u = 0; u < BPC; ++u) {
                const uint32_t off = threadIdx.x + (uint32_t)u * (kStagedWarps * 32);
                const uint32_t mb = span * kSpanBlocks + off;  // stored block
                r[u] = (__umulhi(mb, p.cpb_mul) + mb) >> p.cpb_shift;
                kb[u] = mb - r[u] * p.cpb;
                idx[u] = r[u] * p.nsb + kb[u];
                end[u] = mb < dense ? p.total : 0u;
                if (mb < dense) {
                    const uint4* src = reinterpret_cast<const uint4*>(s_stage[s] + off * 32u);
                    const uint4 v0 = src[0], v1 = src[1];
                    w[u][0] = v0.x; w[u][1] = v0.y; w[u][2] = v0.z; w[u][3] = v0.w;
                    w[u][4] = v1.x; w[u][5] = v1.y; w[u][6] = v1.z; w[u][7] = v1.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) w[u][i] = 0u;
                }
            }
#pragma unroll
            for (int u = 0; u < BPC; ++u) quantize_and_store(p, idx[u], end[u], w[u], r[u], kb[u], lane, tab);
            // The stage's bytes were consumed above (the stores depend on them).
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[s]);
        }
        // Blocks not stored in memory: the K padding of rows [0, rows), then the
        // padding rows; zeros (code 0, scale 0x01).  Warp-uniform trips; four
        // consecutive lanes hold four consecutive blocks of one row (the K
        // padding and K_pad / 16 are multiples of 4).
        const uint32_t kpad = p.nsb - p.cpb;
        const uint32_t n_kpad = p.rows * kpad;
        const uint32_t n_pad = n_kpad + (p.total - p.rows * p.nsb);
        const uint32_t zero[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        for (uint32_t i0 = (blockIdx.x * kStagedWarps + warp) * 32u; i0 < n_pad && !timed_out;
             i0 += gridDim.x * kStagedWarps * 32u) {
            const uint32_t i = i0 + lane;
            uint32_t r, kb;
            if (i < n_kpad) {
                r = i / kpad;
                kb = p.cpb + (i - r * kpad);
            } else {
                const uint32_t j = i - n_kpad;
                r = p.rows + j / p.nsb;
                kb = j - (r - p.rows) * p.nsb;
            }
            quantize_and_store(p, r * p.nsb + kb, i < n_pad ? p.total : 0u, zero, r, kb, lane, tab);
        }
    }
    if (timed_out) {
        if (err) atomicCAS(err, 0, kErrQuantStageTimeout);
        atomicExch(&s_abort, 1);
    }
    __syncthreads();
    if (s_abort) {
        // Copies issued before the timeout still land in this CTA's shared memory.
        const uint64_t t0 = ptx::global_timer_ns();
        while (ptx::global_timer_ns() - t0 < kQuantDrainNs) {
        }
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
    p.cpb = (uint32_t)(a.cols / kSfVec);
    qcore::make_fast_div(p.cpb > 0 ? p.cpb : 1u, &p.cpb_mul, &p.cpb_shift);
    return p;
}

namespace {

// Launch with programmatic stream serialization (the kernels wait for the
// previous kernel on the stream before touching global memory).
template <typename K, typename... Args>
cudaError_t launch_pdl(K kernel, uint32_t grid, uint32_t threads, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Resident CTAs of `kernel` on the current device (once per device and kernel).
template <typename K>
int resident_ctas(K kernel, int threads, std::once_flag* once, int* cache) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [&] {
        int occ = 0, sms = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, 0) != cudaSuccess || occ < 1) occ = 1;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const char* e = getenv("FP4B_QUANT_CTAS_PER_SM");
        if (e && atoi(e) > 0 && atoi(e) < occ) occ = atoi(e);
        cache[dev & 63] = occ * (sms > 0 ? sms : 148);
    });
    cudaGetLastError();
    return cache[dev & 63];
}

}  // namespace

cudaError_t quantize_launch(const QuantizeArgs& a, cudaStream_t stream) {
    const QuantParams p = make_quant_params(a);
    if (!quant_tables_device()) return cudaErrorInvalidValue;
    if (p.total == 0) return cudaSuccess;
    // Dense input: rows back to back with no column padding -> staged kernel.
    const char* staged_env = getenv("FP4B_QUANT_STAGED");
    const bool staged_ok = staged_env ? atoi(staged_env) != 0 : true;
    if (staged_ok && p.vec_ok && p.ld == p.cols && p.cols % 64 == 0) {
        if (p.total >= kTwoBlocksFrom) {
            auto kernel = nvfp4_quantize_staged_kernel<2, 2, 4>;
            static std::once_flag once[64];
            static int cache[64];
            const uint64_t need = ((uint64_t)p.total + 511) / 512;
            const uint64_t cap = (uint64_t)resident_ctas(kernel, kStagedThreads, once, cache);
            return launch_pdl(kernel, (uint32_t)(need < cap ? need : cap), kStagedThreads, stream, p,
                              device_error_word());
        }
        auto kernel = nvfp4_quantize_staged_kernel<1, 4, 5>;
        static std::once_flag once[64];
        static int cache[64];
        const uint64_t need = ((uint64_t)p.total + 255) / 256;
        const uint64_t cap = (uint64_t)resident_ctas(kernel, kStagedThreads, once, cache);
        return launch_pdl(kernel, (uint32_t)(need < cap ? need : cap), kStagedThreads, stream, p,
                          device_error_word());
    }
    static std::once_flag once[64];
    static int cache[64];
    const uint64_t need = ((uint64_t)p.total + kThreads - 1) / kThreads;
    const uint64_t cap = (uint64_t)resident_ctas(nvfp4_quantize_kernel, kThreads, once, cache);
    return launch_pdl(nvfp4_quantize_kernel, (uint32_t)(need < cap ? need : cap), kThreads, stream, p);
}

}  // namespace fp4b
