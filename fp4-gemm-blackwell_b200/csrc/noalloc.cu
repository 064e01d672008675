// noalloc.cu -- a cached linear that never allocates device memory.
//
// fp4b_run_cached_ex quantizes the activations into a per-device scratch
// buffer that the library grows with cudaMalloc (and frees with cudaFree,
// which waits for the whole device).  Some callers cannot allow either: a
// serving engine that has already handed nearly all of HBM to its own
// allocator (weights, KV cache, activation pools) and must not see a library
// take memory behind its back, or a pipeline that cannot absorb a
// device-wide synchronisation in the middle of its stream of work.  For them,
// fp4b_run_cached_noalloc keeps its scratch in a fixed array that is part of
// the loaded module instead.
//
// The array (kNoallocScratchBytes, 9 MiB: room for 16 Mi padded activation
// elements as packed E2M1 plus their UE4M3 scales, e.g. 2048 x 8192) is
// device memory of this library's module: it exists on every GPU where the
// module is loaded, until the process exits.  Larger inputs are rejected.  All
// calls on a device share it: two calls whose kernels overlap on the GPU
// (different streams, or the host not ordering them) race on it.  Each call
// rewrites every byte of the region it reads before reading it, so the
// contents left by the previous call never matter and nothing is cleared.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"

#define FP4B_EXPORT extern "C" __attribute__((visibility("default")))

namespace fp4b {
namespace {

constexpr size_t kNoallocMaxElements = size_t(16) << 20;              // padded rows x padded K
constexpr size_t kNoallocFp4Bytes = kNoallocMaxElements / 2;          // 8 MiB of packed E2M1
constexpr size_t kNoallocSfBytes = kNoallocMaxElements / kSfVec;      // 1 MiB of scales
constexpr size_t kNoallocScratchBytes = kNoallocFp4Bytes + kNoallocSfBytes;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[kMaxDevices];

// The host-side name of g_noalloc_scratch is not a device address; the
// device address comes from cudaGetSymbolAddress, once per device, with that
// device current.  The first call on a device does this set-up.
uint8_t* scratch_for_current_device(int* dev_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return nullptr;
    }
    *dev_out = dev;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            set_last_error("fp4b_run_cached_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                           cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace fp4b

using namespace fp4b;

FP4B_EXPORT int fp4b_run_cached_noalloc(const void* A, int m, int k_in, int lda, const void* cache_handle, int n_out,
                                        const void* C, int ldc, void* D, int ldd, const void* bias, float alpha,
                                        float beta, void* stream) {
    CacheView c{};
    if (!cache_view(cache_handle, &c)) {
        set_last_error("fp4b_run_cached_noalloc: null or invalid cache handle");
        return -1;
    }
    if (!A || !D || m <= 0 || k_in <= 0 || k_in > c.K || lda < k_in || n_out <= 0 || n_out > c.N) {
        set_last_error("fp4b_run_cached_noalloc: bad shape (m=%d k=%d n=%d vs cache %dx%d)", m, k_in, n_out, c.N,
                       c.K);
        return -1;
    }
    const long m_pad = (m + 127L) / 128 * 128;
    if ((size_t)m_pad * (size_t)c.K > kNoallocMaxElements) {
        set_last_error(
            "fp4b_run_cached_noalloc: %ld x %d padded activations exceed the fixed scratch of %zu elements "
            "(use fp4b_run_cached_ex, or split M)",
            m_pad, c.K, kNoallocMaxElements);
        return -1;
    }
    int dev = 0;
    uint8_t* scratch = scratch_for_current_device(&dev);
    if (!scratch) return -1;  // the scratch is unavailable, as an allocation failure is in fp4b_run_cached_ex
    uint8_t* a_fp4 = scratch;
    uint8_t* a_sf = scratch + kNoallocFp4Bytes;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    QuantizeArgs q{A, m, k_in, lda, m_pad, c.K, a_fp4, a_sf};
    GemmArgs g{a_fp4, a_sf, c.fp4, c.sf, m, n_out, c.K, m_pad, c.N, C, ldc, D, ldd, bias, alpha * c.w_alpha, beta};
    // Geometry the kernels cannot take: -2 ("cannot implement"), checked for
    // both kernels before either is launched.
    if (const char* why = quantize_check(q)) {
        set_last_error("fp4b_run_cached_noalloc: quantize: %s", why);
        return -2;
    }
    if (const char* why = gemm_check(g)) {
        set_last_error("fp4b_run_cached_noalloc: gemm: %s", why);
        return -2;
    }
    if (int rc = launch_status(quantize_launch(q, st), "fp4b_run_cached_noalloc: quantize launch")) return rc;
    g.b_cached = true;  // right behind the activation quantizer
    return launch_status(gemm_launch(g, st), "fp4b_run_cached_noalloc: gemm launch");
}
