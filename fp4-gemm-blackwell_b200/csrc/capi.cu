// capi.cu -- the C ABI of libfp4gemm.so (declared in include/fp4gemm.h).
//
// Keeps the reference library's exported symbols and their behaviour
// (fp4_gemm_lib.cu:401-842): the same return codes, the same shape rules, the
// same synchronisation points, the same handle semantics.  What changes is
// underneath: the reference's single global FP4GemmState becomes one scratch
// state per CUDA device behind a mutex, every allocation is checked, and the
// kernels are the sm_100a ones in quantize.cu / gemm_sm100.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"

#define FP4B_EXPORT extern "C" __attribute__((visibility("default")))

namespace fp4b {

namespace {

constexpr int kMaxDevices = 64;
constexpr uint32_t kCacheMagic = 0xF4CAC4E1u;

thread_local char t_last_error[512] = "";

struct Buffer {
    uint8_t* ptr = nullptr;
    size_t cap = 0;
};

// Scratch for per-call quantized operands; mirrors FP4GemmState
// (fp4_gemm_lib.cu:346-379) minus the host mirrors and the CUTLASS workspace.
struct DeviceState {
    bool initialized = false;
    int M = 0, N = 0, K = 0;
    Buffer a_fp4, a_sf, b_fp4, b_sf;
    Buffer sync;  // zeroed unit counters of the overlapped quantize + GEMM
};

// g_mu guards the scratch state; launchers run while it is held, so anything
// they call (device_error_word) must use its own lock.
std::mutex g_mu;
DeviceState g_state[kMaxDevices];
std::mutex g_err_mu;
int* g_err_word[kMaxDevices];

struct WeightCache {
    uint32_t magic;
    uint8_t* fp4;  // [N, K/2]
    uint8_t* sf;   // N*K/16 bytes
    int N, K;
    int device;
    bool owns;
    // The cached bytes are of weight * (1 / w_alpha); every GEMM with this cache
    // multiplies its alpha by w_alpha (1 unless a global weight scale was set).
    float w_alpha;
};

__device__ int g_device_error;

long round_up(long x, long m) { return (x + m - 1) / m * m; }

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return (d >= 0 && d < kMaxDevices) ? d : 0;
}

void release(Buffer& b) {
    if (b.ptr) cudaFree(b.ptr);
    b = Buffer{};
}

// Grow-only scratch; cudaFree of the old buffer waits for the device, so no
// kernel can still be reading it.
bool reserve(Buffer& b, size_t bytes) {
    if (b.cap >= bytes && b.ptr) return true;
    release(b);
    if (bytes == 0) return true;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        set_last_error("cudaMalloc(%zu) failed", bytes);
        return false;
    }
    b.ptr = static_cast<uint8_t*>(p);
    b.cap = bytes;
    return true;
}

// Grow-only buffer that is all zeros when handed out (the kernels using it
// leave it zero).
bool reserve_zeroed(Buffer& b, size_t bytes) {
    if (b.cap >= bytes && b.ptr) return true;
    if (!reserve(b, bytes)) return false;
    if (cudaMemset(b.ptr, 0, b.cap) != cudaSuccess) {
        cudaGetLastError();
        release(b);
        set_last_error("cudaMemset of the counter buffer failed");
        return false;
    }
    return true;
}

void cleanup_state(DeviceState& s) {
    release(s.sync);
    release(s.a_fp4);
    release(s.a_sf);
    release(s.b_fp4);
    release(s.b_sf);
    s = DeviceState{};
}

WeightCache* as_cache(const void* h) {
    auto* c = static_cast<WeightCache*>(const_cast<void*>(h));
    return (c && c->magic == kCacheMagic) ? c : nullptr;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Reference fp4_gemm_init (fp4_gemm_lib.cu:435-500); caller holds g_mu.
int init_locked(DeviceState& s, int M, int N, int K) {
    if (s.initialized && s.M == M && s.N == N && s.K == K) return 0;
    const size_t need_a = (size_t)M * K / 2, need_b = (size_t)N * K / 2;
    const size_t need_sfa = (size_t)M * K / 16, need_sfb = (size_t)N * K / 16;
    if (s.initialized && M > 0 && N > 0 && K > 0 && s.a_fp4.cap >= need_a && s.b_fp4.cap >= need_b &&
        s.a_sf.cap >= need_sfa && s.b_sf.cap >= need_sfb) {
        s.M = M;
        s.N = N;
        s.K = K;
        return 0;
    }
    cleanup_state(s);
    if (M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128 || K % 128) {
        fprintf(stderr, "fp4_gemm: M=%d, N=%d, K=%d must all be multiples of 128\n", M, N, K);
        set_last_error("M=%d, N=%d, K=%d must all be multiples of 128", M, N, K);
        return -1;
    }
    if (!reserve(s.a_fp4, need_a) || !reserve(s.b_fp4, need_b) || !reserve(s.a_sf, need_sfa) ||
        !reserve(s.b_sf, need_sfb)) {
        cleanup_state(s);
        return -1;
    }
    s.M = M;
    s.N = N;
    s.K = K;
    s.initialized = true;
    return 0;
}

int quantize_into(const void* src, long rows, long cols, long ld, uint8_t* fp4, uint8_t* sf, long rows_pad,
                  long k_pad, cudaStream_t st) {
    QuantizeArgs q{src, rows, cols, ld, rows_pad, k_pad, fp4, sf};
    if (const char* why = quantize_check(q)) {
        set_last_error("quantize: %s", why);
        return -2;
    }
    return launch_status(quantize_launch(q, st), "quantize launch");
}

int gemm_into(const GemmArgs& g, cudaStream_t st) {
    if (const char* why = gemm_check(g)) {
        set_last_error("gemm: %s", why);
        return -2;
    }
    return launch_status(gemm_launch(g, st), "gemm launch");
}

}  // namespace

int launch_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    set_last_error("%s: %s", what, cudaGetErrorString(e));
    fprintf(stderr, "fp4_gemm: %s: %s\n", what, cudaGetErrorString(e));
    return -4;
}

int* device_error_word() {
    const int d = current_device();
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err_word[d]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_err_word[d] = static_cast<int*>(p);
    }
    return g_err_word[d];
}

int read_and_clear_device_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    }
    return v;
}

bool cache_view(const void* handle, CacheView* out) {
    WeightCache* c = as_cache(handle);
    if (!c) return false;
    *out = CacheView{c->fp4, c->sf, c->N, c->K, c->w_alpha};
    return true;
}

void set_last_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
}

}  // namespace fp4b

using namespace fp4b;

// =============================================================== reference ABI

FP4B_EXPORT int fp4_gemm_sf_vec_size(void) { return kSfVec; }

FP4B_EXPORT int fp4_gemm_init(int M, int N, int K) {
    std::lock_guard<std::mutex> lk(g_mu);
    return init_locked(g_state[current_device()], M, N, K);
}

FP4B_EXPORT int fp4_gemm_prealloc(int max_M, int max_N, int max_K) { return fp4_gemm_init(max_M, max_N, max_K); }

FP4B_EXPORT int fp4_gemm_run(const void* A, const void* B, const void* C, void* D, int M, int N, int K, float alpha,
                             float beta) {
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = g_state[current_device()];
    if (int rc = init_locked(s, M, N, K)) return rc;
    if (M % 128 || N % 128 || K % 128) {
        set_last_error("M=%d, N=%d, K=%d must all be multiples of 128", M, N, K);
        return -2;
    }
    cudaStream_t st = nullptr;
    if (int rc = quantize_into(A, M, K, K, s.a_fp4.ptr, s.a_sf.ptr, M, K, st)) return rc;
    if (int rc = quantize_into(B, N, K, K, s.b_fp4.ptr, s.b_sf.ptr, N, K, st)) return rc;
    GemmArgs g{s.a_fp4.ptr, s.a_sf.ptr, s.b_fp4.ptr, s.b_sf.ptr, M, N, K, M, N, C ? C : D, N, D, N, nullptr,
               alpha, beta};
    if (int rc = gemm_into(g, st)) return rc;
    cudaDeviceSynchronize();
    return 0;
}

FP4B_EXPORT int fp4_gemm_run_host(const void*, const void*, const void*, void*, int, int, int, float, float) {
    set_last_error("fp4_gemm_run_host (host quantization) is not provided by this library");
    fprintf(stderr, "fp4_gemm_run_host: host quantization is not provided; use fp4_gemm_run\n");
    return -2;
}

FP4B_EXPORT void fp4_gemm_cleanup(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    cleanup_state(g_state[current_device()]);
}

FP4B_EXPORT void fp4_gemm_sync(void) { cudaDeviceSynchronize(); }

FP4B_EXPORT void* fp4b_quantize_weights_ex(const void* w, int n, int k, int ldw, void* stream, int sync) {
    if (!w || n <= 0 || k <= 0 || ldw < k) {
        set_last_error("fp4b_quantize_weights_ex: bad arguments");
        return nullptr;
    }
    const long N = round_up(n, 128), K = round_up(k, 128);
    auto* c = new WeightCache{kCacheMagic, nullptr, nullptr, (int)N, (int)K, current_device(), true, 1.0f};
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)N * K / 2) != cudaSuccess) {
        cudaGetLastError();
        fprintf(stderr, "fp4_quantize_weights: cudaMalloc fp4 failed\n");
        set_last_error("cudaMalloc fp4 failed");
        delete c;
        return nullptr;
    }
    c->fp4 = static_cast<uint8_t*>(p);
    if (cudaMalloc(&p, (size_t)N * K / 16) != cudaSuccess) {
        cudaGetLastError();
        fprintf(stderr, "fp4_quantize_weights: cudaMalloc sf failed\n");
        set_last_error("cudaMalloc sf failed");
        cudaFree(c->fp4);
        delete c;
        return nullptr;
    }
    c->sf = static_cast<uint8_t*>(p);
    if (quantize_into(w, n, k, ldw, c->fp4, c->sf, N, K, as_stream(stream)) != 0) {
        cudaFree(c->fp4);
        cudaFree(c->sf);
        delete c;
        return nullptr;
    }
    if (sync) cudaDeviceSynchronize();
    return c;
}

FP4B_EXPORT void* fp4_quantize_weights(const void* weight_bf16, int N, int K) {
    if (N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0) {
        fprintf(stderr, "fp4_quantize_weights: N=%d, K=%d must be multiples of 128\n", N, K);
        set_last_error("N=%d, K=%d must be multiples of 128", N, K);
        return nullptr;
    }
    return fp4b_quantize_weights_ex(weight_bf16, N, K, K, nullptr, 1);
}

FP4B_EXPORT const void* fp4_weight_cache_fp4_ptr(const void* h) {
    WeightCache* c = as_cache(h);
    return c ? c->fp4 : nullptr;
}

FP4B_EXPORT const void* fp4_weight_cache_sf_ptr(const void* h) {
    WeightCache* c = as_cache(h);
    return c ? c->sf : nullptr;
}

FP4B_EXPORT int fp4_weight_cache_N(const void* h) {
    WeightCache* c = as_cache(h);
    return c ? c->N : 0;
}

FP4B_EXPORT int fp4_weight_cache_K(const void* h) {
    WeightCache* c = as_cache(h);
    return c ? c->K : 0;
}

FP4B_EXPORT void fp4_weight_cache_free(void* h) {
    WeightCache* c = as_cache(h);
    if (!c) return;
    if (c->owns) {
        cudaFree(c->fp4);
        cudaFree(c->sf);
    }
    c->magic = 0;
    delete c;
}

FP4B_EXPORT int fp4b_run_cached_ex(const void* A, int m, int k_in, int lda, const void* h, int n_out, const void* C,
                                   int ldc, void* D, int ldd, const void* bias, float alpha, float beta,
                                   void* stream) {
    WeightCache* c = as_cache(h);
    if (!c) {
        set_last_error("null or invalid cache handle");
        return -1;
    }
    if (!A || !D || m <= 0 || k_in <= 0 || k_in > c->K || lda < k_in || n_out <= 0 || n_out > c->N) {
        set_last_error("fp4b_run_cached_ex: bad shape (m=%d k=%d n=%d vs cache %dx%d)", m, k_in, n_out, c->N, c->K);
        return -1;
    }
    const long m_pad = round_up(m, 128);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = g_state[current_device()];
    if (!reserve(s.a_fp4, (size_t)m_pad * c->K / 2) || !reserve(s.a_sf, (size_t)m_pad * c->K / 16)) return -1;
    cudaStream_t st = as_stream(stream);
    GemmArgs g{s.a_fp4.ptr, s.a_sf.ptr, c->fp4, c->sf, m, n_out, c->K, m_pad, c->N, C, ldc, D, ldd, bias,
               alpha * c->w_alpha, beta};
    QuantizeArgs q{A, m, k_in, lda, m_pad, c->K, s.a_fp4.ptr, s.a_sf.ptr};
    g.b_cached = true;  // right behind the activation quantizer
    if (m > 128 && !quantize_check(q) && !gemm_check(g) &&
        reserve_zeroed(s.sync, (size_t)(1 + (m_pad / 128) * ((c->K + 255) / 256)) * sizeof(uint32_t))) {
        // The quantizer and the GEMM run side by side (CTA-pair path, one round of tiles).
        const cudaError_t e = gemm_launch_overlapped(g, q, reinterpret_cast<uint32_t*>(s.sync.ptr), st);
        if (e != cudaErrorNotSupported) return launch_status(e, "overlapped quantize+gemm launch");
    }
    if (int rc = quantize_into(A, m, k_in, lda, s.a_fp4.ptr, s.a_sf.ptr, m_pad, c->K, st)) return rc;
    return gemm_into(g, st);
}

FP4B_EXPORT int fp4b_run_cached_peers(const void* A, int m, int k_in, int lda, const void* h, int n_out,
                                      void* D, int ldd, void* const* peer_d, int npeers, const void* bias,
                                      void* stream) {
    // The epilogue writes D and every peer buffer with TMA stores, whose tensor
    // maps need 16-byte aligned rows: a misaligned peer address or row stride
    // is refused here, before anything is looked up or launched.
    if (peer_d && npeers >= 1 && npeers <= 7) {
        bool aligned = ldd % 8 == 0 && (reinterpret_cast<uintptr_t>(D) & 15) == 0;
        for (int i = 0; i < npeers && aligned; ++i)
            aligned = peer_d[i] && (reinterpret_cast<uintptr_t>(peer_d[i]) & 15) == 0;
        if (!aligned) {
            set_last_error("fp4b_run_cached_peers: D, every peer_d[i] and ldd must give 16-byte aligned rows "
                           "(addresses multiples of 16 bytes, ldd a multiple of 8 elements, no NULL peer)");
            return -2;
        }
    }
    WeightCache* c = as_cache(h);
    if (!c) {
        set_last_error("null or invalid cache handle");
        return -1;
    }
    if (!A || !D || m <= 0 || k_in <= 0 || k_in > c->K || lda < k_in || n_out <= 0 || n_out > c->N ||
        !peer_d || npeers < 1 || npeers > 7) {
        set_last_error("fp4b_run_cached_peers: bad arguments (m=%d, 1..7 peers)", m);
        return -1;
    }
    const long m_pad = round_up(m, 128);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = g_state[current_device()];
    if (!reserve(s.a_fp4, (size_t)m_pad * c->K / 2) || !reserve(s.a_sf, (size_t)m_pad * c->K / 16)) return -1;
    cudaStream_t st = as_stream(stream);
    GemmArgs g{s.a_fp4.ptr, s.a_sf.ptr, c->fp4, c->sf, m, n_out, c->K, m_pad, c->N, nullptr, 0, D, ldd, bias,
               c->w_alpha, 0.0f};
    if (const char* why = gemm_check(g)) {
        set_last_error("gemm: %s", why);
        return -2;
    }
    if (int rc = quantize_into(A, m, k_in, lda, s.a_fp4.ptr, s.a_sf.ptr, m_pad, c->K, st)) return rc;
    g.b_cached = true;
    const cudaError_t e = gemm_launch_peers(g, peer_d, npeers, st);
    if (e == cudaErrorNotSupported) {
        set_last_error("fp4b_run_cached_peers: the output tensor map could not be built for D");
        return -2;
    }
    return launch_status(e, "peer gemm launch");
}

FP4B_EXPORT int fp4b_copy2d(void* dst, long dpitch, const void* src, long spitch, long width_bytes, long height,
                            void* stream) {
    if (!dst || !src || width_bytes <= 0 || height <= 0 || dpitch < width_bytes || spitch < width_bytes) {
        set_last_error("fp4b_copy2d: bad arguments");
        return -1;
    }
    return launch_status(cudaMemcpy2DAsync(dst, (size_t)dpitch, src, (size_t)spitch, (size_t)width_bytes,
                                           (size_t)height, cudaMemcpyDeviceToDevice, as_stream(stream)),
                         "fp4b_copy2d");
}

namespace {
using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
GetAddressRangeFn address_range_fn() {
    static GetAddressRangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<GetAddressRangeFn>(f);
    }();
    return fn;
}
}  // namespace

FP4B_EXPORT int fp4b_ipc_get_handle(const void* ptr, void* handle_out, long* offset_out) {
    GetAddressRangeFn range = address_range_fn();
    if (!ptr || !handle_out || !offset_out || !range) {
        set_last_error("fp4b_ipc_get_handle: bad arguments or no driver entry point");
        return -1;
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        set_last_error("fp4b_ipc_get_handle: pointer is not device memory");
        return -1;
    }
    cudaIpcMemHandle_t hdl;
    if (cudaIpcGetMemHandle(&hdl, reinterpret_cast<void*>(base)) != cudaSuccess) {
        cudaGetLastError();
        set_last_error("cudaIpcGetMemHandle failed");
        return -1;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    memcpy(handle_out, &hdl, sizeof(hdl));
    *offset_out = (long)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return 0;
}

FP4B_EXPORT void* fp4b_ipc_open_handle(const void* handle, long offset) {
    if (!handle || offset < 0) return nullptr;
    cudaIpcMemHandle_t hdl;
    memcpy(&hdl, handle, sizeof(hdl));
    void* base = nullptr;
    if (cudaIpcOpenMemHandle(&base, hdl, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        set_last_error("cudaIpcOpenMemHandle failed");
        return nullptr;
    }
    return static_cast<uint8_t*>(base) + offset;
}

FP4B_EXPORT int fp4b_ipc_close(void* ptr, long offset) {
    if (!ptr) return -1;
    if (cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset) != cudaSuccess) {
        cudaGetLastError();
        set_last_error("cudaIpcCloseMemHandle failed");
        return -1;
    }
    return 0;
}

FP4B_EXPORT int fp4_gemm_run_cached(const void* A, const void* h, const void* C, void* D, int M, float alpha,
                                    float beta) {
    WeightCache* c = as_cache(h);
    if (!c) {
        fprintf(stderr, "fp4_gemm_run_cached: null cache handle\n");
        set_last_error("null cache handle");
        return -1;
    }
    if (M <= 0 || M % 128 != 0) {
        fprintf(stderr, "fp4_gemm_run_cached: M=%d must be a multiple of 128\n", M);
        set_last_error("M=%d must be a multiple of 128", M);
        return -1;
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (int rc = init_locked(g_state[current_device()], M, c->N, c->K)) return rc;
    }
    return fp4b_run_cached_ex(A, M, c->K, c->K, h, c->N, C ? C : D, c->N, D, c->N, nullptr, alpha, beta, nullptr);
}

// ============================================================== additive ABI

FP4B_EXPORT int fp4b_version(void) { return 1; }

FP4B_EXPORT int fp4b_gemm_tile_width(int m, int n, int k, int sms) {
    if (m <= 0 || n <= 0 || k <= 0 || sms < 2) {
        set_last_error("fp4b_gemm_tile_width: m, n, k must be positive and sms at least 2");
        return -1;
    }
    return gemm_tile_width(m, n, round_up(k, 128), sms);
}

FP4B_EXPORT const char* fp4b_last_error(void) { return t_last_error; }

FP4B_EXPORT int fp4b_device_error(int clear) {
    cudaDeviceSynchronize();
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    }
    return v;
}

FP4B_EXPORT int fp4b_quantize(const void* src, int rows, int cols, int ld, void* dst_fp4, void* dst_sf,
                              int rows_pad, int k_pad, void* stream) {
    const int rc = quantize_into(src, rows, cols, ld, static_cast<uint8_t*>(dst_fp4), static_cast<uint8_t*>(dst_sf),
                                 rows_pad, k_pad, as_stream(stream));
    return rc == -2 ? -1 : rc;
}

FP4B_EXPORT int fp4b_gemm_prequant(const void* a_fp4, const void* a_sf, int m, int m_rows_pad, const void* b_fp4,
                                   const void* b_sf, int n_out, int n_rows_pad, int k_pad, const void* C, int ldc,
                                   void* D, int ldd, const void* bias, float alpha, float beta, void* stream) {
    GemmArgs g{static_cast<const uint8_t*>(a_fp4), static_cast<const uint8_t*>(a_sf),
               static_cast<const uint8_t*>(b_fp4), static_cast<const uint8_t*>(b_sf), m, n_out, k_pad, m_rows_pad,
               n_rows_pad, C, ldc, D, ldd, bias, alpha, beta};
    const int rc = gemm_into(g, as_stream(stream));
    return rc == -2 ? -1 : rc;
}

FP4B_EXPORT int fp4b_run_ex(const void* A, int m, int k, int lda, const void* B, int n, int ldb, const void* C,
                            int ldc, void* D, int ldd, const void* bias, float alpha, float beta, void* stream) {
    if (!A || !B || !D || m <= 0 || n <= 0 || k <= 0 || lda < k || ldb < k) {
        set_last_error("fp4b_run_ex: bad arguments");
        return -1;
    }
    const long m_pad = round_up(m, 128), n_pad = round_up(n, 128), k_pad = round_up(k, 128);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = g_state[current_device()];
    if (!reserve(s.a_fp4, (size_t)m_pad * k_pad / 2) || !reserve(s.a_sf, (size_t)m_pad * k_pad / 16) ||
        !reserve(s.b_fp4, (size_t)n_pad * k_pad / 2) || !reserve(s.b_sf, (size_t)n_pad * k_pad / 16))
        return -1;
    cudaStream_t st = as_stream(stream);
    if (int rc = quantize_into(A, m, k, lda, s.a_fp4.ptr, s.a_sf.ptr, m_pad, k_pad, st)) return rc;
    if (int rc = quantize_into(B, n, k, ldb, s.b_fp4.ptr, s.b_sf.ptr, n_pad, k_pad, st)) return rc;
    GemmArgs g{s.a_fp4.ptr, s.a_sf.ptr, s.b_fp4.ptr, s.b_sf.ptr, m, n, k_pad, m_pad, n_pad, C, ldc, D, ldd, bias,
               alpha, beta};
    return gemm_into(g, st);
}

FP4B_EXPORT void* fp4b_weight_cache_slice(const void* h, int row0, int rows) {
    WeightCache* c = as_cache(h);
    if (!c || row0 < 0 || rows <= 0 || row0 % 128 || rows % 128 || row0 + rows > c->N) {
        set_last_error("fp4b_weight_cache_slice: bad slice");
        return nullptr;
    }
    return new WeightCache{kCacheMagic, c->fp4 + (size_t)row0 * c->K / 2, c->sf + (size_t)row0 * c->K / 16, rows,
                           c->K, c->device, false, c->w_alpha};
}

FP4B_EXPORT int fp4b_weight_cache_set_alpha(void* h, float w_alpha) {
    WeightCache* c = as_cache(h);
    if (!c || !(w_alpha > 0.0f) || !std::isfinite(w_alpha)) {
        set_last_error("fp4b_weight_cache_set_alpha: null handle or non-positive / non-finite factor");
        return -1;
    }
    c->w_alpha = w_alpha;
    return 0;
}

FP4B_EXPORT float fp4b_weight_cache_alpha(const void* h) {
    WeightCache* c = as_cache(h);
    return c ? c->w_alpha : 0.0f;
}

FP4B_EXPORT int fp4b_weight_cache_export(const void* h, void* dst_fp4, void* dst_sf, void* stream) {
    WeightCache* c = as_cache(h);
    if (!c || !dst_fp4 || !dst_sf) {
        set_last_error("fp4b_weight_cache_export: bad arguments");
        return -1;
    }
    cudaStream_t st = as_stream(stream);
    cudaError_t e = cudaMemcpyAsync(dst_fp4, c->fp4, (size_t)c->N * c->K / 2, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dst_sf, c->sf, (size_t)c->N * c->K / 16, cudaMemcpyDeviceToDevice, st);
    return launch_status(e, "weight cache export");
}

FP4B_EXPORT void* fp4b_weight_cache_import(const void* src_fp4, const void* src_sf, int N, int K, void* stream) {
    if (!src_fp4 || !src_sf || N <= 0 || K <= 0 || N % 128 || K % 128) {
        set_last_error("fp4b_weight_cache_import: bad arguments (N, K must be multiples of 128)");
        return nullptr;
    }
    void* a = nullptr;
    void* b = nullptr;
    if (cudaMalloc(&a, (size_t)N * K / 2) != cudaSuccess || cudaMalloc(&b, (size_t)N * K / 16) != cudaSuccess) {
        cudaGetLastError();
        if (a) cudaFree(a);
        set_last_error("fp4b_weight_cache_import: allocation failed");
        return nullptr;
    }
    cudaStream_t st = as_stream(stream);
    cudaError_t e = cudaMemcpyAsync(a, src_fp4, (size_t)N * K / 2, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b, src_sf, (size_t)N * K / 16, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        set_last_error("fp4b_weight_cache_import: %s", cudaGetErrorString(e));
        cudaFree(a);
        cudaFree(b);
        return nullptr;
    }
    return new WeightCache{kCacheMagic, static_cast<uint8_t*>(a), static_cast<uint8_t*>(b), N, K, current_device(),
                           true, 1.0f};
}
