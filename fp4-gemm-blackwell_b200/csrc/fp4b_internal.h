// fp4b_internal.h -- host-side interfaces between the kernels and the C ABI.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace fp4b {

// A BF16 matrix [rows, cols] with row stride `ld` elements, quantized into a
// zero-padded NVFP4 operand [rows_pad, k_pad/2] + interleaved scales
// (rows_pad * k_pad / 16 bytes).  rows_pad, k_pad: multiples of 128.
struct QuantizeArgs {
    const void* src;
    long rows, cols, ld;
    long rows_pad, k_pad;
    uint8_t* fp4;
    uint8_t* sf;
};

// Check the geometry; returns nullptr when valid, else a message.
const char* quantize_check(const QuantizeArgs& a);
cudaError_t quantize_launch(const QuantizeArgs& a, cudaStream_t stream);

// D[M, n_out] = epilogue(A_fp4 x B_fp4^T): alpha * acc + beta * C, rounded to
// bf16, then + bias[n] rounded to bf16 again (bias optional).  A has
// m_rows_pad rows, B has n_rows_pad rows, both k_pad wide (multiples of 128).
struct GemmArgs {
    const uint8_t* a_fp4;
    const uint8_t* a_sf;
    const uint8_t* b_fp4;
    const uint8_t* b_sf;
    long m, n_out, k_pad;
    long m_rows_pad, n_rows_pad;
    const void* c;  // bf16 [m, ldc] or null
    long ldc;
    void* d;        // bf16 [m, ldd]
    long ldd;
    const void* bias;  // bf16 [n_out] or null
    float alpha, beta;
    // B is a weight cache and the GEMM is launched right behind the activation
    // quantizer on the same stream.  That quantizer lets the GEMM launch only
    // after its own programmatic wait, i.e. after every earlier kernel
    // (including one that wrote the cache) completed, so the CTA-pair kernel
    // may load B before its own programmatic wait.
    bool b_cached = false;
};

const char* gemm_check(const GemmArgs& g);
// Output columns per tile that gemm_launch picks without FP4B_PAIR / FP4B_FORCE_BN:
// the CTA-pair kernel's 128 / 192 / 256 / 320 / 384 (pairs at every M); -1 on
// bad arguments.  Host only.
int gemm_tile_width(long m, long n, long k_pad, int sms);
cudaError_t gemm_launch(const GemmArgs& g, cudaStream_t stream);

// Overlapped cached linear (CTA-pair path, M > 128, tiles in one round of CTA
// pairs; opt-in with FP4B_OVERLAP=1): launches the activation quantizer of
// quantize_units.cu (`qa`, whose outputs must be g.a_fp4 / g.a_sf) and, right
// behind it, the GEMM, which runs beside the quantizer on the same SMs and
// waits for the units of A it needs.  `ready` is a device array of
// 1 + (m_rows_pad / 128) * ceil(k_pad / 256) words that is zero before the
// first launch; the GEMM leaves it zero.  Launches that share `ready` must be
// ordered (same stream).  Returns cudaErrorNotSupported, having launched
// nothing, when the path does not apply; the caller then runs quantize_launch
// and gemm_launch.
cudaError_t gemm_launch_overlapped(const GemmArgs& g, const QuantizeArgs& qa, uint32_t* ready,
                                   cudaStream_t stream);

// The overlapped path's quantizer (quantize_units.cu): nullptr if `a` suits
// it (16-byte aligned rows, padded rows a multiple of 64), else a message;
// its dynamic shared memory for a ring of `ring` 8 KB stages; its launch
// (`grid` CTAs, one per SM) publishing unit counters into `ready`.
const char* quantize_units_check(const QuantizeArgs& a);
int quantize_units_smem_bytes(int ring);
cudaError_t quantize_units_launch(const QuantizeArgs& a, uint32_t* ready, int ring, int grid, cudaStream_t stream);

// GEMM whose output tile is also stored into `npeers` (1..7) other BF16
// buffers with the same row stride (other GPUs' memory mapped into this
// process, each offset to the columns this rank computes): the column-parallel
// all-gather done by the epilogue.  CTA-pair kernel, no C, D rows 16-byte
// aligned; else cudaErrorNotSupported.
cudaError_t gemm_launch_peers(const GemmArgs& g, void* const* peers, int npeers, cudaStream_t stream);



// Read-only view of a weight-cache handle created by the C ABI.
struct CacheView {
    const uint8_t* fp4;
    const uint8_t* sf;
    int N, K;
    float w_alpha;  // factor every GEMM with the cache applies (global weight scale)
};
// False for a null or foreign handle.
bool cache_view(const void* handle, CacheView* out);

// Device-side error word written by kernels that gave up on a bounded wait.
int* device_error_word();
int read_and_clear_device_error();

// Per-thread message of the last failure in the C ABI.
void set_last_error(const char* fmt, ...);

// 0 for cudaSuccess; otherwise records "<what>: <CUDA error>" as the last
// error, prints it to stderr like the reference's messages, and returns -4
// (the C ABI's launch-failure code).
int launch_status(cudaError_t e, const char* what);

}  // namespace fp4b
