// peak.cu -- the tensor-pipe rate of the block-scaled MMA on this GPU, measured.
//
// fp4b_mma_rate launches CTA pairs (clusters of two, one CTA per SM) whose
// even CTA issues tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16
// instructions (M = 256 across the pair, K = 64 each) from operand tiles that
// stay resident in shared memory: no TMA loads, no global memory in the loop.
// The caller times the launch with CUDA events; the FLOPs are
//   pairs x stages x 4 k-blocks x 2 x 256 x (n0 + n1) x 64.
// With n0 = 256, n1 = 0 and no scale copies this is the dense NVFP4 peak that
// the GEMM's roofline is measured against.  The other arguments reproduce the
// GEMM mainloop's tensor-pipe work per k-block without its loads: two MMAs of
// widths n0 and n1 on the same A tile (the 320- and 384-wide tiles) and the
// tcgen05.cp copies of the scale atoms (one for A plus `sfb_atoms` for B),
// issued like the GEMM issues them: each k-block's copies right before its MMAs.
// The final wait is bounded; the stage count is capped so that a launch runs
// for well under a second.
#include <cuda_runtime.h>

#include <cstdint>

#include "fp4b_internal.h"
#include "ptx_sm100.cuh"

#define FP4B_EXPORT extern "C" __attribute__((visibility("default")))

namespace fp4b {
namespace {

constexpr int kRateThreads = 128;
constexpr int kRateSmemBytes = 120 * 1024;  // more than half an SM: one CTA per SM
constexpr int kAtom = 512;                  // 128 rows x 4 scale bytes
constexpr int kMaxSfbAtoms = 3;
constexpr uint32_t kRateTmemCols = 512;
constexpr uint32_t kTmemSfa = 384;                         // after the widest accumulator (384 columns)
constexpr uint32_t kTmemSfb = kTmemSfa + 16;               // 4 k-blocks x 4 columns of scale-A
constexpr int kErrRateTimeout = 9;                         // device error word: the final wait gave up
constexpr int kMaxRateStages = 1 << 20;

// SFB: scale-B atoms copied per k-block (0..3); TWO: a second MMA of width n1
// per k-block on the same A tile.  Like the GEMM, the whole issuing warp walks
// the loop and one elected lane issues each stage from unrolled code.
template <int SFB, bool TWO>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kRateThreads, 1)
    mma_rate_kernel(int n0, int n1, int sf_copies, int stages, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // A: 128 rows x 128 bytes; B: up to 192 rows x 128 bytes (this CTA's half of
    // n0 + n1 <= 384 rows); scale atoms: 4 for A, 4 x 3 for B.
    uint8_t* sA = smem;
    uint8_t* sB = sA + 128 * 128;
    uint8_t* sSFA = sB + 192 * 128;
    uint8_t* sSFB = sSFA + 4 * kAtom;
    uint64_t* done = reinterpret_cast<uint64_t*>(sSFB + 4 * kMaxSfbAtoms * kAtom);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    // Operands: E2M1 nibbles from an integer hash (finite values of both
    // signs), every scale 0x38 (= 1.0): ordinary data for the tensor pipe.
    const uint32_t total = 128 * 128 + 192 * 128;
    for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
        uint32_t h = (i + 0x9E3779B9u * (blockIdx.x + 1)) * 0x85EBCA6Bu;
        h ^= h >> 13;
        sA[i] = static_cast<uint8_t>(h * 0xC2B2AE35u >> 24);
    }
    for (uint32_t i = threadIdx.x; i < (4 + 4 * kMaxSfbAtoms) * kAtom; i += blockDim.x) sSFA[i] = 0x38;
    if (threadIdx.x == 0) {
        ptx::mbar_init(done, 1);
        ptx::fence_mbar_init();
    }
    ptx::fence_proxy_async_smem();  // the generic-proxy writes above are read by the tensor pipe
    const int warp = threadIdx.x >> 5;
    if (warp == 0) {
        ptx::tmem_alloc_pair(tmem_slot, kRateTmemCols);
        ptx::tmem_relinquish_pair();
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (ptx::cluster_ctarank() == 0 && warp == 0) {
        const uint64_t adesc = ptx::desc_kmajor_sw128(ptx::smem_u32(sA));
        const uint64_t bdesc = ptx::desc_kmajor_sw128(ptx::smem_u32(sB));
        const uint64_t b1desc = ptx::desc_kmajor_sw128(ptx::smem_u32(sB + (n0 / 2) * 128));
        const uint64_t sfadesc = ptx::desc_sf_atom(ptx::smem_u32(sSFA));
        const uint64_t sfbdesc = ptx::desc_sf_atom(ptx::smem_u32(sSFB));
        const uint32_t idesc0 = ptx::idesc_nvf4((uint32_t)n0, 256);
        const uint32_t idesc1 = ptx::idesc_nvf4((uint32_t)(TWO ? n1 : 64), 256);
        const uint32_t sfa_t = tmem + kTmemSfa, sfb_t = tmem + kTmemSfb;
        for (int it = 0; it < stages; ++it) {
            if (ptx::elect_one()) {
                // Like the GEMM: each k-block's scale copies right before its MMAs.
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (it == 0 || sf_copies) {
                        ptx::tc_cp_32x128b_warpx4_pair(sfa_t + 4 * j, sfadesc + (uint64_t)((j * kAtom) >> 4));
#pragma unroll
                        for (int r = 0; r < kMaxSfbAtoms; ++r)
                            if (it == 0 || r < SFB)  // the first stage fills every scale column the MMAs read
                                ptx::tc_cp_32x128b_warpx4_pair(sfb_t + j * 4 * kMaxSfbAtoms + 4 * r,
                                                               sfbdesc + (uint64_t)(((r * 4 + j) * kAtom) >> 4));
                    }
                    const uint32_t koff = (uint32_t)((32 * j) >> 4);
                    const uint32_t acc_flag = (it | j) ? 1u : 0u;
                    ptx::tc_mma_nvf4_pair(tmem, adesc + koff, bdesc + koff, idesc0, sfa_t + 4 * j,
                                          sfb_t + j * 4 * kMaxSfbAtoms, acc_flag);
                    if (TWO)
                        ptx::tc_mma_nvf4_pair(tmem + (uint32_t)n0, adesc + koff, b1desc + koff, idesc1,
                                              sfa_t + 4 * j, sfb_t + j * 4 * kMaxSfbAtoms + (uint32_t)n0 / 32,
                                              acc_flag);
                }
            }
            __syncwarp();
        }
        if (ptx::elect_one()) ptx::tc_commit_pair(done, 0x3);  // both CTAs: every MMA of the pair has completed
        __syncwarp();
    }
    if (threadIdx.x == 0 && !ptx::mbar_wait(done, 0) && err) atomicCAS(err, 0, kErrRateTimeout);
    ptx::tc_fence_before();
    ptx::cluster_sync();
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc_pair(tmem, kRateTmemCols);
    }
}

using RateKernel = void (*)(int, int, int, int, int*);

RateKernel rate_kernel(int sfb_atoms, bool two) {
    switch (sfb_atoms * 2 + (two ? 1 : 0)) {
        case 0: return mma_rate_kernel<0, false>;
        case 1: return mma_rate_kernel<0, true>;
        case 2: return mma_rate_kernel<1, false>;
        case 3: return mma_rate_kernel<1, true>;
        case 4: return mma_rate_kernel<2, false>;
        case 5: return mma_rate_kernel<2, true>;
        case 6: return mma_rate_kernel<3, false>;
        default: return mma_rate_kernel<3, true>;
    }
}

bool valid_width(int n) { return n >= 64 && n <= 256 && n % 64 == 0; }

}  // namespace
}  // namespace fp4b

using namespace fp4b;

FP4B_EXPORT int fp4b_mma_rate(int n0, int n1, int sf_copies, int sfb_atoms, int stages, int* pairs_out,
                              void* stream) {
    if (!valid_width(n0) || (n1 != 0 && !valid_width(n1)) || n0 + n1 > 384 || sfb_atoms < 0 ||
        sfb_atoms > kMaxSfbAtoms || stages <= 0 || stages > kMaxRateStages) {
        set_last_error("fp4b_mma_rate: n0, n1 multiples of 64 in [64, 256] (n1 may be 0) with n0 + n1 <= 384, "
                       "sfb_atoms 0..3, 0 < stages <= %d", kMaxRateStages);
        return -1;
    }
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int smem = kRateSmemBytes;
    const RateKernel kernel = rate_kernel(sfb_atoms, n1 > 0);
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return launch_status(cudaGetLastError(), "fp4b_mma_rate: shared memory attribute");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(kRateThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    int pairs = 0;
    if (cudaOccupancyMaxActiveClusters(&pairs, (const void*)kernel, &cfg) != cudaSuccess || pairs <= 0) {
        cudaGetLastError();
        pairs = sms / 2;
    }
    if (pairs > sms / 2) pairs = sms / 2;
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    int* err = device_error_word();
    if (pairs_out) *pairs_out = pairs;
    return launch_status(cudaLaunchKernelEx(&cfg, kernel, n0, n1, sf_copies, stages, err),
                         "fp4b_mma_rate launch");
}
