// quantize_units.cu -- the activation quantizer that runs beside the GEMM.
//
// In the overlapped cached linear the activation quantizer and the CTA-pair
// GEMM run at the same time on the same SMs: this kernel is launched first,
// one small CTA per SM, and the GEMM is launched right behind it with
// programmatic stream serialization, so that its CTAs take the rest of every
// SM.  The two use different parts of the machine -- the quantizer issue slots
// and HBM, the GEMM the tensor pipe and the L2 -> SM path -- and the GEMM's A
// producers wait for the units of A they need instead of for this whole grid.
//
// The same bytes as the standalone quantizer (quantize.cu, the reference's
// semantics): only the order of the work and the staging differ.  The padded
// rows of A are cut into units of 64 rows x one 256-wide K-stage, ordered
// K-stage by K-stage (unit u: K-stage u / R of the 64-row group u % R, R =
// rows_pad / 64); CTA c quantizes units c, c + G, c + 2G, ...  Per CTA:
//   warp 0      producer: each unit is four 16-row x 256-column slices (8 KB
//               of BF16), brought into a ring of shared-memory stages by 2-D
//               TMA loads (positions past the tensor read as zeros, which is
//               the reference's zero padding);
//   warps 1-4   consumers: two 16-element blocks per lane and slice, written
//               as packed E2M1 codes and UE4M3 scales to the operand buffers;
//   warp 5      publisher: after each unit (a named barrier with the
//               consumers) it fences and adds one to the counter of the
//               unit's 128-row tile and K-stage, ready[(g / 2) * stages + ks];
//               it has no loads or stores of its own in flight, so its fence
//               waits only for the consumers' stores.
// The GEMM waits (bounded) until a counter reaches 2 before loading that part
// of A and zeroes the counters when it finishes.  Every ring wait is bounded
// (ptx::mbar_wait); a timeout records kErrQuantUnitsTimeout.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"
#include "ptx_sm100.cuh"
#include "quantize_core.cuh"

namespace fp4b {
namespace {

using namespace qcore;

constexpr int kUnitRows = 64;
constexpr int kSliceRows = 16;                        // rows of one ring stage
constexpr int kSliceBytes = kSliceRows * 256 * 2;     // 8 KB of BF16
constexpr int kUnitThreads = 192;
constexpr int kConsumerWarps = 4;
constexpr uint32_t kUnitBarrier = 1;                  // consumers + publisher
constexpr int kErrQuantUnitsTimeout = 6;              // device error word
constexpr uint64_t kUnitsDrainNs = 200000;

__device__ __forceinline__ void tma_load_2d_local(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    ptx::tma_load_2d(dst, map, bar, x, y);
}

// Dynamic shared memory: `ring` stages of 8 KB, the tables, the barriers.
__global__ void __launch_bounds__(kUnitThreads, 5)
    nvfp4_quantize_units_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ QuantParams p,
                                const QuantTables* qtab, uint32_t* ready, int groups, int stages, int ring,
                                int* err) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* s_ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* s_tables = s_ring + (size_t)ring * kSliceBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(s_tables + kSmemTableBytes);
    uint64_t* empty = full + ring;
    int* s_abort = reinterpret_cast<int*>(empty + ring);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t R = (uint32_t)groups, U = R * (uint32_t)stages, G = gridDim.x;
    if (threadIdx.x == 0) {
        for (int i = 0; i < ring; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], kConsumerWarps);
        }
        *s_abort = 0;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tmap_x);
    }
    const SmemTables tab = copy_tables(qtab, s_tables, threadIdx.x, kUnitThreads);
    __syncthreads();
    // The previous kernel on the stream (e.g. the previous GEMM, which may still
    // read the operand buffers written here) completes before anything here
    // touches global memory; only then may the GEMM behind this kernel start.
    ptx::grid_dependency_wait();
    ptx::launch_dependents();

    bool timed_out = false;
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t k = 0;
            for (uint32_t u = blockIdx.x; u < U && !timed_out; u += G) {
                const uint32_t ks = u / R, grp = u - ks * R;
                for (int j = 0; j < kUnitRows / kSliceRows; ++j, ++k) {
                    const uint32_t s = k % (uint32_t)ring;
                    if (k >= (uint32_t)ring && !ptx::mbar_wait(&empty[s], ((k / ring) - 1) & 1)) {
                        timed_out = true;
                        break;
                    }
                    if (*reinterpret_cast<volatile int*>(s_abort)) {
                        timed_out = true;
                        break;
                    }
                    ptx::mbar_arrive_expect_tx(&full[s], kSliceBytes);
                    tma_load_2d_local(s_ring + (size_t)s * kSliceBytes, &tmap_x, &full[s], (int)(ks * 256),
                                      (int)(grp * kUnitRows + j * kSliceRows));
                }
            }
        }
    } else if (warp <= kConsumerWarps) {
        // ------------------------------------------------------------ consumers
        const uint32_t cl = threadIdx.x - 32;  // 0..127
        uint32_t k = 0;
        for (uint32_t u = blockIdx.x; u < U; u += G) {
            const uint32_t ks = u / R, grp = u - ks * R;
            for (int j = 0; j < kUnitRows / kSliceRows; ++j, ++k) {
                const uint32_t s = k % (uint32_t)ring;
                const bool ok = !timed_out && __all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (k / ring) & 1));
                if (!ok) timed_out = true;
                uint32_t w[2][8];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (ok) {
                        // Block b of the slice: row b / 16, block b % 16 of the K-stage;
                        // a warp reads 1 KB of contiguous shared memory per half.
                        const uint4* src = reinterpret_cast<const uint4*>(s_ring + (size_t)s * kSliceBytes +
                                                                          (cl + 128u * h) * 32u);
                        const uint4 v0 = src[0], v1 = src[1];
                        w[h][0] = v0.x; w[h][1] = v0.y; w[h][2] = v0.z; w[h][3] = v0.w;
                        w[h][4] = v1.x; w[h][5] = v1.y; w[h][6] = v1.z; w[h][7] = v1.w;
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) w[h][i] = 0u;
                    }
                }
                if (ok) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t b = cl + 128u * h;
                        const uint32_t r = grp * kUnitRows + (uint32_t)j * kSliceRows + (b >> 4);
                        const uint32_t kb = ks * 16u + (b & 15u);
                        quantize_and_store(p, r * p.nsb + kb, kb < p.nsb ? p.total : 0u, w[h], r, kb,
                                           (uint32_t)lane, tab);
                    }
                    // The stage's bytes were consumed above (the stores depend on them).
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&empty[s]);
                }
            }
            __syncwarp();
            ptx::named_barrier(kUnitBarrier, (kConsumerWarps + 1) * 32);  // the unit's stores are issued
        }
    } else {
        // ------------------------------------------------------------ publisher
        for (uint32_t u = blockIdx.x; u < U; u += G) {
            ptx::named_barrier(kUnitBarrier, (kConsumerWarps + 1) * 32);
            if (lane == 0) {
                const uint32_t ks = u / R, grp = u - ks * R;
                ptx::fence_proxy_async_global();  // the GEMM reads these bytes with TMA
                __threadfence();
                atomicAdd(ready + (grp >> 1) * (uint32_t)stages + ks, 1u);
            }
            __syncwarp();
        }
    }
    if (timed_out) {
        if (err) atomicCAS(err, 0, kErrQuantUnitsTimeout);
        atomicExch(s_abort, 1);
    }
    __syncthreads();
    if (*reinterpret_cast<volatile int*>(s_abort)) {
        // Copies issued before the timeout still land in this CTA's shared memory.
        const uint64_t t0 = ptx::global_timer_ns();
        while (ptx::global_timer_ns() - t0 < kUnitsDrainNs) {
        }
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

}  // namespace

int quantize_units_smem_bytes(int ring) { return ring * kSliceBytes + kSmemTableBytes + ring * 16 + 16 + 128; }

const char* quantize_units_check(const QuantizeArgs& a) {
    if (const char* why = quantize_check(a)) return why;
    if ((reinterpret_cast<uintptr_t>(a.src) & 15) || (a.ld % 8) || a.rows < 1 || a.cols < 1)
        return "overlapped quantizer: rows must be 16-byte aligned";
    if (a.rows_pad % kUnitRows) return "overlapped quantizer: padded rows must be a multiple of 64";
    return nullptr;
}

cudaError_t quantize_units_launch(const QuantizeArgs& a, uint32_t* ready, int ring, int grid, cudaStream_t stream) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc || ring < 2 || grid < 1) return cudaErrorInvalidValue;
    CUtensorMap map;
    memset(&map, 0, sizeof(map));
    const cuuint64_t dims[2] = {(cuuint64_t)a.cols, (cuuint64_t)a.rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(a.ld * 2)};
    const cuuint32_t box[2] = {256, (cuuint32_t)kSliceRows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.src), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    const QuantParams p = make_quant_params(a);
    const QuantTables* qtab = quant_tables_device();
    const int smem = quantize_units_smem_bytes(ring);
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [&] {
        cudaFuncSetAttribute(nvfp4_quantize_units_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        // The SMs this kernel runs on keep the largest shared-memory partition,
        // so that the GEMM's CTAs (which need it) can be placed beside it.
        cudaFuncSetAttribute(nvfp4_quantize_units_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    });
    if (smem > 96 * 1024) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kUnitThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!qtab) return cudaErrorInvalidValue;
    return cudaLaunchKernelEx(&cfg, nvfp4_quantize_units_kernel, map, p, qtab, ready, (int)(a.rows_pad / kUnitRows),
                              (int)((a.k_pad + 255) / 256), ring, device_error_word());
}

}  // namespace fp4b
