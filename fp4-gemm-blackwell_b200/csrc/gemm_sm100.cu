// gemm_sm100.cu -- NVFP4 x NVFP4 -> BF16 block-scaled GEMM on sm_100a tcgen05.
//
// Replaces the CUTLASS SM120 GemmUniversal of fp4_gemm_lib.cu:41-100 / 540-580
// / 794-834:  D = alpha * (A*SFA)(B*SFB)^T + beta * C, fp32 accumulate, BF16
// out, A [M, K] and B [N, K] both K-major packed E2M1, scales UE4M3 per 16
// elements in the 128x4 interleaved layout (the layout tcgen05 wants, so the
// scale bytes are copied to tensor memory as they are).
//
// One CTA computes a 128 x BN tile, 192 threads in three roles:
//   warp 0     TMA producer: per 256-wide K stage, one 2-D TMA (128B swizzle)
//              for the A tile and one for the B tile, plus 1-D bulk copies of
//              the contiguous 512-byte scale atoms, all completing on the
//              stage's `full` mbarrier;
//   warp 1     allocates TMEM and, from one elected lane, issues tcgen05.cp of
//              the scale atoms into TMEM and four
//              tcgen05.mma.kind::mxf4nvf4.block_scale.block16 (K = 64 each)
//              per stage; tcgen05.commit frees the stage's smem;
//   warps 2-5  epilogue: tcgen05.ld the fp32 accumulator (one row per
//              thread), alpha/beta/C, BF16, optional bias, 16-byte stores.
// No TMA multicast anywhere (the library also runs on multi-GPU nodes).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"
#include "ptx_sm100.cuh"

namespace fp4b {

namespace {

constexpr int kBM = 128;            // rows of A per tile (one tcgen05 M)
constexpr int kStageKBytes = 128;   // K bytes per stage and row (256 FP4 elements)
constexpr int kKbPerStage = 4;      // 64-element MMA k-blocks per stage
constexpr int kAtomBytes = 512;     // 128 rows x 4 scale bytes
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemSfaCol = 256;
constexpr uint32_t kTmemSfbCol = kTmemSfaCol + 4 * kKbPerStage;

// Largest number of 128-row scale tiles one BN-wide tile can touch when tiles
// start at multiples of BN (all starts are multiples of 32).
constexpr int max_row_tiles(int bn) {
    int best = 0;
    for (int t = 0; t < 128; ++t) {
        const int off = (t * bn) % 128;
        const int n = (off + bn + 127) / 128;
        if (n > best) best = n;
    }
    return best;
}

// Tile widths are multiples of 64, so every tile starts 0 or 64 rows into a
// 128-row scale atom and the MMA's scale-B TMEM address moves by 0 or 2
// columns.  An odd column (a tile starting 32 or 96 rows into an atom, e.g.
// BN = 160) raised a misaligned-address error on B200.
template <int BN, int STAGES>
struct Cfg {
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 64 in [64, 256]");
    static constexpr int NRT = max_row_tiles(BN);
    static constexpr int A_BYTES = kBM * kStageKBytes;
    static constexpr int B_BYTES = BN * kStageKBytes;
    static constexpr int SFA_BYTES = kKbPerStage * kAtomBytes;
    static constexpr int SFB_BYTES = NRT * kKbPerStage * kAtomBytes;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
    static_assert(kTmemSfbCol + kKbPerStage * 4 * NRT <= kTmemCols, "TMEM budget exceeded");
    static_assert(BN <= (int)kTmemSfaCol, "accumulator overlaps the scale columns");
};

struct Params {
    const uint8_t* a_sf;
    const uint8_t* b_sf;
    const __nv_bfloat16* c;
    __nv_bfloat16* d;
    const __nv_bfloat16* bias;
    int* err;
    int m, n_out, num_kb;  // num_kb = k_pad / 64
    int n_rows_pad;
    long ldc, ldd;
    float alpha, beta;
    int vec_store;  // D/C rows 16-byte aligned
};

// Error codes written to the device error word.
constexpr int kErrProducerTimeout = 1;
constexpr int kErrMmaTimeout = 2;
constexpr int kErrEpilogueTimeout = 3;

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    nvf4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ Params p) {
    using C = Cfg<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * C::A_BYTES;
    uint8_t* sSFA = sB + STAGES * C::B_BYTES;
    uint8_t* sSFB = sSFA + STAGES * C::SFA_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * C::SFB_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
    int* s_last_issued = s_abort + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * kBM;
    const int num_kb = p.num_kb;
    const int num_ks = (num_kb + kKbPerStage - 1) / kKbPerStage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(acc_full, 1);
        *s_abort = 0;
        *s_last_issued = -1;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Scale row tiles covering B rows [n0, n0 + BN), clipped to the buffer.
    const int rt0 = n0 >> 7;
    const int shift_words = (n0 & 127) >> 5;
    int nrt = ((n0 & 127) + BN + 127) >> 7;
    if (rt0 + nrt > (p.n_rows_pad >> 7)) nrt = (p.n_rows_pad >> 7) - rt0;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (ptx::elect_one()) {
            const uint8_t* sfa_tile = p.a_sf + (size_t)blockIdx.y * kAtomBytes * num_kb;
            for (int ks = 0; ks < num_ks; ++ks) {
                const int s = ks % STAGES;
                if (ks >= STAGES && !ptx::mbar_wait(&empty[s], ((ks / STAGES) & 1) ^ 1)) {
                    record_error(p.err, kErrProducerTimeout);
                    atomicExch(s_abort, 1);
                    break;
                }
                if (*reinterpret_cast<volatile int*>(s_abort)) break;
                const int kb0 = ks * kKbPerStage;
                const int nkb = min(kKbPerStage, num_kb - kb0);
                const uint32_t sf_bytes = (uint32_t)nkb * kAtomBytes;
                ptx::mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES + sf_bytes * (1 + nrt));
                ptx::tma_load_2d(sA + s * C::A_BYTES, &tmap_a, &full[s], ks * kStageKBytes, m0);
                ptx::tma_load_2d(sB + s * C::B_BYTES, &tmap_b, &full[s], ks * kStageKBytes, n0);
                ptx::bulk_load(sSFA + s * C::SFA_BYTES, sfa_tile + (size_t)kb0 * kAtomBytes, sf_bytes, &full[s]);
                for (int j = 0; j < nrt; ++j) {
                    const uint8_t* src = p.b_sf + ((size_t)(rt0 + j) * num_kb + kb0) * kAtomBytes;
                    ptx::bulk_load(sSFB + s * C::SFB_BYTES + j * kKbPerStage * kAtomBytes, src, sf_bytes, &full[s]);
                }
                *s_last_issued = ks;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (ptx::elect_one()) {
            constexpr uint32_t idesc = ptx::idesc_nvf4(BN);
            const uint32_t a_base = ptx::smem_u32(sA), b_base = ptx::smem_u32(sB);
            const uint32_t sfa_base = ptx::smem_u32(sSFA), sfb_base = ptx::smem_u32(sSFB);
            for (int ks = 0; ks < num_ks; ++ks) {
                const int s = ks % STAGES;
                if (!ptx::mbar_wait(&full[s], (ks / STAGES) & 1)) {
                    record_error(p.err, kErrMmaTimeout);
                    atomicExch(s_abort, 1);
                    break;
                }
                ptx::tc_fence_after();
                const int nkb = min(kKbPerStage, num_kb - ks * kKbPerStage);
                for (int j = 0; j < nkb; ++j) {
                    ptx::tc_cp_32x128b_warpx4(tmem + kTmemSfaCol + 4 * j,
                                              ptx::desc_sf_atom(sfa_base + s * C::SFA_BYTES + j * kAtomBytes));
                    for (int t = 0; t < nrt; ++t)
                        ptx::tc_cp_32x128b_warpx4(
                            tmem + kTmemSfbCol + j * 4 * C::NRT + 4 * t,
                            ptx::desc_sf_atom(sfb_base + s * C::SFB_BYTES + (t * kKbPerStage + j) * kAtomBytes));
                }
                for (int j = 0; j < nkb; ++j) {
                    const uint64_t adesc = ptx::desc_kmajor_sw128(a_base + s * C::A_BYTES + 32 * j);
                    const uint64_t bdesc = ptx::desc_kmajor_sw128(b_base + s * C::B_BYTES + 32 * j);
                    ptx::tc_mma_nvf4(tmem, adesc, bdesc, idesc, tmem + kTmemSfaCol + 4 * j,
                                     tmem + kTmemSfbCol + j * 4 * C::NRT + shift_words, (ks | j) != 0);
                }
                ptx::tc_commit(&empty[s]);
            }
            ptx::tc_commit(acc_full);  // also on abort: completes once issued MMAs are done
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may read
        const int row = q * 32 + lane;
        const int m = m0 + row;
        const bool ok = ptx::mbar_wait(acc_full, 0);
        if (!ok) record_error(p.err, kErrEpilogueTimeout);
        ptx::tc_fence_after();
        const bool aborted = !ok || *reinterpret_cast<volatile int*>(s_abort);
        if (!aborted) {
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + 32 * c, r);
                ptx::tmem_ld_wait();
                const int nb = n0 + 32 * c;
                if (m >= p.m || nb >= p.n_out) continue;
                __nv_bfloat16* drow = p.d + (size_t)m * p.ldd;
                const __nv_bfloat16* crow = p.c ? p.c + (size_t)m * p.ldc : nullptr;
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int n = nb + 8 * g;
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = p.alpha * __uint_as_float(r[8 * g + i]);
                    const bool full8 = p.vec_store && n + 8 <= p.n_out;
                    if (p.beta != 0.0f && crow) {
                        if (full8) {
                            const uint4 cv = *reinterpret_cast<const uint4*>(crow + n);
                            const __nv_bfloat16* cb = reinterpret_cast<const __nv_bfloat16*>(&cv);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                v[i] = fmaf(p.alpha, __uint_as_float(r[8 * g + i]), p.beta * __bfloat162float(cb[i]));
                        } else {
                            for (int i = 0; i < 8 && n + i < p.n_out; ++i)
                                v[i] = fmaf(p.alpha, __uint_as_float(r[8 * g + i]), p.beta * __bfloat162float(crow[n + i]));
                        }
                    }
                    if (p.bias) {
                        // Reference order: BF16 GEMM output, then a BF16 bias add.
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float b = (n + i < p.n_out) ? __bfloat162float(p.bias[n + i]) : 0.0f;
                            v[i] = __bfloat162float(__float2bfloat16_rn(v[i])) + b;
                        }
                    }
                    if (full8) {
                        uint4 o;
                        o.x = bf16x2_bits(v[0], v[1]);
                        o.y = bf16x2_bits(v[2], v[3]);
                        o.z = bf16x2_bits(v[4], v[5]);
                        o.w = bf16x2_bits(v[6], v[7]);
                        *reinterpret_cast<uint4*>(drow + n) = o;
                    } else {
                        for (int i = 0; i < 8 && n + i < p.n_out; ++i) drow[n + i] = __float2bfloat16_rn(v[i]);
                    }
                }
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(s_abort)) {
        // Let every copy already issued land before the CTA's smem goes away.
        const int last = *s_last_issued;
        for (int ks = (last - STAGES + 1 > 0 ? last - STAGES + 1 : 0); ks <= last; ++ks)
            ptx::mbar_wait(&full[ks % STAGES], (ks / STAGES) & 1);
        ptx::mbar_wait(acc_full, 0);
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// Packed FP4 operand [rows, k_pad/2] bytes, 128-byte x box_rows boxes, 128B swizzle.
bool make_operand_map(CUtensorMap* map, const void* base, long rows, long k_pad, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(k_pad / 2), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(k_pad / 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kStageKBytes, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int STAGES>
cudaError_t launch_tile(const GemmArgs& g, cudaStream_t stream, int sms) {
    using C = Cfg<BN, STAGES>;
    auto kernel = nvf4_gemm_kernel<BN, STAGES>;
    static std::once_flag attr_once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 63], [&] {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    CUtensorMap ma, mb;
    if (!make_operand_map(&ma, g.a_fp4, g.m_rows_pad, g.k_pad, kBM) ||
        !make_operand_map(&mb, g.b_fp4, g.n_rows_pad, g.k_pad, BN))
        return cudaErrorInvalidValue;
    Params p{};
    p.a_sf = g.a_sf;
    p.b_sf = g.b_sf;
    p.c = static_cast<const __nv_bfloat16*>(g.c);
    p.d = static_cast<__nv_bfloat16*>(g.d);
    p.bias = static_cast<const __nv_bfloat16*>(g.bias);
    p.err = device_error_word();
    p.m = (int)g.m;
    p.n_out = (int)g.n_out;
    p.num_kb = (int)(g.k_pad / 64);
    p.n_rows_pad = (int)g.n_rows_pad;
    p.ldc = g.ldc;
    p.ldd = g.ldd;
    p.alpha = g.alpha;
    p.beta = g.beta;
    const bool d_al = (reinterpret_cast<uintptr_t>(g.d) & 15) == 0 && g.ldd % 8 == 0;
    const bool c_al = !g.c || ((reinterpret_cast<uintptr_t>(g.c) & 15) == 0 && g.ldc % 8 == 0);
    p.vec_store = (d_al && c_al) ? 1 : 0;
    (void)sms;
    dim3 grid((unsigned)((g.n_out + BN - 1) / BN), (unsigned)((g.m + kBM - 1) / kBM));
    kernel<<<grid, kThreads, C::SMEM_BYTES, stream>>>(ma, mb, p);
    return cudaGetLastError();
}

// Pick the tile width that minimises (waves x BN) on this device.
int choose_bn(long m, long n, int sms) {
    static const int cands[] = {256, 192, 128};
    const long mt = (m + kBM - 1) / kBM;
    int best = 128;
    long best_cost = -1;
    for (int bn : cands) {
        const long tiles = mt * ((n + bn - 1) / bn);
        const long waves = (tiles + sms - 1) / sms;
        const long cost = waves * bn;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

}  // namespace

const char* gemm_check(const GemmArgs& g) {
    if (!g.a_fp4 || !g.a_sf || !g.b_fp4 || !g.b_sf || !g.d) return "null pointer";
    if (g.m <= 0 || g.n_out <= 0) return "empty problem";
    if (g.k_pad <= 0 || g.k_pad % 128) return "K must be a positive multiple of 128";
    if (g.m_rows_pad % 128 || g.n_rows_pad % 128) return "operand rows must be padded to multiples of 128";
    if (g.m > g.m_rows_pad || g.n_out > g.n_rows_pad) return "output larger than the operands";
    if (g.ldd < g.n_out || (g.c && g.ldc < g.n_out)) return "row stride smaller than N";
    if ((reinterpret_cast<uintptr_t>(g.a_fp4) | reinterpret_cast<uintptr_t>(g.b_fp4) |
         reinterpret_cast<uintptr_t>(g.a_sf) | reinterpret_cast<uintptr_t>(g.b_sf)) & 15)
        return "operand buffers must be 16-byte aligned";
    if (g.m_rows_pad >= (1l << 31) || g.n_rows_pad >= (1l << 31)) return "operand too large";
    return nullptr;
}

cudaError_t gemm_launch(const GemmArgs& g, cudaStream_t stream) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const char* force = getenv("FP4B_FORCE_BN");
    const int bn = force ? atoi(force) : choose_bn(g.m, g.n_out, sms);
    switch (bn) {
        case 256: return launch_tile<256, 4>(g, stream, sms);
        case 192: return launch_tile<192, 4>(g, stream, sms);
        case 128: return launch_tile<128, 6>(g, stream, sms);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace fp4b
