// gemm_sm100.cu -- NVFP4 x NVFP4 -> BF16 block-scaled GEMM on sm_100a tcgen05.
//
// Replaces the CUTLASS SM120 GemmUniversal of fp4_gemm_lib.cu:41-100 / 540-580
// / 794-834:  D = alpha * (A*SFA)(B*SFB)^T + beta * C, fp32 accumulate, BF16
// out, A [M, K] and B [N, K] both K-major packed E2M1, scales UE4M3 per 16
// elements in the 128x4 interleaved layout (the layout tcgen05 wants, so the
// scale bytes are copied to tensor memory as they are).
//
// Two persistent kernels.  When A has more than 128 rows, CTA pairs (clusters
// of two, tcgen05 cta_group::2) walk 256 x BN tiles; see the pair kernel
// below.  Otherwise (and on request) one CTA per SM walks 128 x BN output
// tiles with 192 threads in three roles:
//   warp 0     TMA producer.  A stage covers K = 512: two 128-byte-wide TMA
//              boxes (128B swizzle) for A, two for B, one bulk copy of the A
//              scale atoms and one per 128-row tile of B scales, all
//              completing on the stage's `full` mbarrier.  A copy completes
//              one at a time per issuing thread (~0.4 us each from L2), so the
//              copies of a stage go out from different lanes, and consecutive
//              stages use different lanes.
//   warp 1     allocates TMEM and walks the same loop converged; one elected
//              lane issues per stage the tcgen05.cp of the scale atoms and
//              eight tcgen05.mma.kind::mxf4nvf4.block_scale.block16 (K = 64
//              each), then tcgen05.commit frees the stage.  Issuing from a
//              converged warp with unrolled, predicated k-block loops keeps
//              the tensor pipe fed; issuing from a lone diverged thread was
//              several times slower on B200.
//   warps 2-5  epilogue: tcgen05.ld the fp32 accumulator (one row per thread),
//              alpha/beta/C, BF16, optional bias, 16-byte stores.  Two TMEM
//              accumulators (when they fit) let the epilogue of one tile run
//              under the MMAs of the next.
// No TMA multicast anywhere (the library also runs on multi-GPU nodes).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "fp4b_internal.h"
#include "nvfp4_codec.cuh"
#include "ptx_sm100.cuh"
#include "quantize_core.cuh"

namespace fp4b {

namespace {

constexpr int kBM = 128;            // rows of A per tile (one tcgen05 M)
constexpr int kChunkBytes = 128;    // one 128B-swizzle atom row: 256 FP4 elements of K
constexpr int kAtomBytes = 512;     // 128 rows x 4 scale bytes
constexpr int kThreads = 192;
constexpr int kEpilogueWarps = 4;
constexpr uint32_t kTmemCols = 512;

// Largest number of 128-row scale tiles one BN-wide tile can touch when tiles
// start at multiples of BN (starts are multiples of 64, see Cfg).
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
template <int BN, int STAGES, int CHUNKS>
struct Cfg {
    // CHUNKS 128-byte-wide chunks of K per stage: a stage covers K = 256 * CHUNKS.
    static constexpr int kChunks = CHUNKS;
    static constexpr int kStageKBytes = CHUNKS * kChunkBytes;
    static constexpr int kKbPerStage = 4 * CHUNKS;  // 64-element MMA k-blocks per stage
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 64 in [64, 256]");
    static constexpr int NRT = max_row_tiles(BN);
    static constexpr int A_CHUNK = kBM * kChunkBytes;   // one TMA box
    static constexpr int B_CHUNK = BN * kChunkBytes;
    static constexpr int A_BYTES = kChunks * A_CHUNK;
    static constexpr int B_BYTES = kChunks * B_CHUNK;
    static constexpr int SFA_BYTES = kKbPerStage * kAtomBytes;
    static constexpr int SFB_BYTES = NRT * kKbPerStage * kAtomBytes;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    // TMEM columns: ACC_BUFS accumulators of BN fp32 columns, then the scales
    // of one stage (4 k-blocks x 4 columns for A, 4 x 4*NRT for B).
    static constexpr int SF_COLS = 4 * kKbPerStage * (1 + NRT);
    static constexpr int ACC_BUFS = (2 * BN + SF_COLS <= (int)kTmemCols) ? 2 : 1;
    static constexpr uint32_t TMEM_SFA = ACC_BUFS * BN;
    static constexpr uint32_t TMEM_SFB = TMEM_SFA + 4 * kKbPerStage;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
    static_assert(TMEM_SFA + SF_COLS <= kTmemCols, "TMEM budget exceeded");
};

constexpr int kMaxPeers = 7;

struct Params {
    const uint8_t* a_sf;
    const uint8_t* b_sf;
    const __nv_bfloat16* c;
    __nv_bfloat16* d;
    const __nv_bfloat16* bias;
    int* err;
    int m, n_out, num_kb;  // num_kb = k_pad / 64
    int n_rows_pad;
    int n_tiles, num_tiles;
    int m_tiles;  // row tiles of the output (128 rows, or 256 for CTA pairs)
    long ldc, ldd;
    float alpha, beta;
    int vec_store;  // D/C rows 16-byte aligned
    int tma_store;  // D written by TMA from shared memory (C unused, D rows 16-byte aligned)
    int bias_vec;   // bias 16-byte aligned: read 8 values per load
    int b_early;    // B and its scales do not depend on the preceding kernel: load them before its completion
    // Await mode (pair kernel, AWAIT): [a_tiles128][a_stages] units of A
    // quantized per 128-row tile and K-stage (published by the quantizer running
    // beside this kernel), then one CTA-exit counter (ready_count words before it).
    uint32_t* ready;
    int a_tiles128, a_stages, ready_count;
    // Column-parallel output (pair kernel, TMA-store epilogue): every tile is
    // also written to npeers other [m, ldd] BF16 buffers (other GPUs' memory
    // mapped into this process), each already offset to this rank's columns;
    // their tensor maps are the kernel's PeerMaps argument.
    int npeers;
};

// Output tensor maps of the peer buffers (column-parallel mode; 16 x 64
// boxes like the local pieces); all zero and unused otherwise.
struct PeerMaps {
    CUtensorMap map[kMaxPeers];
};

// Tile t -> (row tile, column tile) in groups of kTileGroupRows rows of A: the
// tiles in flight at one time cover a few row tiles and a few column tiles,
// so the A and B tiles they read stay in L2 even when B is larger than L2
// (the group's row tiles are revisited for every column tile of B).
constexpr int kTileGroupRows = 2048;

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int tile_m, int& m_tile, int& n_tile) {
    const int group = kTileGroupRows / tile_m;
    const int per_group = group * n_tiles;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(group, m_tiles - first_m);
    const int local = t - g * per_group;
    m_tile = first_m + local % gm;
    n_tile = local / gm;
}

// Error codes written to the device error word.
constexpr int kErrProducerTimeout = 1;
constexpr int kErrMmaTimeout = 2;
constexpr int kErrEpilogueTimeout = 3;
constexpr int kErrQuantizeWaitTimeout = 4;

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ bool aborted(const int* flag) { return *reinterpret_cast<const volatile int*>(flag) != 0; }

// Epilogue of one 32-column chunk for one output row: alpha*acc (+beta*C),
// BF16, (+bias in BF16), 16-byte stores.
__device__ __forceinline__ void store_chunk(const Params& p, const uint32_t (&r)[32], int m, int nb) {
    __nv_bfloat16* drow = p.d + (size_t)m * p.ldd;
    const __nv_bfloat16* crow = p.c ? p.c + (size_t)m * p.ldc : nullptr;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int n = nb + 8 * g;
        if (n >= p.n_out) break;
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

// Copies bias[n0, n0 + bn) into `dst` as BF16, 8 per uint4 (zeros past N),
// with the lanes of one warp, so the epilogue reads it from shared memory.
__device__ __forceinline__ void stage_bias(const Params& p, uint4* dst, int n0, int bn, int lane) {
    for (int i = lane; i < bn / 8; i += 32) {
        const int nb = n0 + 8 * i;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (p.bias_vec && nb + 8 <= p.n_out) {
            v = __ldg(reinterpret_cast<const uint4*>(p.bias + nb));
        } else {
            __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&v);
            for (int j = 0; j < 8 && nb + j < p.n_out; ++j) vb[j] = p.bias[nb + j];
        }
        dst[i] = v;
    }
}

// Two BF16 additions, each rounded once from the exact sum.  For BF16 operands
// this equals the reference's bias add (the BF16 values widened to fp32,
// added, rounded to BF16): when their exponents differ by at most 16 the fp32
// sum is exact, and otherwise the smaller operand is below 2^-16 of the larger,
// whose BF16 neighbours are 2^-9 of it or more away, so both roundings return
// the larger operand.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Epilogue of one 32 x 32 chunk through shared memory: thread t converts row
// t (alpha*acc, BF16, optional BF16 bias) into a 2 KB buffer laid out in the
// TMA 64-byte swizzle (16-byte unit u of row r at unit u ^ ((r >> 1) & 3),
// which keeps the 16-byte shared stores of 8 consecutive rows on distinct
// banks), then one lane stores the box [row0, row0 + 32) x [n, n + 32) with
// TMA; rows past M and columns past N are clipped by the tensor map.
// One thread's TMA copies run one after another (~0.4 us each), so chunk i
// is stored by lane i % 32, and the lane that stored the buffer's previous
// contents (chunk i - 1) waits until that store has read it.
// Accumulator chunk (32 fp32 columns of this lane's row) -> 16 packed BF16
// pairs: alpha, BF16, then the BF16 bias add of the reference.
__device__ __forceinline__ void convert_chunk(const Params& p, const uint32_t (&r)[32], const uint4* sbias,
                                              uint32_t (&packed)[16]) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    if (p.alpha != 1.0f) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) packed[i] = bf16x2_bits(v[2 * i], v[2 * i + 1]);
    if (p.bias) {
        // Reference order: BF16 GEMM output, then the BF16 bias add.
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint4 b = sbias[g];
            packed[4 * g + 0] = add_bf16x2(packed[4 * g + 0], b.x);
            packed[4 * g + 1] = add_bf16x2(packed[4 * g + 1], b.y);
            packed[4 * g + 2] = add_bf16x2(packed[4 * g + 2], b.z);
            packed[4 * g + 3] = add_bf16x2(packed[4 * g + 3], b.w);
        }
    }
}

// Epilogue of one 32 x 32 chunk through shared memory (the single-GPU form):
// thread t's converted row goes into the warp's 2 KB buffer in the TMA 64-byte
// swizzle (16-byte unit u of row r at unit u ^ ((r >> 1) & 3), which keeps the
// 16-byte shared stores of 8 consecutive rows on distinct banks), then one
// lane stores the box [row0, row0 + 32) x [n, n + 32) with TMA; rows past M
// and columns past N are clipped by the tensor map.  One thread's TMA copies
// run one after another (~0.4 us each), so chunk i is stored by lane i % 32,
// and the lane that stored the buffer's previous contents (chunk i - 1) first
// waits until that store has read it.  `fresh`: the buffer has not been used
// since the operand ring went idle, so no earlier store can still read it.
__device__ __forceinline__ void store_staged_chunk(const CUtensorMap* tmap_d, const uint32_t (&packed)[16],
                                                   uint8_t* buf, int row0, int n, int lane, int chunk_iter,
                                                   bool fresh = false) {
    if (!fresh && lane == ((chunk_iter - 1) & 31)) ptx::bulk_wait_group_read<0>();
    __syncwarp();
    uint8_t* row = buf + 64 * lane;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(row + 16 * (u ^ sw)) =
            make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == (chunk_iter & 31)) {
        ptx::tma_store_2d(tmap_d, buf, n, row0);
        ptx::bulk_commit_group();
    }
}

// Stores a 16 x 64 piece of the output: rows [row0, row0 + 16) (held by lanes
// 16 half .. 16 half + 15) of two adjacent converted 32-column chunks (lo:
// columns [n, n + 32), hi: [n + 32, n + 64)).  The rows go into the warp's
// 2 KB buffer in the TMA 128-byte swizzle (16-byte unit u of row r at unit
// u ^ (r & 7): 8 consecutive rows on distinct banks), then one lane stores
// the box locally and into every peer's buffer (the column-parallel form).  A
// piece has 128-byte rows: SM-issued stores into another GPU's memory reach
// ~640 GB/s in each
// direction at once with rows of 128 bytes or more, ~430 GB/s with 64-byte
// rows (measured on B200, two GPUs).  One thread's TMA copies run one after
// another (~0.4 us each), so piece i is stored by lane i % 32, and the lane
// that stored the buffer's previous contents (piece i - 1) first waits until
// that store has read it.
__device__ __forceinline__ void store_piece(const Params& p, const CUtensorMap* tmap_d, const PeerMaps* pm,
                                            const uint32_t (&lo)[16], const uint32_t (&hi)[16], uint8_t* buf,
                                            int row0, int n, int half, int lane, int chunk_iter) {
    if (lane == ((chunk_iter - 1) & 31)) ptx::bulk_wait_group_read<0>();
    __syncwarp();
    const unsigned r = (unsigned)(lane - 16 * half);
    if (r < 16u) {
        // Row r starts 128-byte aligned, so unit u ^ (r & 7) of it is at
        // (row + 16 (r & 7)) ^ 16 u: one base register, an XOR per store.
        const uint32_t a = ptx::smem_u32(buf) + 128u * r + 16u * (r & 7u);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            ptx::st_shared_v4(a ^ (16u * u), lo[4 * u], lo[4 * u + 1], lo[4 * u + 2], lo[4 * u + 3]);
            ptx::st_shared_v4(a ^ (16u * (u + 4)), hi[4 * u], hi[4 * u + 1], hi[4 * u + 2], hi[4 * u + 3]);
        }
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == (chunk_iter & 31)) {
        ptx::tma_store_2d(tmap_d, buf, n, row0);
        for (int d = 0; d < p.npeers; ++d) ptx::tma_store_2d(&pm->map[d], buf, n, row0);
        ptx::bulk_commit_group();
    }
}

// Persistent kernel: CTA b processes tiles b, b + gridDim.x, ... (N fastest).
// The smem ring and the TMEM accumulators carry across tiles, so loads of the
// next tile and the epilogue of the previous one overlap the MMAs.
template <int BN, int STAGES, int CHUNKS>
__global__ void __launch_bounds__(kThreads, 1)
    nvf4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ Params p) {
    using C = Cfg<BN, STAGES, CHUNKS>;
    constexpr int TILE_M = kBM;
    constexpr int kChunks = C::kChunks;
    constexpr int kStageKBytes = C::kStageKBytes;
    constexpr int kKbPerStage = C::kKbPerStage;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * C::A_BYTES;
    uint8_t* sSFA = sB + STAGES * C::B_BYTES;
    uint8_t* sSFB = sSFA + STAGES * C::SFA_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * C::SFB_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;     // [2]
    uint64_t* acc_empty = acc_full + 2;      // [2]
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
    int* s_last_issued = s_abort + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_kb = p.num_kb;
    const int num_ks = (num_kb + kKbPerStage - 1) / kKbPerStage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], kEpilogueWarps);
        }
        ptx::mbar_init(mma_done, 1);
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
    // Launched behind the activation quantizer: barriers and TMEM are set up
    // while it finishes; no global memory is touched before this point.
    ptx::grid_dependency_wait();
    // The kernel after this one (the next quantizer) may be scheduled on SMs
    // this grid leaves; it waits for this grid to complete before it reads or
    // writes global memory.
    ptx::launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // A TMA or bulk copy completes one at a time per issuing thread, so the
        // loads of a stage are spread over up to 7 lanes, and consecutive stages
        // use different groups of 8 lanes: 4 stages can be in flight at once.
        int it = 0;
        bool stop = false;
        for (int t = blockIdx.x; t < p.num_tiles && !stop; t += gridDim.x) {
            int m_tile, n_tile;
            tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile, n_tile);
            const int n0 = n_tile * BN;
            const int m0 = m_tile * kBM;
            const int rt0 = n0 >> 7;
            int nrt = ((n0 & 127) + BN + 127) >> 7;
            if (rt0 + nrt > (p.n_rows_pad >> 7)) nrt = (p.n_rows_pad >> 7) - rt0;
            const uint8_t* sfa_tile = p.a_sf + (size_t)m_tile * kAtomBytes * num_kb;
            for (int ks = 0; ks < num_ks; ++ks, ++it) {
                const int s = it % STAGES;
                if (it >= STAGES) {
                    const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1));
                    if (!ok) {
                        if (lane == 0) {
                            record_error(p.err, kErrProducerTimeout);
                            atomicExch(s_abort, 1);
                        }
                        stop = true;
                        break;
                    }
                }
                if (__any_sync(0xffffffffu, aborted(s_abort))) {
                    stop = true;
                    break;
                }
                const int kb0 = ks * kKbPerStage;
                const int nkb = min(kKbPerStage, num_kb - kb0);
                const uint32_t sf_bytes = (uint32_t)nkb * kAtomBytes;
                const int j = lane - (it & 3) * 8;
                if (j == 0) ptx::mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES + sf_bytes * (1 + nrt));
                __syncwarp();
                const int kx = ks * kStageKBytes;
                if (j >= 0 && j < kChunks) {
                    ptx::tma_load_2d(sA + s * C::A_BYTES + j * C::A_CHUNK, &tmap_a, &full[s], kx + j * kChunkBytes, m0);
                } else if (j >= kChunks && j < 2 * kChunks) {
                    ptx::tma_load_2d(sB + s * C::B_BYTES + (j - kChunks) * C::B_CHUNK, &tmap_b, &full[s],
                                     kx + (j - kChunks) * kChunkBytes, n0);
                } else if (j == 2 * kChunks) {
                    ptx::bulk_load(sSFA + s * C::SFA_BYTES, sfa_tile + (size_t)kb0 * kAtomBytes, sf_bytes, &full[s]);
                } else if (j > 2 * kChunks && j <= 2 * kChunks + nrt) {
                    const int rt = j - 2 * kChunks - 1;
                    const uint8_t* src = p.b_sf + ((size_t)(rt0 + rt) * num_kb + kb0) * kAtomBytes;
                    ptx::bulk_load(sSFB + s * C::SFB_BYTES + rt * kKbPerStage * kAtomBytes, src, sf_bytes, &full[s]);
                }
                __syncwarp();
                if (lane == 0) *s_last_issued = it;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp walks the loop (so stage indices and descriptors are
        // warp-uniform values) and one elected lane issues each stage's
        // tcgen05 instructions from fully unrolled, predicated k-block loops.
        const uint64_t adesc0 = ptx::desc_kmajor_sw128(ptx::smem_u32(sA));
        const uint64_t bdesc0 = ptx::desc_kmajor_sw128(ptx::smem_u32(sB));
        const uint64_t sfadesc0 = ptx::desc_sf_atom(ptx::smem_u32(sSFA));
        const uint64_t sfbdesc0 = ptx::desc_sf_atom(ptx::smem_u32(sSFB));
        constexpr uint32_t idesc = ptx::idesc_nvf4(BN);
        int it = 0, tile_iter = 0;
        bool stop = false;
        for (int t = blockIdx.x; t < p.num_tiles && !stop; t += gridDim.x, ++tile_iter) {
            int m_tile_unused, n_tile;
            tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile_unused, n_tile);
            const int n0 = n_tile * BN;
            int nrt = ((n0 & 127) + BN + 127) >> 7;
            if ((n0 >> 7) + nrt > (p.n_rows_pad >> 7)) nrt = (p.n_rows_pad >> 7) - (n0 >> 7);
            const uint32_t shift_words = (n0 & 127) >> 5;
            const int b = tile_iter % C::ACC_BUFS;
            if (tile_iter >= C::ACC_BUFS) {
                const bool ok =
                    __all_sync(0xffffffffu, ptx::mbar_wait(&acc_empty[b], ((tile_iter / C::ACC_BUFS) & 1) ^ 1));
                if (!ok) {
                    if (lane == 0) {
                        record_error(p.err, kErrMmaTimeout);
                        atomicExch(s_abort, 1);
                    }
                    break;
                }
            }
            ptx::tc_fence_after();
            const uint32_t acc = tmem + b * BN;
            const uint32_t sfa_t = tmem + C::TMEM_SFA;
            const uint32_t sfb_t = tmem + C::TMEM_SFB;
            for (int ks = 0; ks < num_ks; ++ks, ++it) {
                const int s = it % STAGES;
                const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (it / STAGES) & 1));
                if (!ok || __any_sync(0xffffffffu, aborted(s_abort))) {
                    if (lane == 0) {
                        record_error(p.err, kErrMmaTimeout);
                        atomicExch(s_abort, 1);
                    }
                    stop = true;
                    break;
                }
                ptx::tc_fence_after();
                const int nkb = min(kKbPerStage, num_kb - ks * kKbPerStage);
                // Descriptor start addresses are in 16-byte units in the low bits.
                const uint64_t a_s = adesc0 + (uint64_t)((s * C::A_BYTES) >> 4);
                const uint64_t b_s = bdesc0 + (uint64_t)((s * C::B_BYTES) >> 4);
                const uint64_t sfa_s = sfadesc0 + (uint64_t)((s * C::SFA_BYTES) >> 4);
                const uint64_t sfb_s = sfbdesc0 + (uint64_t)((s * C::SFB_BYTES) >> 4);
                const uint32_t first = (ks == 0) ? 0u : 1u;
                if (ptx::elect_one()) {
                    // Each k-block's scale copies right before its MMA (see the pair kernel).
#pragma unroll
                    for (int j = 0; j < kKbPerStage; ++j) {
                        if (j < nkb) {
                            ptx::tc_cp_32x128b_warpx4(sfa_t + 4 * j, sfa_s + (uint64_t)((j * kAtomBytes) >> 4));
#pragma unroll
                            for (int r = 0; r < C::NRT; ++r)
                                if (r < nrt)
                                    ptx::tc_cp_32x128b_warpx4(
                                        sfb_t + j * 4 * C::NRT + 4 * r,
                                        sfb_s + (uint64_t)(((r * kKbPerStage + j) * kAtomBytes) >> 4));
                            const uint32_t koff = (uint32_t)(((j >> 2) * C::A_CHUNK + 32 * (j & 3)) >> 4);
                            const uint32_t kofb = (uint32_t)(((j >> 2) * C::B_CHUNK + 32 * (j & 3)) >> 4);
                            ptx::tc_mma_nvf4(acc, a_s + koff, b_s + kofb, idesc, sfa_t + 4 * j,
                                             sfb_t + j * 4 * C::NRT + shift_words, (j == 0) ? first : 1u);
                        }
                    }
                    ptx::tc_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (!stop) {
                if (ptx::elect_one()) ptx::tc_commit(&acc_full[b]);
                __syncwarp();
            }
        }
        if (ptx::elect_one()) ptx::tc_commit(mma_done);  // completes once every MMA issued above is done
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may read
        int tile_iter = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++tile_iter) {
            int m_tile, n_tile;
            tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile, n_tile);
            const int n0 = n_tile * BN;
            const int m = m_tile * kBM + q * 32 + lane;
            const int b = tile_iter % C::ACC_BUFS;
            const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&acc_full[b], (tile_iter / C::ACC_BUFS) & 1));
            if (!ok || __any_sync(0xffffffffu, aborted(s_abort))) {
                if (lane == 0 && !ok) {
                    record_error(p.err, kErrEpilogueTimeout);
                    atomicExch(s_abort, 1);
                }
                break;
            }
            ptx::tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + b * BN + 32 * c, r);
                ptx::tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    // All TMEM reads of this buffer are done: hand it back to the MMA warp.
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&acc_empty[b]);
                }
                if (m < p.m && n0 + 32 * c < p.n_out) store_chunk(p, r, m, n0 + 32 * c);
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        // Every MMA has completed before TMEM is released; on an abort, let the
        // copies already issued land before the CTA's smem goes away.
        ptx::mbar_wait(mma_done, 0);
        if (aborted(s_abort)) {
            const int last = *s_last_issued;
            for (int k = (last - STAGES + 1 > 0 ? last - STAGES + 1 : 0); k <= last; ++k)
                ptx::mbar_wait(&full[k % STAGES], (k / STAGES) & 1);
        }
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------------ CTA-pair kernel
// 256 x BN output tiles (or 256 x 2BN, see PairCfg) on a cluster of two CTAs
// with tcgen05 cta_group::2: CTA r of the pair loads rows [128r, 128r + 128)
// of the A tile, rows [r*BN/2, (r+1)*BN/2) of the B tile, the scale atoms of
// its own A rows and the scale atoms of all B rows of the tile; the even CTA
// issues one M=256 MMA per 64-wide k-block (and N-subtile) for both.  Per SM this moves a third less operand data per
// FLOP than a 128 x BN tile on one SM, and halves the MMA instructions.
//
// Synchronisation across the pair:
//   full[s]      in CTA 0 only: both CTAs' TMA loads of stage s complete on it
//                (cta_group::2 loads may signal the peer's barrier); CTA 0's
//                producer posts the expected bytes of both.
//   empty[s]     in both CTAs: CTA 0's commit arrives on both.
//   acc_full[b]  in both CTAs: CTA 0's commit arrives on both.
//   acc_empty[b] in CTA 0: the 8 epilogue warps of both CTAs arrive (16 arrivals).
//   mma_done     in both CTAs: the last commit; every MMA of the pair is done.
//   bias_ready   in each CTA: its 8 epilogue warps staged the last tile's bias,
//                which the whole team of the last tile reads.
// Scale-factor boxes are loaded with 3-D tensor maps over the atom array
// ([row tile][k-block][512 bytes]) so they too can complete on CTA 0's barrier.
//
// 416 threads: warps 0-7 epilogue (warp w reads TMEM lanes 32(w%4)..+31 and
// stores the 64-column super-chunks s with s % 2 == w / 4 as 16 x 64 pieces;
// with an odd count the last super-chunk is split by rows: warp w stores its
// rows 16 (w / 4) .. +15), warp 8 TMEM allocation
// and MMA issue, warps 9-12 one producer per copy type
// (A, B, scale-A, scale-B).  The pair's last tile is stored by all 13 warps
// (team_epilogue): the MMA and producer warps have nothing left to do.  A TMA issue keeps its warp busy for ~130 ns on
// B200 and one thread's copies run one after another (~0.4 us each), so the
// four copies of a stage go out from four warps in parallel, each from a lane
// that has not issued for 32 stages.
constexpr int kPairEpiWarps = 8;  // two per TMEM lane quadrant, each storing half of the columns

// A pair tile is 256 x TW: with NSUB = 2, two MMAs per k-block (N = BN on
// columns [0, BN), N = BN1 on [BN, BN + BN1)) share the A tile, which moves
// fewer operand bytes per column; its accumulator is single-buffered, so it
// suits problems whose tiles fit in one round of CTA pairs.
// CHUNKS: 128-byte-wide chunks of K per stage (K = 256 each), loaded as one
// TMA box per operand and chunk, back to back.  Two chunks per stage stream a
// weight that comes from HBM (small M) faster: each weight row is read 256
// contiguous bytes at a time instead of 128.
template <int BN, int STAGES, int NSUB = 1, int BN1 = BN, int CHUNKS = 1>
struct PairCfg {
    static constexpr int kKbPerStage = 4 * CHUNKS;   // 64-element k-blocks per stage
    static_assert(BN % 64 == 0 && BN >= 128 && BN <= 256, "BN must be 128, 192 or 256");
    static_assert(BN1 % 64 == 0 && BN1 >= 128 && BN1 <= 256, "BN1 must be 128, 192 or 256");
    static_assert(NSUB == 1 || NSUB == 2, "one or two MMAs per k-block");
    static_assert(NSUB == 2 || BN1 == BN, "a second width needs a second MMA");
    static constexpr int TW = BN + (NSUB - 1) * BN1;  // tile width
    static constexpr int BH = BN / 2;       // B rows of the first MMA held by each CTA
    static constexpr int BH1 = BN1 / 2;     // B rows of the second MMA held by each CTA
    static constexpr int NRT = max_row_tiles(TW);
    static constexpr int A_CHUNK = kBM * kChunkBytes;          // one TMA box of A
    static constexpr int A_BYTES = CHUNKS * A_CHUNK;
    static constexpr int B_SUB_BYTES = BH * kChunkBytes;
    static constexpr int B_SUB1_BYTES = BH1 * kChunkBytes;
    static constexpr int B_CHUNK = B_SUB_BYTES + (NSUB - 1) * B_SUB1_BYTES;  // the B boxes of one chunk
    static constexpr int B_BYTES = CHUNKS * B_CHUNK;
    static constexpr int SFA_BYTES = kKbPerStage * kAtomBytes;
    static constexpr int SFB_BYTES = NRT * kKbPerStage * kAtomBytes;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    // Every box is loaded whole (out-of-range parts read as zero), so a stage
    // always brings the same bytes: those of both CTAs land on CTA 0's barrier.
    static constexpr uint32_t TX_BYTES = 2u * STAGE_BYTES;
    static constexpr int BAR_BYTES = 256;
    // Epilogue staging: one 2 KB BF16 buffer (a 32 x 32 chunk or a 16 x 64
    // piece) and room for the tile's BF16 bias per epilogue warp.
    static constexpr int EPI_BYTES = kPairEpiWarps * 2048;
    static constexpr int BIAS_BYTES = kPairEpiWarps * TW * 2;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + BIAS_BYTES + BAR_BYTES + 1024;
    static constexpr int SF_COLS = 4 * kKbPerStage * (1 + NRT);
    static constexpr int ACC_BUFS = (2 * TW + SF_COLS <= (int)kTmemCols) ? 2 : 1;
    static constexpr uint32_t TMEM_SFA = ACC_BUFS * TW;
    static constexpr uint32_t TMEM_SFB = TMEM_SFA + 4 * kKbPerStage;
    static_assert(B_SUB_BYTES % 1024 == 0 && B_SUB1_BYTES % 1024 == 0, "B stage must keep the 128B-swizzle alignment");
    static_assert(STAGE_BYTES % 1024 == 0, "epilogue buffers must stay 1024-byte aligned");
    static_assert(STAGES * STAGE_BYTES >= 4 * (TW / 64) * 4096, "the idle ring stages all of the last tile");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
    static_assert(TMEM_SFA + SF_COLS <= kTmemCols, "TMEM budget exceeded");
};

constexpr uint64_t kAbortDrainNs = 200000;  // after an abort, let issued copies land
constexpr int kPairThreads = 416;
constexpr int kPairMmaWarp = 8;
constexpr int kPairFirstProducer = 9;

// Await mode (AWAIT, the overlapped cached linear): the activation quantizer
// (quantize_units.cu) runs beside this kernel on the same SMs and publishes,
// for every 128-row tile of A and 256-wide K-stage, a counter that reaches 2
// once both of its 64-row units are stored.  The A and scale-A producers wait
// (bounded) for their tile's counter of each stage instead of for the whole
// quantizer grid, and the MMA and producer warps skip the programmatic wait
// altogether; only the epilogue warps wait for the quantizer to complete.
// The last CTA to exit zeroes the counters for the next launch.

// Epilogue of a CTA pair's last tile by a team of warps per TMEM lane
// quadrant q: the two epilogue warps q and q + 4 (members 0, 1) and the warps
// whose roles have ended (8 and 12 on quadrant 0, 9, 10, 11 on quadrants 1-3).
// The operand ring is idle once the last tile's MMAs have completed: every
// chunk gets a staging slot of its own there, so no store waits for an earlier
// one to finish reading.  tq: TMEM address of the quadrant's accumulator; m:
// this lane's output row.
// Single-GPU form: member ti of ts takes the 32-column chunks c = ti, ti + ts,
// ... (slot q * CH + c, 2 KB); chunk c's BF16 bias was staged by epilogue warp
// q + 4 (c & 1) (uint4 offset 4 c).
template <int TW>
__device__ __forceinline__ void team_epilogue_chunks(const Params& p, const CUtensorMap* tmap_d, uint32_t tq,
                                                     const uint4* sBias, int q, int ti, int ts, uint8_t* ring,
                                                     int& chunk_iter, int m, int n0, int lane) {
    constexpr int CH = TW / 32;
    // The next chunk's TMEM load is issued once this one is converted, so its
    // latency overlaps the staging and the store.
    uint32_t r[32];
    if (ti < CH) ptx::tmem_ld_32x32b_x32(tq + 32 * ti, r);
#pragma unroll 1
    for (int c = ti; c < CH; c += ts) {
        ptx::tmem_ld_wait();
        const bool live = n0 + 32 * c < p.n_out;
        if (p.tma_store) {
            uint32_t pk[16];
            convert_chunk(p, r, sBias + (q + 4 * (c & 1)) * (TW / 8) + 4 * c, pk);
            if (c + ts < CH) ptx::tmem_ld_32x32b_x32(tq + 32 * (c + ts), r);
            if (live && m - lane < p.m)  // the warp's 32 rows start inside D
                store_staged_chunk(tmap_d, pk, ring + (size_t)(q * CH + c) * 2048, m - lane, n0 + 32 * c, lane,
                                   chunk_iter++, true);
        } else {
            if (live && m < p.m) store_chunk(p, r, m, n0 + 32 * c);
            if (c + ts < CH) ptx::tmem_ld_32x32b_x32(tq + 32 * (c + ts), r);
        }
    }
}

// Column-parallel form (TMA stores, peers): member ti of ts takes the
// 64-column super-chunks s = ti, ti + ts, ...: it converts both 32-column
// halves, stages the quadrant's 32 rows of the super-chunk in slot q * S + s
// (4 KB, 128-byte swizzle) and stores them as two 16 x 64 pieces (128-byte
// rows), locally and into every peer's buffer.  The tile's BF16 bias was
// staged whole by epilogue warp q (chunk c at uint4 offset 4 c).
template <int TW>
__device__ __forceinline__ void team_epilogue_pieces(const Params& p, const CUtensorMap* tmap_d, const PeerMaps* pm,
                                                     uint32_t tq, const uint4* sBias, int q, int ti, int ts,
                                                     uint8_t* ring, int& chunk_iter, int m, int n0, int lane) {
    constexpr int S = TW / 64;
    const uint4* qbias = sBias + q * (TW / 8);
    const int row0 = m - lane;  // the warp's first row
    // The next super-chunk's TMEM loads are issued once this one is converted,
    // so their latency overlaps the staging and the stores.  (Column-parallel
    // launches always have TMA stores.)
    uint32_t ra[32], rb[32];
    if (ti < S) {
        ptx::tmem_ld_32x32b_x32(tq + 64 * ti, ra);
        ptx::tmem_ld_32x32b_x32(tq + 64 * ti + 32, rb);
    }
#pragma unroll 1
    for (int s = ti; s < S; s += ts) {
        ptx::tmem_ld_wait();
        const int nc = n0 + 64 * s;
        const bool live = nc < p.n_out && row0 < p.m;  // columns and the warp's first row inside D
        uint8_t* slot = ring + (size_t)(q * S + s) * 4096;
        // Row `lane` starts 128-byte aligned: unit u ^ (lane & 7) of it is at
        // (row + 16 (lane & 7)) ^ 16 u.
        const uint32_t a = ptx::smem_u32(slot) + 128u * lane + 16u * (lane & 7u);
        uint32_t pk[16];
        if (live) {
            convert_chunk(p, ra, qbias + 8 * s, pk);
#pragma unroll
            for (int u = 0; u < 4; ++u)
                ptx::st_shared_v4(a ^ (16u * u), pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            convert_chunk(p, rb, qbias + 8 * s + 4, pk);
        }
        if (s + ts < S) {
            ptx::tmem_ld_32x32b_x32(tq + 64 * (s + ts), ra);
            ptx::tmem_ld_32x32b_x32(tq + 64 * (s + ts) + 32, rb);
        }
        if (live) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
                ptx::st_shared_v4(a ^ (16u * (u + 4)), pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == (chunk_iter & 31)) {
                ptx::tma_store_2d(tmap_d, slot, nc, row0);
                for (int d = 0; d < p.npeers; ++d) ptx::tma_store_2d(&pm->map[d], slot, nc, row0);
                if (row0 + 16 < p.m) {
                    ptx::tma_store_2d(tmap_d, slot + 2048, nc, row0 + 16);
                    for (int d = 0; d < p.npeers; ++d) ptx::tma_store_2d(&pm->map[d], slot + 2048, nc, row0 + 16);
                }
                ptx::bulk_commit_group();
            }
            ++chunk_iter;
        }
    }
}

template <int BN, int STAGES, bool AWAIT, int NSUB, int BN1, bool PIECES, int CHUNKS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    nvf4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_b1,
                          const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                          const __grid_constant__ CUtensorMap tmap_d, const __grid_constant__ CUtensorMap tmap_d64,
                          const __grid_constant__ Params p, const __grid_constant__ PeerMaps pm) {
    using C = PairCfg<BN, STAGES, NSUB, BN1, CHUNKS>;
    static_assert(!AWAIT || CHUNKS == 1, "the quantizer's unit counters cover K stages of 256");
    constexpr int TW = C::TW;
    constexpr int TILE_M = 2 * kBM;
    constexpr int kKbPerStage = C::kKbPerStage;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * C::A_BYTES;
    uint8_t* sSFA = sB + STAGES * C::B_BYTES;
    uint8_t* sSFB = sSFA + STAGES * C::SFA_BYTES;
    uint8_t* sEpi = sSFB + STAGES * C::SFB_BYTES;
    uint4* sBias = reinterpret_cast<uint4*>(sEpi + C::EPI_BYTES);
    uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + C::EPI_BYTES + C::BIAS_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;     // [2]
    uint64_t* acc_empty = acc_full + 2;      // [2]
    uint64_t* mma_done = acc_empty + 2;
    uint64_t* bias_ready = mma_done + 1;  // the epilogue warps staged the last tile's bias
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bias_ready + 1);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = ptx::cluster_ctarank();  // 0: issues the pair's MMAs
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int num_kb = p.num_kb;
    const int num_ks = (num_kb + kKbPerStage - 1) / kKbPerStage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], 2 * kPairEpiWarps);
        }
        ptx::mbar_init(mma_done, 1);
        ptx::mbar_init(bias_ready, kPairEpiWarps);
        *s_abort = 0;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
        if (NSUB > 1) ptx::prefetch_tmap(&tmap_b1);
        ptx::prefetch_tmap(&tmap_sfa);
        ptx::prefetch_tmap(&tmap_sfb);
        if (p.tma_store) {
            ptx::prefetch_tmap(&tmap_d);
            if constexpr (PIECES) ptx::prefetch_tmap(&tmap_d64);
        }
    }
    if (warp == kPairMmaWarp) {
        ptx::tmem_alloc_pair(tmem_slot, kTmemCols);
        ptx::tmem_relinquish_pair();
    }
    ptx::tc_fence_before();
    // Both CTAs' barriers exist before any load, commit or arrive reaches them.
    ptx::cluster_sync();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Launched behind the activation quantizer: barriers and TMEM are set up
    // while it finishes.  A cached weight (b_early) was complete before the
    // quantizer started, so the B and scale-B producers start loading it now
    // (their bytes may land on a `full` barrier before the A producer posts the
    // stage's byte count; the phase still needs that arrival).  Every other
    // role touches global memory only after the quantizer has completed; the
    // producers' last-tile epilogue work follows the MMA warp's, which does.
    // In await mode the quantizer is still running: the A producers wait for
    // its counters instead, and the MMA and producer warps do not wait for it.
    const bool early_b = p.b_early && warp >= kPairFirstProducer && ((warp - kPairFirstProducer) & 1) == 1;
    if (!early_b && !(AWAIT && warp >= kPairMmaWarp)) ptx::grid_dependency_wait();
    // The kernel after this one (the next quantizer) may be scheduled on SMs
    // this grid leaves; it waits for this grid to complete before it reads or
    // writes global memory.
    ptx::launch_dependents();

    if (warp >= kPairFirstProducer) {
        // ------------------------------------------------------------ producers (both CTAs)
        const int role = warp - kPairFirstProducer;  // 0 A, 1 B, 2 scale-A, 3 scale-B
        const uint32_t full0 = ptx::map_to_cta(ptx::smem_u32(full), 0);
        int it = 0;
        bool stop = false;
        for (int t = pair; t < p.num_tiles && !stop; t += npairs) {
            int m_tile, n_tile;
            tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile, n_tile);
            const int n0 = n_tile * TW;
            const int a_row = m_tile * 2 * kBM + (int)rank * kBM;
            const int b_row = n0 + (int)rank * C::BH;
            const int sfa_rt = m_tile * 2 + (int)rank;
            const int sfb_rt = n0 >> 7;
            for (int ks = 0; ks < num_ks; ++ks, ++it) {
                const int s = it % STAGES;
                if (it >= STAGES) {
                    const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1));
                    if (!ok) {
                        if (lane == 0) {
                            record_error(p.err, kErrProducerTimeout);
                            atomicExch(s_abort, 1);
                        }
                        stop = true;
                        break;
                    }
                }
                if (__any_sync(0xffffffffu, aborted(s_abort))) {
                    stop = true;
                    break;
                }
                if constexpr (AWAIT) {
                    // A CTA whose 128 rows lie wholly past the padded rows of A (the
                    // second half of a last 256-row tile when rows_pad % 256 == 128)
                    // has no units to wait for: its TMA boxes read zeros.
                    if ((role == 0 || role == 2) && 2 * m_tile + (int)rank < p.a_tiles128) {
                        // Both 64-row units of this CTA's 128 rows of A for this K-stage
                        // are quantized and visible to TMA.
                        bool ok = true;
                        if (lane == 0)
                            ok = ptx::wait_counter_geq(p.ready + (size_t)(2 * m_tile + (int)rank) * p.a_stages + ks,
                                                       2u);
                        ok = __shfl_sync(0xffffffffu, ok, 0);
                        if (!ok) {
                            if (lane == 0) {
                                record_error(p.err, kErrQuantizeWaitTimeout);
                                atomicExch(s_abort, 1);
                            }
                            stop = true;
                            break;
                        }
                        ptx::fence_proxy_async_global();
                    }
                }
                // The B copies of the NSUB MMAs go out from different lanes.
                const int sub = (NSUB > 1 && role == 1 && lane == ((it + 16) & 31)) ? 1 : 0;
                if (lane == (it & 31) || sub == 1) {
                    const uint32_t bar = full0 + (uint32_t)s * 8u;
                    const int kb0 = ks * kKbPerStage;
                    if (role == 0) {
                        if (rank == 0) ptx::mbar_arrive_expect_tx(&full[s], C::TX_BYTES);
#pragma unroll
                        for (int c = 0; c < CHUNKS; ++c)
                            ptx::tma_load_2d_pair(sA + s * C::A_BYTES + c * C::A_CHUNK, &tmap_a, bar,
                                                  (ks * CHUNKS + c) * kChunkBytes, a_row);
                    } else if (role == 1) {
#pragma unroll
                        for (int c = 0; c < CHUNKS; ++c) {
                            const int kx = (ks * CHUNKS + c) * kChunkBytes;
                            uint8_t* dst = sB + s * C::B_BYTES + c * C::B_CHUNK;
                            if (sub == 0)
                                ptx::tma_load_2d_pair(dst, &tmap_b, bar, kx, b_row);
                            else  // the second MMA's rows [n0 + BN, n0 + TW), split between the CTAs
                                ptx::tma_load_2d_pair(dst + C::B_SUB_BYTES, &tmap_b1, bar, kx,
                                                      n0 + BN + (int)rank * C::BH1);
                        }
                    } else if (role == 2) {
                        ptx::tma_load_3d_pair(sSFA + s * C::SFA_BYTES, &tmap_sfa, bar, 0, kb0, sfa_rt);
                    } else {
                        ptx::tma_load_3d_pair(sSFB + s * C::SFB_BYTES, &tmap_sfb, bar, 0, kb0, sfb_rt);
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == kPairMmaWarp) {
        // ------------------------------------------------------------ MMA issuer (CTA 0)
        if (rank == 0) {
            const uint64_t adesc0 = ptx::desc_kmajor_sw128(ptx::smem_u32(sA));
            const uint64_t bdesc0 = ptx::desc_kmajor_sw128(ptx::smem_u32(sB));
            const uint64_t sfadesc0 = ptx::desc_sf_atom(ptx::smem_u32(sSFA));
            const uint64_t sfbdesc0 = ptx::desc_sf_atom(ptx::smem_u32(sSFB));
            constexpr uint32_t idesc = ptx::idesc_nvf4(BN, 2 * kBM);
            constexpr uint32_t idesc1 = ptx::idesc_nvf4(BN1, 2 * kBM);
            int it = 0, tile_iter = 0;
            bool stop = false;
            for (int t = pair; t < p.num_tiles && !stop; t += npairs, ++tile_iter) {
                int m_tile_unused, n_tile;
                tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile_unused, n_tile);
                const int n0 = n_tile * TW;
                const uint32_t shift_words = (n0 & 127) >> 5;
                const int b = tile_iter % C::ACC_BUFS;
                if (tile_iter >= C::ACC_BUFS) {
                    const bool ok = __all_sync(0xffffffffu,
                                               ptx::mbar_wait(&acc_empty[b], ((tile_iter / C::ACC_BUFS) & 1) ^ 1));
                    if (!ok) {
                        if (lane == 0) {
                            record_error(p.err, kErrMmaTimeout);
                            atomicExch(s_abort, 1);
                        }
                        break;
                    }
                }
                ptx::tc_fence_after();
                const uint32_t acc = tmem + b * TW;
                const uint32_t sfa_t = tmem + C::TMEM_SFA;
                const uint32_t sfb_t = tmem + C::TMEM_SFB;
                for (int ks = 0; ks < num_ks; ++ks, ++it) {
                    const int s = it % STAGES;
                    const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (it / STAGES) & 1));
                    if (!ok || __any_sync(0xffffffffu, aborted(s_abort))) {
                        if (lane == 0) {
                            record_error(p.err, kErrMmaTimeout);
                            atomicExch(s_abort, 1);
                        }
                        stop = true;
                        break;
                    }
                    ptx::tc_fence_after();
                    const int nkb = min(kKbPerStage, num_kb - ks * kKbPerStage);
                    const uint64_t a_s = adesc0 + (uint64_t)((s * C::A_BYTES) >> 4);
                    const uint64_t b_s = bdesc0 + (uint64_t)((s * C::B_BYTES) >> 4);
                    const uint64_t sfa_s = sfadesc0 + (uint64_t)((s * C::SFA_BYTES) >> 4);
                    const uint64_t sfb_s = sfbdesc0 + (uint64_t)((s * C::SFB_BYTES) >> 4);
                    const uint32_t first = (ks == 0) ? 0u : 1u;
                    if (ptx::elect_one()) {
                        // Each k-block's scale copies go right before its own MMAs:
                        // on B200 the tensor pipe then overlaps them with the previous
                        // k-block's MMAs (issuing a stage's copies first cost ~5 % of
                        // the MMA rate of the 320-wide tile, ~7 % of the 384-wide one).
#pragma unroll
                        for (int j = 0; j < kKbPerStage; ++j) {
                            if (j < nkb) {
                                ptx::tc_cp_32x128b_warpx4_pair(sfa_t + 4 * j,
                                                               sfa_s + (uint64_t)((j * kAtomBytes) >> 4));
#pragma unroll
                                for (int r = 0; r < C::NRT; ++r)
                                    ptx::tc_cp_32x128b_warpx4_pair(
                                        sfb_t + j * 4 * C::NRT + 4 * r,
                                        sfb_s + (uint64_t)(((r * kKbPerStage + j) * kAtomBytes) >> 4));
                                // k-block j: 32 bytes into its chunk's 128-byte rows
                                const uint32_t koff = (uint32_t)((32 * (j & 3)) >> 4);
                                const uint64_t a_kb = CHUNKS == 1 ? a_s : a_s + (uint64_t)(((j >> 2) * C::A_CHUNK) >> 4);
                                const uint64_t b_kb = CHUNKS == 1 ? b_s : b_s + (uint64_t)(((j >> 2) * C::B_CHUNK) >> 4);
#pragma unroll
                                for (int u = 0; u < NSUB; ++u)
                                    ptx::tc_mma_nvf4_pair(acc + u * BN, a_kb + koff,
                                                          b_kb + (uint64_t)((u * C::B_SUB_BYTES) >> 4) + koff,
                                                          u == 0 ? idesc : idesc1, sfa_t + 4 * j,
                                                          sfb_t + j * 4 * C::NRT + shift_words + (u * BN) / 32,
                                                          (j == 0) ? first : 1u);
                            }
                        }
                        ptx::tc_commit_pair(&empty[s], 0x3);
                    }
                    __syncwarp();
                }
                if (!stop) {
                    if (ptx::elect_one()) ptx::tc_commit_pair(&acc_full[b], 0x3);
                    __syncwarp();
                }
            }
            if (ptx::elect_one()) ptx::tc_commit_pair(mma_done, 0x3);
            __syncwarp();
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Single-GPU form (!PIECES): warp w stores the 32-column chunks
        // c = h, h + 2, ... as 32 x 32 boxes.  Column-parallel form: the 64-column
        // super-chunks s = h, h + 2, ... as 16 x 64 pieces (128-byte rows for the
        // stores over NVLink); with an odd count the last super-chunk is split by
        // rows, warp w storing rows 16 h .. 16 h + 15 of it.  (Pieces cost the
        // single-GPU GEMM 1-5 %: half the lanes stage each piece; and one kernel
        // holding both forms spilled registers on the 384-wide tile.)
        const int q = warp & 3;   // TMEM lane quadrant
        const int h = warp >> 2;
        constexpr bool pieces = PIECES;
        constexpr int kMyChunks = TW / 64;              // chunks per warp, single-GPU form
        constexpr int S = TW / 64;                      // 64-column super-chunks of a tile
        constexpr int kFull = S / 2;                    // whole super-chunks per warp
        constexpr bool kSplit = (S & 1) != 0;           // the last one is split by rows between the two warps
        constexpr int kIters = kFull + (kSplit ? 1 : 0);
        const uint32_t acc_empty0 = ptx::map_to_cta(ptx::smem_u32(acc_empty), 0);
        uint8_t* epi = sEpi + warp * 2048;
        uint4* wbias = sBias + warp * (TW / 8);
        int chunk_iter = 0;
        int tile_iter = 0;
        for (int t = pair; t < p.num_tiles; t += npairs, ++tile_iter) {
            int m_tile, n_tile;
            tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile, n_tile);
            const int n0 = n_tile * TW;
            const int m = m_tile * 2 * kBM + (int)rank * kBM + q * 32 + lane;
            const int b = tile_iter % C::ACC_BUFS;
            const bool last_tile = t + npairs >= p.num_tiles;
            if (p.bias) {
                // Chunk c's bias at wbias + 4 c: every chunk of the tile for the
                // pieces, this warp's chunks for the single-GPU form.
                __syncwarp();  // the previous tile's reads of wbias are done
                if constexpr (pieces) {
#pragma unroll
                    for (int c = 0; c < TW / 32; ++c) stage_bias(p, wbias + 4 * c, n0 + 32 * c, 32, lane);
                } else {
#pragma unroll
                    for (int j = 0; j < kMyChunks; ++j)
                        stage_bias(p, wbias + 4 * (h + 2 * j), n0 + 32 * (h + 2 * j), 32, lane);
                }
                __syncwarp();
            }
            if (last_tile && lane == 0) ptx::mbar_arrive(bias_ready);
            const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&acc_full[b], (tile_iter / C::ACC_BUFS) & 1));
            if (!ok || __any_sync(0xffffffffu, aborted(s_abort))) {
                if (lane == 0 && !ok) {
                    record_error(p.err, kErrEpilogueTimeout);
                    atomicExch(s_abort, 1);
                }
                break;
            }
            ptx::tc_fence_after();
            if (last_tile) {
                // Shared with the warps whose roles have ended (team_epilogue).
                if (!__all_sync(0xffffffffu, ptx::mbar_wait(bias_ready, 0))) {
                    if (lane == 0) {
                        record_error(p.err, kErrEpilogueTimeout);
                        atomicExch(s_abort, 1);
                    }
                    break;
                }
                const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + b * TW;
                if constexpr (pieces)
                    team_epilogue_pieces<TW>(p, &tmap_d64, &pm, tq, sBias, q, h, q == 0 ? 4 : 3, smem, chunk_iter, m,
                                             n0, lane);
                else
                    team_epilogue_chunks<TW>(p, &tmap_d, tq, sBias, q, h, q == 0 ? 4 : 3, smem, chunk_iter, m, n0,
                                             lane);
                continue;
            }
            // Only a later tile of this pair that reuses accumulator b waits for it.
            const bool release = t + C::ACC_BUFS * npairs < p.num_tiles;
            if constexpr (!pieces) {
                // Chunks go two at a time: both are converted together (independent
                // work for the warp's latency), then the next two TMEM loads are issued
                // into the freed registers while the converted pair is stored.
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + b * TW + 32 * h;
                uint32_t ra[32], rb[32];
                ptx::tmem_ld_32x32b_x32(tbase, ra);
                if (kMyChunks > 1) ptx::tmem_ld_32x32b_x32(tbase + 64, rb);
#pragma unroll
                for (int j = 0; j < kMyChunks; j += 2) {
                    const bool two = j + 1 < kMyChunks;
                    const int c0 = h + 2 * j, c1 = c0 + 2;
                    const bool in0 = n0 + 32 * c0 < p.n_out, in1 = two && n0 + 32 * c1 < p.n_out;
                    ptx::tmem_ld_wait();
                    if (p.tma_store) {
                        uint32_t pa[16], pb[16];
                        convert_chunk(p, ra, wbias + 4 * c0, pa);
                        if (two) convert_chunk(p, rb, wbias + 4 * c1, pb);
                        if (j + 2 < kMyChunks) {
                            ptx::tmem_ld_32x32b_x32(tbase + 64 * (j + 2), ra);
                            if (j + 3 < kMyChunks) ptx::tmem_ld_32x32b_x32(tbase + 64 * (j + 3), rb);
                        } else if (release) {
                            // Every TMEM read of this accumulator is done: hand it back to the MMA issuer.
                            ptx::tc_fence_before();
                            __syncwarp();
                            if (lane == 0) ptx::mbar_arrive_cluster(acc_empty0 + (uint32_t)b * 8u);
                        }
                        if (m - lane < p.m) {  // the warp's 32 rows start inside D
                            if (in0) store_staged_chunk(&tmap_d, pa, epi, m - lane, n0 + 32 * c0, lane, chunk_iter++);
                            if (in1) store_staged_chunk(&tmap_d, pb, epi, m - lane, n0 + 32 * c1, lane, chunk_iter++);
                        }
                    } else {
                        if (m < p.m) {
                            if (in0) store_chunk(p, ra, m, n0 + 32 * c0);
                            if (in1) store_chunk(p, rb, m, n0 + 32 * c1);
                        }
                        if (j + 2 < kMyChunks) {
                            ptx::tmem_ld_32x32b_x32(tbase + 64 * (j + 2), ra);
                            if (j + 3 < kMyChunks) ptx::tmem_ld_32x32b_x32(tbase + 64 * (j + 3), rb);
                        } else if (release) {
                            ptx::tc_fence_before();
                            __syncwarp();
                            if (lane == 0) ptx::mbar_arrive_cluster(acc_empty0 + (uint32_t)b * 8u);
                        }
                    }
                }
                continue;
            }
            // Column-parallel form (TMA stores; launch_pair refuses peers without
            // them).  One super-chunk (two 32-column TMEM loads) per iteration: both halves
            // are converted together (independent work for the warp's latency), then
            // the next super-chunk's loads are issued into the freed registers while
            // the converted one is stored.
            const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + b * TW;
            const int row0 = m - lane;  // the warp's first row
            const uint4* wbh = wbias + 8 * h;
            uint32_t ra[32], rb[32];
            ptx::tmem_ld_32x32b_x32(tacc + 64 * h, ra);
            ptx::tmem_ld_32x32b_x32(tacc + 64 * h + 32, rb);
#pragma unroll
            for (int j = 0; j < kIters; ++j) {
                const bool split = kSplit && j == kFull;
                const int sc = split ? S - 1 : h + 2 * j;
                const int nsc = (j + 1 == kFull && kSplit) ? S - 1 : h + 2 * (j + 1);  // next iteration's
                const int nc = n0 + 64 * sc;
                ptx::tmem_ld_wait();
                uint32_t pa[16], pb[16];
                const uint4* bsc = (kSplit && split) ? wbias + 8 * (S - 1) : wbh + 16 * j;  // chunks 2 sc, 2 sc + 1
                convert_chunk(p, ra, bsc, pa);
                convert_chunk(p, rb, bsc + 4, pb);
                if (j + 1 < kIters) {
                    ptx::tmem_ld_32x32b_x32(tacc + 64 * nsc, ra);
                    ptx::tmem_ld_32x32b_x32(tacc + 64 * nsc + 32, rb);
                } else if (release) {
                    // Every TMEM read of this accumulator is done: hand it back to the MMA issuer.
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive_cluster(acc_empty0 + (uint32_t)b * 8u);
                }
                if (nc < p.n_out) {
                    if (!split) {
                        if (row0 < p.m) store_piece(p, &tmap_d64, &pm, pa, pb, epi, row0, nc, 0, lane, chunk_iter++);
                        if (row0 + 16 < p.m)
                            store_piece(p, &tmap_d64, &pm, pa, pb, epi, row0 + 16, nc, 1, lane, chunk_iter++);
                    } else if (row0 + 16 * h < p.m) {
                        store_piece(p, &tmap_d64, &pm, pa, pb, epi, row0 + 16 * h, nc, h, lane, chunk_iter++);
                    }
                }
            }
        }
        ptx::bulk_wait_group_all();  // every lane's stores have read shared memory and written D
        if (p.npeers > 0) {
            // The peer stores (async proxy) are complete; order them before the
            // rank-ordering signal that follows the kernel.
            ptx::fence_proxy_async_global();
            __threadfence_system();
        }
    }

    if (warp >= kPairMmaWarp && !__any_sync(0xffffffffu, aborted(s_abort))) {
        // -------------------------------------------- MMA and producer warps: help with the last tile
        const int q = warp & 3;
        const int ti = warp == kPairThreads / 32 - 1 ? 3 : 2;  // warp 12 is quadrant 0's fourth member
        const int n_pair = (p.num_tiles - pair + npairs - 1) / npairs;
        const int t = pair + (n_pair - 1) * npairs;
        const int last_iter = n_pair - 1;
        const int b = last_iter % C::ACC_BUFS;
        int m_tile, n_tile;
        tile_coords(t, p.m_tiles, p.n_tiles, TILE_M, m_tile, n_tile);
        const int n0 = n_tile * TW;
        const int m = m_tile * 2 * kBM + (int)rank * kBM + q * 32 + lane;
        const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(bias_ready, 0)) &&
                        __all_sync(0xffffffffu, ptx::mbar_wait(&acc_full[b], (last_iter / C::ACC_BUFS) & 1));
        if (!ok) {
            if (lane == 0) {
                record_error(p.err, kErrEpilogueTimeout);
                atomicExch(s_abort, 1);
            }
        } else if (!__any_sync(0xffffffffu, aborted(s_abort))) {
            ptx::tc_fence_after();
            // Every MMA has completed and no load is left: the operand ring is idle.
            int chunk_iter = 0;
            const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + b * TW;
            if constexpr (PIECES)
                team_epilogue_pieces<TW>(p, &tmap_d64, &pm, tq, sBias, q, ti, q == 0 ? 4 : 3, smem, chunk_iter, m,
                                         n0, lane);
            else
                team_epilogue_chunks<TW>(p, &tmap_d, tq, sBias, q, ti, q == 0 ? 4 : 3, smem, chunk_iter, m, n0,
                                         lane);
            ptx::bulk_wait_group_all();
            if (p.npeers > 0) {
                ptx::fence_proxy_async_global();
                __threadfence_system();
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        // The last commit of CTA 0 reaches both CTAs once every MMA of the pair
        // has completed (it reads both CTAs' shared memory and TMEM).
        ptx::mbar_wait(mma_done, 0);
        if (aborted(s_abort)) {
            const uint64_t t0 = ptx::global_timer_ns();
            while (ptx::global_timer_ns() - t0 < kAbortDrainNs) {
            }
        }
    }
    if constexpr (AWAIT) {
        // The last CTA to get here (all producers are past their waits) zeroes
        // the unit counters for the next launch.
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(p.ready + p.ready_count, 1u) == gridDim.x - 1) {
                for (int j = 0; j < p.ready_count; ++j) atomicExch(p.ready + j, 0u);
                atomicExch(p.ready + p.ready_count, 0u);
                __threadfence();
            }
        }
    }
    // Neither CTA leaves or frees TMEM while its peer may still signal it.
    ptx::cluster_sync();
    if (warp == kPairMmaWarp) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc_pair(tmem, kTmemCols);
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
// A box wholly or partly past K reads zeros (TMA out-of-bounds fill).
bool make_operand_map(CUtensorMap* map, const void* base, long rows, long k_pad, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(k_pad / 2), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(k_pad / 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kChunkBytes, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel on the stream finishes, and waits for it
// (grid_dependency_wait) before touching global memory.
template <typename K, typename... Args>
cudaError_t launch_dependent(K kernel, dim3 grid, dim3 block, int smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Scale atoms of an operand with `rows_pad` rows as a 3-D array of 64-bit
// words: [row tile][k-block][64 words = 512 bytes], boxes of kb_box k-blocks
// x rt_box row tiles.  Boxes past the last k-block or row tile read zeros.
bool make_scale_map(CUtensorMap* map, const void* base, long rows_pad, long k_pad, int kb_box, int rt_box) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const long num_kb = k_pad / 64;
    const cuuint64_t dims[3] = {(cuuint64_t)(kAtomBytes / 8), (cuuint64_t)num_kb, (cuuint64_t)(rows_pad / 128)};
    const cuuint64_t strides[2] = {(cuuint64_t)kAtomBytes, (cuuint64_t)(kAtomBytes * num_kb)};
    const cuuint32_t box[3] = {(cuuint32_t)(kAtomBytes / 8), (cuuint32_t)kb_box, (cuuint32_t)rt_box};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// BF16 output D [m, n_out] with row stride ldd: 32 x 32 boxes with the 64-byte
// swizzle (single-GPU chunks), or (wide) 16-row x 64-column boxes (128-byte
// rows) with the 128-byte swizzle (column-parallel pieces).
bool make_output_map(CUtensorMap* map, void* base, long m, long n_out, long ldd, bool wide) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)n_out, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)(ldd * 2)};
    const cuuint32_t box[2] = {wide ? 64u : 32u, wide ? 16u : 32u};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

Params make_params(const GemmArgs& g, int bn, int tile_m) {
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
    p.bias_vec = (reinterpret_cast<uintptr_t>(g.bias) & 15) == 0 ? 1 : 0;
    p.tma_store = 0;
    const char* early_env = getenv("FP4B_EARLY_B");  // "0": every role waits for the preceding kernel
    p.b_early = (g.b_cached && !(early_env && atoi(early_env) == 0)) ? 1 : 0;
    p.n_tiles = (int)((g.n_out + bn - 1) / bn);
    p.m_tiles = (int)((g.m + tile_m - 1) / tile_m);
    p.num_tiles = p.n_tiles * p.m_tiles;
    return p;
}

// Clusters of two resident at once for a pair kernel (one CTA per SM).
template <typename K>
int max_pairs(K kernel, int smem, int sms, int threads) {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int& c = cached[dev & 63];
    if (c == 0) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
        cfg.blockDim = dim3(threads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (const void*)kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sms / 2;
        }
        c = n;
    }
    return c;
}

// Shared memory of one SM (233472 bytes on B200) minus a CTA's reserved 1 KB.
constexpr int kSmemPerSm = 233472;

template <int BN, int STAGES, bool AWAIT = false, int NSUB = 1, int BN1 = BN, bool PIECES = false, int CHUNKS = 1>
cudaError_t launch_pair(const GemmArgs& g, cudaStream_t stream, int sms, const QuantizeArgs* qa = nullptr,
                        uint32_t* ready = nullptr, void* const* peers = nullptr, int npeers = 0) {
    using C = PairCfg<BN, STAGES, NSUB, BN1, CHUNKS>;
    auto kernel = nvf4_gemm_pair_kernel<BN, STAGES, AWAIT, NSUB, BN1, PIECES, CHUNKS>;
    static std::once_flag attr_once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 63], [&] {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    CUtensorMap ma, mb, mb1, msa, msb, md, md64;
    if (!make_operand_map(&ma, g.a_fp4, g.m_rows_pad, g.k_pad, kBM) ||
        !make_operand_map(&mb, g.b_fp4, g.n_rows_pad, g.k_pad, C::BH) ||
        !make_operand_map(&mb1, g.b_fp4, g.n_rows_pad, g.k_pad, C::BH1) ||
        !make_scale_map(&msa, g.a_sf, g.m_rows_pad, g.k_pad, C::kKbPerStage, 1) ||
        !make_scale_map(&msb, g.b_sf, g.n_rows_pad, g.k_pad, C::kKbPerStage, C::NRT))
        return cudaErrorInvalidValue;
    Params p = make_params(g, C::TW, 2 * kBM);
    // D through TMA stores when C is not read and D's rows are 16-byte aligned.
    memset(&md, 0, sizeof(md));
    memset(&md64, 0, sizeof(md64));
    const bool no_c = !g.c || g.beta == 0.0f;
    const bool d_ok = (reinterpret_cast<uintptr_t>(g.d) & 15) == 0 && g.ldd % 8 == 0;
    if (no_c && d_ok && make_output_map(&md, g.d, g.m, g.n_out, g.ldd, false) &&
        make_output_map(&md64, g.d, g.m, g.n_out, g.ldd, true))
        p.tma_store = 1;
    PeerMaps pm;
    memset(&pm, 0, sizeof(pm));
    if constexpr (PIECES) {
        if (npeers > 0) {
            if (!p.tma_store || npeers > kMaxPeers) return cudaErrorNotSupported;
            for (int i = 0; i < npeers; ++i)
                if (!make_output_map(&pm.map[i], peers[i], g.m, g.n_out, g.ldd, true)) return cudaErrorNotSupported;
            p.npeers = npeers;
        }
    } else if (npeers > 0) {
        return cudaErrorNotSupported;  // peer stores need the column-parallel epilogue form
    }
    const int pairs = max_pairs(kernel, C::SMEM_BYTES, sms, kPairThreads);
    const int grid = 2 * (p.num_tiles < pairs ? p.num_tiles : pairs);
    if constexpr (AWAIT) {
        if (!qa || !ready) return cudaErrorInvalidValue;
        // One round of tiles, and room beside this kernel's CTA on an SM for a
        // quantizer CTA with at least 3 stages of 8 KB; else two kernels run.
        const int ring_room = kSmemPerSm - C::SMEM_BYTES - 2 * 1024 - quantize_units_smem_bytes(0);
        const int ring = ring_room / 8192 > 8 ? 8 : ring_room / 8192;
        if (p.num_tiles > pairs || ring < 3) return cudaErrorNotSupported;
        p.ready = ready;
        p.a_tiles128 = (int)(g.m_rows_pad / 128);
        p.a_stages = (int)((g.k_pad + 255) / 256);
        p.ready_count = p.a_tiles128 * p.a_stages;
        // The quantizer first (one CTA per SM), then this kernel behind it.
        const cudaError_t e = quantize_units_launch(*qa, ready, ring, sms, stream);
        if (e != cudaSuccess) return e;
        const cudaError_t e2 = launch_dependent(kernel, dim3(grid), dim3(kPairThreads), C::SMEM_BYTES, stream, ma,
                                                mb, mb1, msa, msb, md, md64, p, pm);
        if (e2 != cudaSuccess)  // the quantizer ran alone: leave the counters zero for the next launch
            cudaMemsetAsync(ready, 0, (size_t)(p.ready_count + 1) * sizeof(uint32_t), stream);
        return e2;
    }
    return launch_dependent(kernel, dim3(grid), dim3(kPairThreads), C::SMEM_BYTES, stream, ma, mb, mb1, msa, msb, md,
                            md64, p, pm);
}

template <int BN, int STAGES, int CHUNKS>
cudaError_t launch_tile(const GemmArgs& g, cudaStream_t stream, int sms) {
    using C = Cfg<BN, STAGES, CHUNKS>;
    auto kernel = nvf4_gemm_kernel<BN, STAGES, CHUNKS>;
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
    const Params p = make_params(g, BN, kBM);
    const int grid = p.num_tiles < sms ? p.num_tiles : sms;
    return launch_dependent(kernel, dim3(grid), dim3(kThreads), C::SMEM_BYTES, stream, ma, mb, p);
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

// Tile width of the CTA-pair kernel: the one with the smallest modelled time,
//   rounds x (stages x stage time + per-round overhead),
// rounds = ceil(tiles / pairs), a stage = K of 256 (the fixed cost is the same
// for every width).  Least-squares fit to back-to-back cached-linear steps on
// B200 over 15 shapes from 256x2880x2880 to 8192x15360x2880, every width
// (rms error 0.8 us; the pick is the measured best on 14 of them, 4.7 % off
// on the last): stage time 0.213 / 0.221 / 0.317 / 0.350 / 0.392 us and
// per-round overhead 0.61 / 1.23 / 1.88 / 2.72 / 2.60 us for BN = 128 / 192 /
// 256 / 320 (= 128 + 192, two MMAs per k-block on one A tile) / 384 (= 2 x
// 192).  The 128- and 192-wide tiles load two K chunks per stage, which makes
// the 192-wide one the choice for most multi-round shapes with K <= 4096
// (8192 x 5120 x 2880: 72.5 us against 79.5 with the 384-wide tile); the
// 320-wide one wins where its tiles need no more rounds (the headline: 72
// tiles on 74 pairs) and at long K; the 384-wide one on wide-N short-K
// shapes (8192 x 15360 x 2880: 180.8 us against 188.3 with 192).
// Returns 128, 192, 256, 320 (= 128 + 192) or 384 (= 2 x 192).
int choose_bn_pair(long m, long n, long k_pad, int sms) {
    struct Width { int code; double stage_us, round_us; };
    static const Width cands[] = {{384, 0.392, 2.60}, {320, 0.350, 2.72}, {256, 0.317, 1.88},
                                  {192, 0.221, 1.23}, {128, 0.213, 0.61}};
    const long mt = (m + 2 * kBM - 1) / (2 * kBM);
    const long pairs = sms / 2 > 0 ? sms / 2 : 1;
    const double stages = (double)((k_pad + 255) / 256);
    int best = 128;
    double best_cost = -1.0;
    for (const Width& w : cands) {
        const long tiles = mt * ((n + w.code - 1) / w.code);
        const long rounds = (tiles + pairs - 1) / pairs;
        const double cost = (double)rounds * (stages * w.stage_us + w.round_us);
        if (best_cost < 0.0 || cost < best_cost) {
            best_cost = cost;
            best = w.code;
        }
    }
    return best;
}

}  // namespace

cudaError_t gemm_launch_overlapped(const GemmArgs& g, const QuantizeArgs& qa, uint32_t* ready, cudaStream_t stream) {
    // Opt-in (FP4B_OVERLAP=1).  On B200 the quantizer CTA that fits beside a
    // GEMM CTA (at most ~12 K registers: four quantizing warps) cannot hide the
    // latency of its per-block work: alone it takes 28.8 us for the headline's
    // 2048 x 7680 activations (10.6 us for the standalone kernel with 40 warps
    // per SM), and the overlapped step took 68 us against 30.4 us for the two
    // kernels in turn.  Bytes are identical either way.
    const char* env = getenv("FP4B_OVERLAP");
    if (!env || atoi(env) == 0 || g.m <= kBM || (getenv("FP4B_PAIR") && atoi(getenv("FP4B_PAIR")) == 0))
        return cudaErrorNotSupported;
    if (qa.rows_pad != g.m_rows_pad || qa.k_pad != g.k_pad || qa.fp4 != g.a_fp4 || qa.sf != g.a_sf)
        return cudaErrorInvalidValue;
    if (quantize_units_check(qa)) return cudaErrorNotSupported;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const char* force = getenv("FP4B_FORCE_BN");
    const int bn = force ? atoi(force) : choose_bn_pair(g.m, g.n_out, g.k_pad, sms);
    // One stage fewer than the two-kernel instantiations, so that a quantizer
    // CTA fits beside the GEMM's CTA on every SM.
    switch (bn) {
        case 256: return launch_pair<256, 4, true>(g, stream, sms, &qa, ready);
        case 192: return launch_pair<192, 4, true>(g, stream, sms, &qa, ready);
        case 128: return launch_pair<128, 5, true>(g, stream, sms, &qa, ready);
        case 384: return launch_pair<192, 3, true, 2>(g, stream, sms, &qa, ready);
        case 320: return launch_pair<128, 3, true, 2, 192>(g, stream, sms, &qa, ready);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_launch_peers(const GemmArgs& g, void* const* peers, int npeers, cudaStream_t stream) {
    if (npeers < 1 || npeers > kMaxPeers) return cudaErrorNotSupported;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const char* force = getenv("FP4B_FORCE_BN");
    const int bn = force ? atoi(force) : choose_bn_pair(g.m, g.n_out, g.k_pad, sms);
    switch (bn) {
        case 256: return launch_pair<256, 5, false, 1, 256, true>(g, stream, sms, nullptr, nullptr, peers, npeers);
        case 192: return launch_pair<192, 3, false, 1, 192, true, 2>(g, stream, sms, nullptr, nullptr, peers, npeers);
        case 128: return launch_pair<128, 3, false, 1, 128, true, 2>(g, stream, sms, nullptr, nullptr, peers, npeers);
        case 384: return launch_pair<192, 4, false, 2, 192, true>(g, stream, sms, nullptr, nullptr, peers, npeers);
        case 320: return launch_pair<128, 4, false, 2, 192, true>(g, stream, sms, nullptr, nullptr, peers, npeers);
        default: return cudaErrorInvalidValue;
    }
}

int gemm_tile_width(long m, long n, long k_pad, int sms) {
    if (m <= 0 || n <= 0 || k_pad <= 0 || k_pad % 128 || sms < 2) return -1;
    return choose_bn_pair(m, n, k_pad, sms);
}

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
    // CTA pairs (256-row tiles) for every M: a pair splits each B tile between
    // two SMs, so even when the second CTA's rows are all padding (M <= 128;
    // its A loads read the tensor map's zero fill) the weight streams in over
    // twice the SMs -- 25-35 % faster than the one-CTA kernel at M = 1..128
    // (cached linears of N = 640..15360, K = 2880..7680 on B200), bytes equal.
    // FP4B_PAIR=0 selects the one-CTA kernel.
    const char* pair_env = getenv("FP4B_PAIR");
    const bool pair = pair_env ? atoi(pair_env) != 0 : true;
    if (pair) {
        const char* force = getenv("FP4B_FORCE_BN");
        const int bn = force ? atoi(force) : choose_bn_pair(g.m, g.n_out, g.k_pad, sms);
        // The 128- and 192-wide tiles load two K chunks per stage (3 stages of
        // 2 x 128-byte chunks instead of 6-7 of one: 4-15 % faster, most at small
        // M, where the weight streams from HBM; FP4B_KCHUNKS=1 selects one).  The
        // wider tiles keep one: two would leave them two stages (6-9 % slower).
        const char* kc_env = getenv("FP4B_KCHUNKS");
        const int kchunks = kc_env ? atoi(kc_env) : 2;
        switch (bn) {
            case 256: return launch_pair<256, 5, false>(g, stream, sms);
            case 192:
                return kchunks == 2 ? launch_pair<192, 3, false, 1, 192, false, 2>(g, stream, sms)
                                    : launch_pair<192, 6, false>(g, stream, sms);
            case 128:
                return kchunks == 2 ? launch_pair<128, 3, false, 1, 128, false, 2>(g, stream, sms)
                                    : launch_pair<128, 7, false>(g, stream, sms);
            case 384: return launch_pair<192, 4, false, 2>(g, stream, sms);
            case 320: return launch_pair<128, 4, false, 2, 192>(g, stream, sms);
            default: return cudaErrorInvalidValue;
        }
    }
    const char* force = getenv("FP4B_FORCE_BN");
    const int bn = force ? atoi(force) : choose_bn(g.m, g.n_out, sms);
    const char* stages_env = getenv("FP4B_DEEP");
    const bool deep = stages_env ? atoi(stages_env) != 0 : true;
    switch (bn) {
        case 256: return deep ? launch_tile<256, 4, 1>(g, stream, sms) : launch_tile<256, 2, 2>(g, stream, sms);
        case 192: return deep ? launch_tile<192, 4, 1>(g, stream, sms) : launch_tile<192, 2, 2>(g, stream, sms);
        case 128: return deep ? launch_tile<128, 6, 1>(g, stream, sms) : launch_tile<128, 3, 2>(g, stream, sms);
        case 64: return deep ? launch_tile<64, 7, 1>(g, stream, sms) : launch_tile<64, 3, 2>(g, stream, sms);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace fp4b
