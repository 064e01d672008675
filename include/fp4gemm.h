/*
 * fp4gemm.h -- C ABI of libfp4gemm.so, the B200 (sm_100a) NVFP4 linear-layer
 * library.  Drop-in for the shared library of VincentKaufmann/fp4-gemm-blackwell:
 * the first block of functions keeps the reference's exported symbols, argument
 * meaning, return codes and synchronisation behaviour (citations are file:line in
 * that project); the fp4b_* block is additive.
 *
 * Conventions shared by every entry point:
 *   - all tensors are device pointers to contiguous row-major data; BF16 is
 *     IEEE bfloat16 bits; no torch or CUDA C++ types appear in the signatures;
 *   - NVFP4 operand = packed E2M1 [rows, K/2] (even element in the low nibble)
 *     plus UE4M3 scales, one per 16 elements, in the 128-row x 4-block
 *     interleaved layout: byte offset of (row r, block kb) =
 *       (r%32)*16 + ((r/32)%4)*4 + kb%4 + (kb/4)*512 + (r/128)*512*(K/64);
 *   - quantization semantics are the reference kernel's (fp4_gemm_lib.cu:107-286):
 *     scale = UE4M3(absmax/6) clamped to [2^-9, 480], elements rounded to the
 *     nearest E2M1 value with ties to the lower magnitude;
 *   - reference entry points run on the legacy default stream like the reference;
 *     fp4b_* entry points take a cudaStream_t as `void* stream` (NULL = legacy default).
 */
#ifndef FP4GEMM_H
#define FP4GEMM_H

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------------------
 * Reference ABI (fp4_gemm_lib.cu:401-842; bound by fp4_gemm.py:30-87)
 * ------------------------------------------------------------------------- */

/* Elements per scale factor: 16.  fp4_gemm_lib.cu:403, read by fp4_gemm.py:87. */
int fp4_gemm_sf_vec_size(void);

/* Size the library's scratch (quantized A/B) for an M x N x K problem.
 * 0 on success; -1 if a reallocation is needed and M, N or K is not a multiple
 * of 128.  A call whose shape fits the current scratch only records the shape.
 * fp4_gemm_lib.cu:435-500 (bound at fp4_gemm.py:33-34). */
int fp4_gemm_init(int M, int N, int K);

/* Same as fp4_gemm_init with the maximum shape.  fp4_gemm_lib.cu:503-505
 * (fp4_gemm.py:52-53). */
int fp4_gemm_prealloc(int max_M, int max_N, int max_K);

/* D = alpha * q(A) @ q(B)^T + beta * C with A [M,K], B [N,K], C/D [M,N] BF16;
 * C may be NULL (then D is the source, as in the reference).  M, N, K multiples
 * of 128.  Quantizes both operands, runs the GEMM, then synchronises the
 * device.  0 ok; -1 shape/allocation; -2 cannot implement; -4 launch failure.
 * fp4_gemm_lib.cu:508-585 (fp4_gemm.py:36-47). */
int fp4_gemm_run(const void* A_bf16, const void* B_bf16, const void* C_bf16, void* D_bf16, int M, int N, int K,
                 float alpha, float beta);

/* Reference host-quantization variant (fp4_gemm_lib.cu:588-650, exported but not
 * bound in fp4_gemm.py).  Its CUTLASS host conversion differs from the device
 * quantizer; this library does not provide it and returns -2. */
int fp4_gemm_run_host(const void* A_bf16, const void* B_bf16, const void* C_bf16, void* D_bf16, int M, int N,
                      int K, float alpha, float beta);

/* Free the scratch of the current device.  fp4_gemm_lib.cu:652 (fp4_gemm.py:49-50). */
void fp4_gemm_cleanup(void);

/* cudaDeviceSynchronize().  fp4_gemm_lib.cu:655 (fp4_gemm.py:55-56). */
void fp4_gemm_sync(void);

/* Quantize a BF16 weight [N, K] once into a device-resident cache; N, K
 * multiples of 128.  Returns an opaque handle or NULL (bad shape, allocation
 * failure).  Synchronises the device.  fp4_gemm_lib.cu:672-720
 * (fp4_gemm.py:59-64). */
void* fp4_quantize_weights(const void* weight_bf16, int N, int K);

/* Device pointers of the cached packed E2M1 data [N, K/2] and scales (N*K/16
 * bytes); NULL for a NULL handle.  fp4_gemm_lib.cu:723-732 (unbound in Python). */
const void* fp4_weight_cache_fp4_ptr(const void* cache_handle);
const void* fp4_weight_cache_sf_ptr(const void* cache_handle);

/* Cached (padded) shape; 0 for NULL.  fp4_gemm_lib.cu:735-741 (fp4_gemm.py:69-73). */
int fp4_weight_cache_N(const void* cache_handle);
int fp4_weight_cache_K(const void* cache_handle);

/* Release a cache; NULL-safe.  fp4_gemm_lib.cu:744-750 (fp4_gemm.py:66-67). */
void fp4_weight_cache_free(void* cache_handle);

/* D[M, N] = alpha * q(A) @ W^T + beta * C with A [M, K] BF16 and W the cached
 * weight (N, K of the cache); M a multiple of 128.  Does not synchronise.
 * 0 ok; -1 NULL handle / bad M / allocation; -2 cannot implement; -4 launch
 * failure.  fp4_gemm_lib.cu:754-840 (fp4_gemm.py:75-84). */
int fp4_gemm_run_cached(const void* A_bf16, const void* cache_handle, const void* C_bf16, void* D_bf16, int M,
                        float alpha, float beta);

/* ----------------------------------------------------------------------------
 * Additive ABI (no counterpart in the reference)
 * ------------------------------------------------------------------------- */

/* Library ABI version (1). */
int fp4b_version(void);

/* Output columns per tile the GEMM picks for an M x N x K problem (K padded to
 * 128) on a device with `sms` SMs, from its time model and without the
 * FP4B_PAIR / FP4B_FORCE_BN overrides: 128 / 192 / 256 (one MMA per k-block),
 * 320 (128 + 192) or 384 (192 + 192), on CTA pairs at every M.  -1 on bad
 * arguments.  Host only: no device work, no GPU needed. */
int fp4b_gemm_tile_width(int m, int n, int k, int sms);

/* Message of the last failed call on this host thread ("" if none). */
const char* fp4b_last_error(void);

/* Non-zero if a kernel on the current device gave up on a bounded wait: the
 * first code recorded (GEMM 1 producer, 2 MMA, 3 epilogue, 4 fused-quantize
 * wait; 5 quantizer ring; 7 / 8 the self-test below; 9 fp4b_mma_rate's final
 * wait; 10 fp4b_peer_barrier); clear != 0 resets it.
 * Synchronises the device. */
int fp4b_device_error(int clear);

/* Failure-path self-test (no counterpart in the reference, whose kernels do
 * not wait): one block waits, with the bounded waits the kernels use, on an
 * mbarrier phase nobody completes (which = 0) or a global word nobody writes
 * (which = 1); after the 2 s bound the wait gives up, records 7 or 8 in the
 * device error word and the kernel returns, leaving the context usable.
 * Asynchronous on `stream`; 0, or -1 bad `which`, -4 launch failure. */
int fp4b_selftest_bounded_wait(int which, void* stream);

/* Measured tensor-pipe rate of the block-scaled NVFP4 MMA (no counterpart in
 * the reference): launches one CTA pair per two SMs whose even CTA issues
 * `stages` x 4 k-blocks of tcgen05.mma.cta_group::2.kind::mxf4nvf4 (M = 256,
 * K = 64) on operands resident in shared memory -- no loads.  Per k-block: an
 * MMA of width n0 and, if n1 > 0, a second of width n1 on the same A tile
 * (n0, n1 multiples of 64 in [64, 256], n0 + n1 <= 384); with sf_copies != 0
 * also the tcgen05.cp scale copies of the GEMM mainloop (1 atom for A and
 * sfb_atoms (0..3) for B per k-block).  FLOPs = pairs x stages x 4 x 2 x 256 x
 * (n0 + n1) x 64, with *pairs_out the pairs launched; the caller times the
 * launch on `stream` (n0 = 256, n1 = 0, no copies: the dense NVFP4 peak).
 * Asynchronous; 0, -1 bad arguments (stages in 1..2^20), -4 launch failure. */
int fp4b_mma_rate(int n0, int n1, int sf_copies, int sfb_atoms, int stages, int* pairs_out, void* stream);

/* Quantize BF16 [rows, cols] (row stride ld elements) into caller buffers:
 * dst_fp4 [rows_pad, k_pad/2], dst_sf rows_pad*k_pad/16 bytes.  Positions
 * outside [rows, cols) quantize as zeros, which reproduces the reference's
 * torch.zeros padding (fp4_gemm.py:146-160).  rows_pad, k_pad multiples of
 * 128.  Asynchronous on `stream`.  0 ok, -1 bad arguments, -4 launch failure. */
int fp4b_quantize(const void* src_bf16, int rows, int cols, int ld, void* dst_fp4, void* dst_sf, int rows_pad,
                  int k_pad, void* stream);

/* GEMM on already-quantized operands: D[m, n_out] = alpha * A @ B^T + beta * C,
 * rounded to BF16, then + bias[n] (BF16, may be NULL) rounded to BF16 again --
 * the reference's order (fp4_gemm.py:223-224, 389-390).  A has m_rows_pad
 * rows, B n_rows_pad rows, both k_pad wide (multiples of 128).  C may be NULL.
 * Asynchronous.  0 ok, -1 bad arguments, -4 launch failure. */
int fp4b_gemm_prequant(const void* a_fp4, const void* a_sf, int m, int m_rows_pad, const void* b_fp4,
                       const void* b_sf, int n_out, int n_rows_pad, int k_pad, const void* C_bf16, int ldc,
                       void* D_bf16, int ldd, const void* bias_bf16, float alpha, float beta, void* stream);

/* Cached linear on unpadded shapes, the fast path behind FP4WeightCache.forward:
 * A [m, k_in] (row stride lda) with k_in <= the cache's K, D [m, n_out]
 * (row stride ldd) with n_out <= the cache's N, optional C (ldc) and bias [n_out].
 * Same values as the reference's pad -> fp4_gemm_run_cached -> unpad -> bias
 * sequence (fp4_gemm.py:324-394), without the pad/unpad copies.  Uses the
 * per-device scratch; asynchronous on `stream`.  0 ok; -1 bad arguments or
 * allocation failure; -2 a geometry the kernels cannot take; -4 launch failure. */
int fp4b_run_cached_ex(const void* A_bf16, int m, int k_in, int lda, const void* cache_handle, int n_out,
                       const void* C_bf16, int ldc, void* D_bf16, int ldd, const void* bias_bf16, float alpha,
                       float beta, void* stream);

/* Dynamic GEMM on unpadded shapes (fp4_matmul / fp4_linear, fp4_gemm.py:95-228):
 * A [m, k] (lda), B [n, k] (ldb) BF16, both quantized per call into the
 * per-device scratch.  Asynchronous on `stream` (the reference synchronises;
 * fp4_gemm.py's wrapper keeps that by calling fp4_gemm_sync()). */
int fp4b_run_ex(const void* A_bf16, int m, int k, int lda, const void* B_bf16, int n, int ldb, const void* C_bf16,
                int ldc, void* D_bf16, int ldd, const void* bias_bf16, float alpha, float beta, void* stream);

/* Weight cache from an unpadded BF16 weight [n, k] (row stride ldw): the cache
 * is [round_up(n,128), round_up(k,128)] and its bytes equal those of
 * fp4_quantize_weights on the zero-padded weight (fp4_gemm.py:296-314).
 * sync != 0 synchronises the device like the reference.  NULL on failure. */
void* fp4b_quantize_weights_ex(const void* weight_bf16, int n, int k, int ldw, void* stream, int sync);

/* A cache handle that views rows [row0, row0 + rows) of another cache (row0
 * and rows multiples of 128) without copying: the N-shard of a column-parallel
 * linear.  The view must be freed with fp4_weight_cache_free before its parent.
 * NULL on failure. */
void* fp4b_weight_cache_slice(const void* cache_handle, int row0, int rows);

/* Global weight scale (two-level NVFP4; no counterpart in the reference): a
 * cache built from weight * s instead of weight carries w_alpha = 1 / s, and
 * every GEMM with it (fp4_gemm_run_cached and the fp4b_run_cached_* entry
 * points) multiplies its alpha by w_alpha.  Caches start at 1 (the reference's
 * bytes); slices inherit their parent's factor.  set: 0, or -1 for a bad
 * handle or a factor that is not positive and finite.  get: 0 for a bad handle. */
int fp4b_weight_cache_set_alpha(void* cache_handle, float w_alpha);
float fp4b_weight_cache_alpha(const void* cache_handle);

/* Copy a cache's bytes (packed E2M1 N*K/2, then scales N*K/16; N, K from the
 * getters) into caller device buffers, asynchronously on `stream`: the payload
 * of a serialised weight cache.  0 ok, -1 bad arguments, -4 copy failure. */
int fp4b_weight_cache_export(const void* cache_handle, void* dst_fp4, void* dst_sf, void* stream);

/* Build a cache of padded shape [N, K] (multiples of 128) from bytes produced by
 * fp4b_weight_cache_export (device pointers); copies them and synchronises
 * `stream`.  NULL on failure. */
void* fp4b_weight_cache_import(const void* src_fp4, const void* src_sf, int N, int K, void* stream);

/* fp4b_run_cached_ex without any device allocation (no counterpart in the
 * reference).  For callers that may not let a library allocate: a serving
 * engine that has given nearly all of HBM to its own allocator, or a pipeline
 * that cannot take the device-wide wait that cudaFree implies.  The quantized
 * activations go to a fixed 9 MiB array that is part of the library's device
 * code (16 Mi padded elements: round_up(m,128) * the cache's K must not exceed
 * 16777216, else -1 with a message).  The first call on a device looks up that
 * array's device address, so make it before capturing work into a CUDA graph;
 * if that lookup fails the call returns -1, as an allocation failure does in
 * fp4b_run_cached_ex.  All calls on a device share the array: calls that
 * overlap on the GPU race.  Arguments, results and the other return codes as
 * fp4b_run_cached_ex. */
int fp4b_run_cached_noalloc(const void* A_bf16, int m, int k_in, int lda, const void* cache_handle, int n_out,
                            const void* C_bf16, int ldc, void* D_bf16, int ldd, const void* bias_bf16, float alpha,
                            float beta, void* stream);

/* Column-parallel cached linear (no counterpart in the reference, which runs
 * on one device): this rank's output columns [m, n_out] are written to D and,
 * by the GEMM epilogue itself, to the npeers (1..7) buffers peer_d[] (other
 * GPUs' [.., ldd] BF16 outputs mapped with fp4b_ipc_open_handle, each already
 * offset to this rank's first column) with NVLink stores.  The caller orders
 * the ranks after the call (fp4b_peer_barrier on the same stream, or a
 * collective).  No C.  D and every peer_d[i] must be 16-byte aligned
 * and ldd a multiple of 8 elements (the epilogue stores 16 bytes at a time);
 * otherwise -2 before any device work.  Asynchronous on `stream`; other return
 * codes as fp4b_run_cached_ex. */
int fp4b_run_cached_peers(const void* A_bf16, int m, int k_in, int lda, const void* cache_handle, int n_out,
                          void* D_bf16, int ldd, void* const* peer_d, int npeers, const void* bias_bf16,
                          void* stream);

/* The ranks' ordering step after fp4b_run_cached_peers (no counterpart in the
 * reference): one GPU warp release-stores `epoch` into slot my_rank of each
 * peer's flag array (peer_flags[i], the peer's array of 8 u64 slots mapped with
 * fp4b_ipc_open_handle), then waits until slot peer_ranks[i] of this rank's own
 * array `my_flags` holds at least `epoch`.  Call it on the stream of the GEMM,
 * right after it, with the same epoch on every rank (a per-call counter that
 * starts at 1 and only grows; the arrays start zeroed and are never reset).
 * Work queued after it sees every peer's output columns.  The wait gives up
 * after 10 s, recording 10 in the device error word (fp4b_device_error).
 * Asynchronous; 0, -1 bad arguments (1..7 peers, ranks 0..7, 8-byte aligned
 * arrays), -4 launch failure. */
int fp4b_peer_barrier(const void* my_flags, void* const* peer_flags, const int* peer_ranks, int npeers,
                      int my_rank, unsigned long long epoch, void* stream);

/* One strided device-to-device copy (cudaMemcpy2DAsync): `height` rows of
 * `width_bytes`, row pitches in bytes; either side may be another GPU's
 * memory mapped with fp4b_ipc_open_handle, in which case the copy engine moves
 * it over NVLink.  The column-parallel linear pushes its output columns to the
 * other ranks with it (no counterpart in the reference).  Asynchronous on
 * `stream`; 0, -1 bad arguments, -4 failure. */
int fp4b_copy2d(void* dst, long dpitch, const void* src, long spitch, long width_bytes, long height, void* stream);

/* CUDA IPC for the peer buffers (no counterpart in the reference): the 64-byte
 * handle of the allocation holding `ptr` and ptr's offset in it; opening maps
 * another process's allocation into this one and returns base + offset. */
int fp4b_ipc_get_handle(const void* ptr, void* handle_out, long* offset_out);
void* fp4b_ipc_open_handle(const void* handle, long offset);
int fp4b_ipc_close(void* ptr, long offset);

#ifdef __cplusplus
}
#endif

#endif /* FP4GEMM_H */
