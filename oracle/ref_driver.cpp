/*
 * ref_driver.cpp -- host driver around the reference's own quantizer source.
 *
 * TEST INFRASTRUCTURE ONLY.  build_ref() in oracle/build.py compiles this file together
 * with the quantizer section of the reference's fp4_gemm_lib.cu (lines
 * 106-286: the E2M1/UE4M3 codecs, compute_sf_index and
 * quantize_bf16_to_fp4_kernel), which it includes as REF_QUANT_SOURCE.  The
 * result, oracle/_ref/libref_quant.so, executes the reference's code on the
 * CPU, so the C restatement in nvfp4_oracle.c can be checked against it and
 * golden vectors can be generated from it.
 */
#include "ref_shim.h"

#include REF_QUANT_SOURCE

extern "C" {

// Launch the reference kernel over its whole grid (fp4_gemm_lib.cu:523-527:
// 256 threads per block, one thread per 16-element scale block).
int ref_quantize(const uint16_t* src, int rows, int K, uint8_t* fp4, uint8_t* sf) {
    if (rows <= 0 || K <= 0 || K % 16) return -1;
    const int nsb = K / 16;
    const long total = (long)rows * nsb;
    const int threads = 256;
    const long blocks = (total + threads - 1) / threads;
#pragma omp parallel for schedule(static)
    for (long b = 0; b < blocks; ++b) {
        blockIdx.x = (unsigned)b;
        blockDim.x = threads;
        for (int t = 0; t < threads; ++t) {
            threadIdx.x = (unsigned)t;
            quantize_bf16_to_fp4_kernel(reinterpret_cast<const __nv_bfloat16*>(src), fp4, sf, rows, K, nsb);
        }
    }
    return 0;
}

uint8_t ref_float_to_fp4(float v) { return d_float_to_fp4(v); }
uint8_t ref_float_to_ue4m3(float v) { return d_float_to_ue4m3(v); }
float ref_ue4m3_to_float(uint8_t raw) { return d_ue4m3_to_float(raw); }
int ref_sf_index(int r, int kb, int rows, int nsb) { return compute_sf_index(r, kb, rows, nsb); }

}  // extern "C"
