/*
 * ref_shim.h -- lets the reference quantizer's CUDA source compile as host C++.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle/build.py, build_ref).  The reference's
 * quantizer (fp4_gemm_lib.cu:106-286 of VincentKaufmann/fp4-gemm-blackwell)
 * uses only CUDA qualifiers, the bf16->fp32 conversion and libm.  This header
 * maps the qualifiers to host C++, supplies a bit-exact bf16->fp32 conversion
 * and per-thread grid coordinates, so the reference's own kernel body can be
 * run on the CPU one (block, thread) pair at a time.
 */
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#define __device__
#define __forceinline__ inline
#define __constant__ static const
#define __global__ static
#define __restrict__ __restrict

using std::max;
using std::min;

struct ref_uint3 {
    unsigned x, y, z;
};
// Grid coordinates of the emulated CUDA thread (one copy per host thread).
static thread_local ref_uint3 blockIdx, threadIdx, blockDim;

struct __nv_bfloat16 {
    uint16_t bits;
};

// Exact: bf16 is the top half of an fp32.
static inline float __bfloat162float(__nv_bfloat16 h) {
    uint32_t u = (uint32_t)h.bits << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
