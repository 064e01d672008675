// selftest.cu -- exercises the kernels' failure path without faulting the GPU.
//
// Every wait in this library's kernels is bounded (ptx::mbar_wait and
// ptx::wait_counter_geq give up after kSpinLimitNs, 2 s): the waiting role
// then records a code in the device error word and the kernel returns, so the
// context stays usable and the host reads the code with fp4b_device_error.
// fp4b_selftest_bounded_wait launches one block that waits, with those same
// helpers, on something that nothing completes -- an mbarrier phase that no
// thread arrives on, or a global word that no code writes -- so that a test
// can check that the wait gives up, that its code reaches the host, and that
// later work runs normally.  Nothing here traps, faults or spins unbounded.
#include <cuda_runtime.h>

#include "fp4b_internal.h"
#include "ptx_sm100.cuh"

#define FP4B_EXPORT extern "C" __attribute__((visibility("default")))

namespace fp4b {
namespace {

constexpr int kErrSelftestBarrier = 7;  // device error word: the self-test's barrier wait gave up
constexpr int kErrSelftestCounter = 8;  // device error word: the self-test's counter wait gave up

__device__ uint32_t g_never_set;  // zero; no code writes it

__global__ void bounded_wait_selftest_kernel(int which, int* err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    // A fresh barrier is in phase 0, which completes only after one arrival.
    const bool ok = which == 0 ? ptx::mbar_wait(&bar, 0) : ptx::wait_counter_geq(&g_never_set, 1u);
    if (!ok && err) atomicCAS(err, 0, which == 0 ? kErrSelftestBarrier : kErrSelftestCounter);
}

}  // namespace
}  // namespace fp4b

using namespace fp4b;

FP4B_EXPORT int fp4b_selftest_bounded_wait(int which, void* stream) {
    if (which != 0 && which != 1) {
        set_last_error("fp4b_selftest_bounded_wait: which must be 0 (barrier) or 1 (counter)");
        return -1;
    }
    int* err = device_error_word();
    if (!err) {
        set_last_error("fp4b_selftest_bounded_wait: no device error word on this device");
        return -4;
    }
    bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(which, err);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("fp4b_selftest_bounded_wait: launch: %s", cudaGetErrorString(e));
        return -4;
    }
    return 0;
}
