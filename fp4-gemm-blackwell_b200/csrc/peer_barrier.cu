// peer_barrier.cu -- the rank-ordering step of the column-parallel linear.
//
// After a rank's GEMM has stored its output columns into every rank's buffer
// (NVLink stores from the epilogue), the ranks must not read their buffers
// before every peer's GEMM has finished.  fp4b_peer_barrier does this with one
// warp on the GPU instead of a collective: thread i release-stores `epoch` into
// slot [my_rank] of peer i's flag array (mapped into this process with CUDA
// IPC), then waits until slot [peer_rank[i]] of this rank's own flag array has
// reached `epoch`.  Launched on the stream right after the GEMM, so the GEMM's
// stores precede the signal; the work after it on the stream sees every
// peer's stores.  It is launched with programmatic stream serialization: the
// block is placed while the GEMM still runs and waits (griddepcontrol.wait)
// for the GEMM grid to complete, which saves a kernel launch gap per linear;
// the kernel behind it may be placed early the same way and waits for this
// one to complete.  Epochs only grow (every rank counts its calls the same way),
// so a flag array is never reset.  The wait is bounded: after kPeerWaitNs
// (10 s: the peers' hosts may run some seconds behind, e.g. while they build
// their caches) it records kErrPeerBarrierTimeout in the device error word and
// the kernel returns, so a rank that never arrives cannot hang the GPU.
#include <cuda_runtime.h>

#include <cstdint>

#include "fp4b_internal.h"
#include "ptx_sm100.cuh"

#define FP4B_EXPORT extern "C" __attribute__((visibility("default")))

namespace fp4b {
namespace {

constexpr int kMaxBarrierPeers = 7;
constexpr int kErrPeerBarrierTimeout = 10;  // device error word: a peer never signalled
constexpr uint64_t kPeerWaitNs = 10000000000ull;

struct PeerFlags {
    unsigned long long* flags[kMaxBarrierPeers];  // peer i's flag array (mapped)
    int rank[kMaxBarrierPeers];                   // peer i's rank
};

__global__ void peer_barrier_kernel(const unsigned long long* my_flags, const __grid_constant__ PeerFlags pf,
                                    int npeers, int my_rank, unsigned long long epoch, int* err) {
    ptx::grid_dependency_wait();  // the GEMM before this kernel has completed
    ptx::launch_dependents();
    const int i = threadIdx.x;
    if (i >= npeers) return;
    // Everything this GPU wrote before (the GEMM's stores into the peers'
    // buffers) is visible system-wide before the flag.
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(pf.flags[i] + my_rank), "l"(epoch) : "memory");
    const unsigned long long* slot = my_flags + pf.rank[i];
    const uint64_t t0 = ptx::global_timer_ns();
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(slot) : "memory");
        if (v >= epoch) break;
        if (ptx::global_timer_ns() - t0 > kPeerWaitNs) {
            if (err) atomicCAS(err, 0, kErrPeerBarrierTimeout);
            break;
        }
        __nanosleep(64);
    }
}

}  // namespace
}  // namespace fp4b

using namespace fp4b;

FP4B_EXPORT int fp4b_peer_barrier(const void* my_flags, void* const* peer_flags, const int* peer_ranks, int npeers,
                                  int my_rank, unsigned long long epoch, void* stream) {
    if (!my_flags || !peer_flags || !peer_ranks || npeers < 1 || npeers > kMaxBarrierPeers || my_rank < 0 ||
        my_rank > kMaxBarrierPeers || epoch == 0 || (reinterpret_cast<uintptr_t>(my_flags) & 7)) {
        set_last_error("fp4b_peer_barrier: bad arguments (1..7 peers, rank 0..7, epoch > 0, 8-byte aligned flags)");
        return -1;
    }
    PeerFlags pf{};
    for (int i = 0; i < npeers; ++i) {
        if (!peer_flags[i] || (reinterpret_cast<uintptr_t>(peer_flags[i]) & 7) || peer_ranks[i] < 0 ||
            peer_ranks[i] > kMaxBarrierPeers || peer_ranks[i] == my_rank) {
            set_last_error("fp4b_peer_barrier: bad peer %d", i);
            return -1;
        }
        pf.flags[i] = static_cast<unsigned long long*>(peer_flags[i]);
        pf.rank[i] = peer_ranks[i];
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return launch_status(cudaLaunchKernelEx(&cfg, peer_barrier_kernel, static_cast<const unsigned long long*>(my_flags),
                                            pf, npeers, my_rank, epoch, device_error_word()),
                         "fp4b_peer_barrier launch");
}
