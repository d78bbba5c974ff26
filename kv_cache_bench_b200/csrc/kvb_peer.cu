// Step barrier of a sharded decode step whose kernel wrote its output rows into every rank's global
// output buffer over peer memory (kvb_paged_decode_gather_async). One CTA of one warp per rank:
//   1. griddepcontrol.wait: the decode kernel before it on the stream has completed, and its stores
//      (local and remote) are performed;
//   2. the rank's epoch (a word of its own device memory) counts up by one;
//   3. lane j stores the epoch into word `rank` of rank j's signal array (system-scope release, after
//      a system-scope fence), which orders the decode's row stores before the signal for every
//      observer;
//   4. lane j waits until word j of this rank's own signal array reached the epoch (system-scope
//      acquire): rank j's rows are then in this rank's buffer.
// Every rank launches the barrier once per step, so the epochs of all ranks move together. A word
// can run ahead of this rank's epoch by at most one step (that rank passed this barrier and signalled
// the next one), so the test is "reached", in wrap-around arithmetic. The wait is bounded by the
// global timer: past timeout_ns it raises KVB_DEVERR_TIMEOUT in the workspace's error word and
// returns, so a rank that never arrives costs a flag and not a hung GPU.
// The kernel lets the next kernel on the stream launch at entry (programmatic dependent launch): the
// next decode step streams its pages while this one waits, and waits for this kernel's completion
// before its first workspace or output store.
#include <cuda_runtime.h>

#include "kvb_internal.h"

namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const PeerBarrierParams p) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x;
    unsigned e = 0;
    if (lane == 0) {
        e = *p.epoch + 1u;
        *p.epoch = e;
    }
    e = __shfl_sync(0xffffffffu, e, 0);
    __threadfence_system();
    unsigned* const mine = p.signal[p.rank];
    if (lane < p.n_peers) st_release_sys(p.signal[lane] + p.rank, e);
    bool ok = true;
    if (lane < p.n_peers) {
        const unsigned long long t0 = global_ns();
        while (static_cast<int>(ld_acquire_sys(mine + lane) - e) < 0) {
            if (global_ns() - t0 > p.timeout_ns) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!__all_sync(0xffffffffu, ok) && lane == 0) atomicOr(p.error_flag, KVB_DEVERR_TIMEOUT);
}

}  // namespace

cudaError_t kvb_launch_peer_barrier(const PeerBarrierParams& p, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, peer_barrier_kernel, p);
}
