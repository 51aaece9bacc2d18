// Cross-GPU barrier for the fused all-gather of O (one process per GPU).
//
// Each rank owns an array of flag words in device memory that every other
// rank has mapped (CUDA IPC): flags[r] is the last epoch rank r has signalled
// to this rank.  The barrier kernel runs on the stream after the attention
// kernel whose epilogue stored O tiles into the peers' outputs, so those
// stores are complete when it starts; it writes this call's epoch into its
// slot of every peer's array (release, system scope) and waits until every
// peer's epoch has arrived in its own array (acquire, system scope).  Work
// queued after it on the stream therefore sees every rank's stores.
//
// The waits are bounded (a peer that never arrives: the kernel records
// SITE_PEER_BARRIER in the status word and returns); the limit is long, since
// a live peer may legitimately be seconds behind.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sm100.cuh"

namespace rdna {
namespace peer {

constexpr int kMaxPeers = 7;
constexpr int SITE_PEER_BARRIER = 0x401;
constexpr uint64_t kBarrierLimitNs = 60ull * 1000000000ull;  // 60 s

struct BarrierParams {
    int world;                          // ranks (<= kMaxPeers + 1)
    int rank;                           // this rank's slot in every array
    unsigned int* peer_flags[kMaxPeers];  // the other ranks' arrays, in rank order without this rank
    unsigned int* my_flags;             // this rank's array (world words)
    unsigned int epoch;                 // this call's epoch (wraps; compared modulo 2^32)
    unsigned long long limit_ns;
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One block of 32 threads: thread i < world - 1 signals peer i, thread r !=
// rank waits for rank r.
__global__ void __launch_bounds__(32) barrier_kernel(BarrierParams p) {
    const int i = threadIdx.x;
    if (i < p.world - 1) {
        __threadfence_system();
        st_release_sys(p.peer_flags[i] + p.rank, p.epoch);
    }
    if (i < p.world && i != p.rank) {
        const uint64_t t0 = sm100::globaltimer_ns();
        while (static_cast<int>(ld_acquire_sys(p.my_flags + i) - p.epoch) < 0) {
            if (sm100::globaltimer_ns() - t0 > p.limit_ns) {
                atomicCAS(&g_rdna_status[0], 0, SITE_PEER_BARRIER);
                atomicAdd(&g_rdna_status[1], 1);
                break;
            }
            __nanosleep(64);
        }
    }
}

}  // namespace peer
}  // namespace rdna
