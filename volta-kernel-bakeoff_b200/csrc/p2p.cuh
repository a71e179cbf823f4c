// Peer-memory (NVLink) output exchange for the fused multi-GPU kernels: each rank's kernel stores its part of the
// output straight into every rank's copy of a symmetric buffer (same size and layout on every rank, mapped into
// every peer by CUDA IPC), ordered by per-call epochs in a flags block that follows the data in the buffer:
//
//   flags[P2P_READY + p] = e   rank p has started call e on its stream (its earlier work, which may still read
//                              this buffer, is done), so call e may write into rank p's buffer
//   flags[P2P_DONE + p]  = e   every store of rank p's call e into this buffer is visible
//   flags[P2P_COUNT]           this rank's count of CTAs that finished call e (local)
//
// Protocol of call e (all waits bounded by time; a timeout raises DEV_ERR_PEER_TIMEOUT and gives up):
//   1. after griddepcontrol.wait, one thread posts READY[rank] = e into every peer's flags (release, system scope);
//   2. before its first remote store a warp waits until READY[p] >= e for every peer p in its own flags (acquire);
//   3. every CTA: fence.acq_rel.sys, then an atomic count; the last CTA posts DONE[rank] = e into every peer and
//      waits until DONE[p] >= e for every p, so the call's kernel ends only when the whole output is in place.
// Epochs only grow (the host numbers the calls of a buffer from 1), so the flags never need resetting.
#pragma once

#include "ptx.cuh"

namespace vkb {

constexpr int P2P_MAX_RANKS = 8;
constexpr int P2P_READY = 0;                      // [P2P_MAX_RANKS]
constexpr int P2P_DONE = P2P_MAX_RANKS;           // [P2P_MAX_RANKS]
constexpr int P2P_COUNT = 2 * P2P_MAX_RANKS;      // CTA counter of the current call
constexpr int P2P_FLAG_WORDS = 64;                // flags block: 256 bytes after the data

struct P2PArgs {
    void* peer_base[P2P_MAX_RANKS];        // the symmetric buffer on every rank (peer_base[rank] = this rank's)
    uint32_t* peer_flags[P2P_MAX_RANKS];   // its flags block on every rank
    int rank, size;
    uint32_t epoch;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Wait until flag >= e (epochs grow monotonically; the comparison is wrap-safe). Bounded.
__device__ __forceinline__ bool p2p_wait_flag(const uint32_t* flag, uint32_t e) {
    if ((int)(ld_acquire_sys(flag) - e) >= 0) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
        if ((int)(ld_acquire_sys(flag) - e) >= 0) return true;
        if ((i & 63u) == 63u) {
            if (globaltimer() - t0 > VKB_WAIT_NS) {
                raise_status(DEV_ERR_PEER_TIMEOUT);
                return false;
            }
            __nanosleep(256);
        }
    }
}

// Step 1 (one thread, after griddepcontrol.wait): this rank may now be written by call e.
__device__ __forceinline__ void p2p_post_ready(const P2PArgs& p) {
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank) st_release_sys(p.peer_flags[r] + P2P_READY + p.rank, p.epoch);
}

// Step 2 (any thread; lane 0 of a warp, then __syncwarp): every peer accepts writes of call e.
__device__ __forceinline__ bool p2p_wait_ready(const P2PArgs& p) {
    const uint32_t* f = p.peer_flags[p.rank];
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank && !p2p_wait_flag(f + P2P_READY + r, p.epoch)) return false;
    return true;
}

// Step 3 (every CTA, after __syncthreads that follows all of its stores; thread 0 only).
__device__ __forceinline__ void p2p_finish(const P2PArgs& p) {
    fence_acq_rel_sys();   // this CTA's stores (local and remote) before its count
    uint32_t* f = p.peer_flags[p.rank];
    const uint32_t old = atomicAdd(f + P2P_COUNT, 1u);
    if (old != gridDim.x - 1) return;
    f[P2P_COUNT] = 0;      // every CTA of this call has counted; the next call starts from zero
    fence_acq_rel_sys();
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank) st_release_sys(p.peer_flags[r] + P2P_DONE + p.rank, p.epoch);
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank && !p2p_wait_flag(f + P2P_DONE + r, p.epoch)) return;
}

}  // namespace vkb
