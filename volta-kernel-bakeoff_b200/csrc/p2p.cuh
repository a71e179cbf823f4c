// Peer-memory (NVLink) output exchange for the fused multi-GPU kernels: each rank's kernel stores its part of the
// output straight into every rank's copy of a symmetric buffer (same size and layout on every rank, mapped into
// every peer by CUDA IPC), ordered by per-call epochs in a flags block that every rank of the communicator shares
// (one block per communicator, also mapped into every peer; every fused call of the communicator is numbered in it).
//
// The kernels store their results into this rank's copy as on one GPU; as soon as a region (a tile) is complete,
// the warps that wrote it push it to every peer with wide vector copies (p2p_push), overlapping the copies with the
// CTA's next tiles. NVLink moves large writes far faster than the scattered 2-byte stores of an epilogue.
//
// Every rank launches the same grid for a call (the calls have equal shapes on every rank, and the grid depends only
// on the shape and the device's SM count); CTA b of one rank pairs with CTA b of every other rank for READY. Flags of
// the block (32-bit words; epochs are 31-bit counters compared modulo 2^31):
//
//   READY[p][b] = e   CTA b of rank p has started call e (rank p's earlier work, which may still read its buffers,
//                     is complete), so call e may write into rank p's buffer
//   DONE[p]     = e   every store of rank p's call e is visible; with the high bit set (P2P_FAIL_MARK) rank p's part
//                     of call e is missing (one of its waits gave up, or the rank refused the call on the host)
//   COUNT             CTAs of this rank that finished the current call (local)
//   EPOCH             the last call completed on this rank (local)
//   FAILED            some CTA of this rank's current call failed (local)
//
// Call e on rank r (all waits bounded by time; a timeout raises DEV_ERR_PEER_TIMEOUT and gives up):
//   1. after griddepcontrol.wait every CTA b reads e = EPOCH + 1 and posts READY[r][b] = e into every peer (relaxed
//      system-scope store: it orders nothing but the end of this rank's earlier kernels, which the grid dependency
//      already did);
//   2. before its first push a warp waits until READY[p][b] >= e for every peer p (in this rank's flags); a warp whose
//      wait gave up pushes nothing;
//   3. after a barrier that follows all of its stores, one thread of every CTA records whether the CTA failed
//      (FAILED), makes a GPU-scope release (fence.acq_rel.gpu, cumulative over the barrier) and counts the CTA; the
//      last CTA acquires the others (fence.acq_rel.sys, which also releases the whole grid's stores to the system),
//      posts DONE[r] = e, marked if any CTA failed, into every peer (relaxed) and waits (acquire) until DONE[p] >= e
//      for every peer p, then stores EPOCH = e. A marked DONE[p] raises DEV_ERR_PEER_FAILED: this rank's copy lacks
//      rank p's part, and vkb_device_status says so instead of the call looking successful.
// So the kernel ends only when every peer's part has arrived (or is known to be missing). A system-scope fence costs
// microseconds on B200, more when many SMs issue one at once; GPU-scope fences, acquire loads and relaxed stores cost
// about the link latency. One uncontended system fence per call is the only one on the critical path.
//
// A rank that refuses a fused call on the host (a bad pointer on that rank only) launches p2p_abstain instead: it
// posts READY for every CTA index and a marked DONE, waits for the peers' DONE and advances EPOCH, so the ranks'
// numbering stays aligned and the next call is exact again.
//
// The epoch lives in device memory, so a call captured in a CUDA graph numbers itself on every replay; epochs only
// grow (from 1; the flags block starts zeroed), so the flags never need resetting. A rank whose grid differs from its
// peers' (shapes that differ between ranks) leaves READY pairs unmatched: the waits time out and raise the status bit.
#pragma once

#include "ptx.cuh"

namespace vkb {

constexpr int P2P_MAX_RANKS = 8;
constexpr int P2P_MAX_CTAS = 256;                                  // grids of the fused kernels (<= SM count)
constexpr int P2P_READY = 0;                                       // [P2P_MAX_RANKS][P2P_MAX_CTAS]
constexpr int P2P_DONE = P2P_MAX_RANKS * P2P_MAX_CTAS;             // [P2P_MAX_RANKS]
constexpr int P2P_COUNT = P2P_DONE + P2P_MAX_RANKS;
constexpr int P2P_EPOCH = P2P_COUNT + 1;
constexpr int P2P_FAILED = P2P_EPOCH + 1;
constexpr int P2P_FLAG_WORDS = P2P_FAILED + 1;
constexpr size_t P2P_FLAG_BYTES = (P2P_FLAG_WORDS * 4 + 255) / 256 * 256;   // the communicator's flags block
constexpr uint32_t P2P_EPOCH_MASK = 0x7fffffffu;   // epochs: 31 bits
constexpr uint32_t P2P_FAIL_MARK = 0x80000000u;    // DONE: this rank's part of the call is missing

struct P2PArgs {
    void* peer_base[P2P_MAX_RANKS];        // the symmetric buffer on every rank (peer_base[rank] = this rank's)
    uint32_t* peer_flags[P2P_MAX_RANKS];   // its flags block on every rank
    int rank, size;
};

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Whether 31-bit epoch v is at or past e (modulo 2^31: the counters wrap).
__device__ __forceinline__ bool epoch_reached(uint32_t v, uint32_t e) {
    return ((v - e) & P2P_EPOCH_MASK) < 0x40000000u;
}

// Wait until the epoch in flag reaches e. 0: reached; 1: reached, and the word for exactly e carries the failure
// mark; 2: the wait gave up (DEV_ERR_PEER_TIMEOUT raised). Bounded.
__device__ __forceinline__ int p2p_wait_epoch(const uint32_t* flag, uint32_t e) {
    uint32_t v = ld_acquire_sys(flag);
    if (!epoch_reached(v & P2P_EPOCH_MASK, e)) {
        const uint64_t t0 = globaltimer();
        for (uint32_t i = 0;; ++i) {
            v = ld_acquire_sys(flag);
            if (epoch_reached(v & P2P_EPOCH_MASK, e)) break;
            if ((i & 63u) == 63u) {
                if (globaltimer() - t0 > VKB_WAIT_NS) {
                    raise_status(DEV_ERR_PEER_TIMEOUT);
                    return 2;
                }
                __nanosleep(64);
            }
        }
    }
    return ((v & P2P_EPOCH_MASK) == e && (v & P2P_FAIL_MARK)) ? 1 : 0;
}
__device__ __forceinline__ bool p2p_wait_flag(const uint32_t* flag, uint32_t e) { return p2p_wait_epoch(flag, e) == 0; }

// The number of the call now running (only after griddepcontrol.wait, or in a thread ordered after one that did).
__device__ __forceinline__ uint32_t p2p_epoch(const P2PArgs& p) {
    const uint32_t last = *reinterpret_cast<volatile const uint32_t*>(p.peer_flags[p.rank] + P2P_EPOCH);
    const uint32_t e = (last + 1u) & P2P_EPOCH_MASK;
    return e == 0 ? 1u : e;
}

// Step 1 (one thread per CTA, after griddepcontrol.wait).
__device__ __forceinline__ void p2p_post_ready(const P2PArgs& p, uint32_t e) {
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank) st_relaxed_sys(p.peer_flags[r] + P2P_READY + p.rank * P2P_MAX_CTAS + blockIdx.x, e);
}

// Step 2 (lane 0 of a warp, then a warp broadcast): every peer's CTA of this index accepts writes of call e.
__device__ __forceinline__ bool p2p_wait_ready(const P2PArgs& p, uint32_t e) {
    const uint32_t* f = p.peer_flags[p.rank] + P2P_READY + blockIdx.x;
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank && !p2p_wait_flag(f + r * P2P_MAX_CTAS, e)) return false;
    return true;
}

// Push finished rows of this rank's copy to the same place in every peer's copy: `rows` rows of row_bytes bytes,
// row r at byte offset row_off(r). Thread t of nth cooperating threads takes every nth vector, loads it once (the
// rows were just written: L2) and stores it to each peer; four loads are in flight per thread. V is the widest word
// that every row offset and row_bytes are multiples of (16 bytes: a warp's store then covers 512 contiguous bytes,
// few and large NVLink writes instead of the scattered 2-byte stores of an epilogue). The rows must be complete and
// visible to the calling threads (a barrier after their stores).
template <typename V, typename RowOff>
__device__ __forceinline__ void p2p_push_rows(const P2PArgs& p, int rows, int row_bytes, RowOff row_off, int t,
                                              int nth) {
    const int vpr = row_bytes / (int)sizeof(V);
    if (rows <= 0 || vpr <= 0) return;
    const int total = rows * vpr;
    const uint8_t* src = static_cast<const uint8_t*>(p.peer_base[p.rank]);
    constexpr int U = 4;
    for (int v0 = t; v0 < total; v0 += U * nth) {
        V val[U];
        size_t o[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int v = v0 + u * nth;
            if (v < total) {
                const int r = v / vpr, c = v - r * vpr;
                o[u] = row_off(r) + (size_t)c * sizeof(V);
                val[u] = *reinterpret_cast<const V*>(src + o[u]);
            }
        }
        for (int k = 0; k < p.size; ++k) {
            if (k == p.rank) continue;
            uint8_t* dst = static_cast<uint8_t*>(p.peer_base[k]);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (v0 + u * nth < total) *reinterpret_cast<V*>(dst + o[u]) = val[u];
        }
    }
}

// The widest copy word for byte offsets / lengths whose OR is m.
template <typename RowOff>
__device__ __forceinline__ void p2p_push(const P2PArgs& p, int rows, int row_bytes, size_t m, RowOff row_off, int t,
                                         int nth) {
    m |= (size_t)row_bytes;
    if ((m & 15) == 0) p2p_push_rows<uint4>(p, rows, row_bytes, row_off, t, nth);
    else if ((m & 3) == 0) p2p_push_rows<uint32_t>(p, rows, row_bytes, row_off, t, nth);
    else p2p_push_rows<uint16_t>(p, rows, row_bytes, row_off, t, nth);
}

// Step 3 (one thread per CTA, after a barrier that follows every store of the CTA). ok: every thread of the CTA did
// its part of the call (no wait gave up, every push was made).
__device__ __forceinline__ void p2p_finish(const P2PArgs& p, bool ok) {
    uint32_t* f = p.peer_flags[p.rank];
    const uint32_t e = p2p_epoch(p);   // read before the count: the last CTA stores the new value after every count
    if (!ok) atomicOr(f + P2P_FAILED, 1u);
    asm volatile("fence.acq_rel.gpu;" ::: "memory");   // this CTA's stores (and its epoch read) before its count
    const uint32_t old = atomicAdd(f + P2P_COUNT, 1u);
    if (old != gridDim.x - 1) return;
    f[P2P_COUNT] = 0;        // every CTA of this call has counted; the next call starts from zero
    fence_acq_rel_sys();     // acquire every CTA's stores, release them (and this CTA's) to the peers
    const bool failed = atomicExch(f + P2P_FAILED, 0u) != 0;
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank) st_relaxed_sys(p.peer_flags[r] + P2P_DONE + p.rank, e | (failed ? P2P_FAIL_MARK : 0u));
    for (int r = 0; r < p.size; ++r) {
        if (r == p.rank) continue;
        const int w = p2p_wait_epoch(f + P2P_DONE + r, e);
        if (w == 1) raise_status(DEV_ERR_PEER_FAILED);
        if (w == 2) break;
    }
    // call e is complete here (also after a timeout, so that a late peer can still catch up on the numbering)
    *reinterpret_cast<volatile uint32_t*>(f + P2P_EPOCH) = e;
}

// The whole call on a rank that refused it on the host (one CTA): READY for every CTA index of every peer, a marked
// DONE, the peers' DONE awaited, EPOCH advanced. Peers' pushes into this rank's copy are harmless (its call failed).
// Raises no status bit for the peers' marks: the refusing rank already returned an error code.
__device__ __forceinline__ void p2p_abstain(const P2PArgs& p) {
    const uint32_t e = p2p_epoch(p);
    for (int b = threadIdx.x; b < P2P_MAX_CTAS; b += blockDim.x)
        for (int r = 0; r < p.size; ++r)
            if (r != p.rank) st_relaxed_sys(p.peer_flags[r] + P2P_READY + p.rank * P2P_MAX_CTAS + b, e);
    __syncthreads();
    if (threadIdx.x != 0) return;
    uint32_t* f = p.peer_flags[p.rank];
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank) st_relaxed_sys(p.peer_flags[r] + P2P_DONE + p.rank, e | P2P_FAIL_MARK);
    for (int r = 0; r < p.size; ++r)
        if (r != p.rank && p2p_wait_epoch(f + P2P_DONE + r, e) == 2) break;
    *reinterpret_cast<volatile uint32_t*>(f + P2P_EPOCH) = e;
}

}  // namespace vkb
