// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA (cp.async.bulk / cp.async.bulk.tensor), programmatic
// dependent launch, the m16n8k16 tensor-core MMA, and the bounded waits every kernel in this library uses.
//
// Every spin in this library goes through wait_parity(): it gives up after VKB_WAIT_NS of %globaltimer time, records
// the failure in the device-wide status word (vkb_dev_status) and returns false, so a lost copy or a logic error shows
// up as an error code on the host instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#ifndef VKB_WAIT_NS
#define VKB_WAIT_NS 2000000000ull  // 2 s: far above any legitimate wait (a whole previous kernel under PDL)
#endif

namespace vkb {

// Status bits a kernel can raise (read and cleared by vkb_device_status()).
enum : unsigned {
    DEV_ERR_WAIT_TIMEOUT = 1u,    // a pipeline wait (mbarrier) gave up
    DEV_ERR_DRAIN_TIMEOUT = 2u,   // waiting for this CTA's own copies in flight gave up
    DEV_ERR_PEER_TIMEOUT = 4u,    // a wait on a peer rank's flag gave up
    DEV_ERR_PEER_FAILED = 8u,     // a peer rank reported its part of a fused call missing
};

}  // namespace vkb

// One status word per translation unit (device variables are not shared across TUs without relocatable device
// code); each TU that launches kernels exposes a host accessor through VKB_STATUS_ACCESSOR and vkb_device_status()
// reads them all.
static __device__ unsigned int vkb_dev_status;

#define VKB_STATUS_ACCESSOR(fn)                                                        \
    int fn(unsigned* bits) {                                                           \
        unsigned v = 0, zero = 0;                                                      \
        cudaError_t e = cudaMemcpyFromSymbol(&v, vkb_dev_status, sizeof(v));            \
        if (e == cudaSuccess) e = cudaMemcpyToSymbol(vkb_dev_status, &zero, sizeof(v)); \
        *bits |= v;                                                                    \
        return e == cudaSuccess ? 0 : -(int)e;                                         \
    }

namespace vkb {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&vkb_dev_status, bits); }

// ---- mbarrier -------------------------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete. Bounded: false (and a status bit) after VKB_WAIT_NS.
__device__ __forceinline__ bool wait_parity(uint64_t* bar, uint32_t parity, unsigned err = DEV_ERR_WAIT_TIMEOUT) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 255u) == 255u && globaltimer() - t0 > VKB_WAIT_NS) {
            raise_status(err);
            return false;
        }
    }
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps until it completes (or the hint,
// ns, elapses) instead of re-issuing the test, so a waiting role leaves its sub-partition's issue slots to others.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase (returns at once): the fast path of the sleeping waits below.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait_cl(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// wait_parity for roles that are not on the critical issue path (producers, the MMA thread, waiting consumers). A
// completed phase is tested first (test_wait returns at once; a try_wait with a suspend hint costs ~150 cycles even
// then), and only an incomplete one sleeps.
__device__ __forceinline__ bool wait_parity_sleep(uint64_t* bar, uint32_t parity,
                                                  unsigned err = DEV_ERR_WAIT_TIMEOUT) {
    const uint32_t a = smem_u32(bar);
    if (mbar_test_wait(a, parity) || mbar_try_wait_sleep(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait_sleep(a, parity)) return true;
        if (globaltimer() - t0 > VKB_WAIT_NS) {
            raise_status(err);
            return false;
        }
    }
}

// ---- clusters (pairs of CTAs) ----------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Shared::cluster address of the variable at this CTA's shared address a, in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
// Arrive on an mbarrier of any CTA of the cluster (address from mapa_shared), releasing at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Every thread of every CTA of the cluster (all threads execute it).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// wait_parity_sleep for barriers that other CTAs of the cluster arrive on (acquire at cluster scope).
__device__ __forceinline__ bool mbar_try_wait_sleep_cl(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool wait_parity_sleep_cl(uint64_t* bar, uint32_t parity,
                                                     unsigned err = DEV_ERR_WAIT_TIMEOUT) {
    const uint32_t a = smem_u32(bar);
    if (mbar_test_wait_cl(a, parity) || mbar_try_wait_sleep_cl(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait_sleep_cl(a, parity)) return true;
        if (globaltimer() - t0 > VKB_WAIT_NS) {
            raise_status(err);
            return false;
        }
    }
}

// ---- TMA ------------------------------------------------------------------------------------------------------

// 2-D tiled tensor load (no multicast) into this CTA's shared memory, completing bytes on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 3-D tiled tensor load of a CTA pair (cta_group::2, no multicast): the box lands in this CTA's shared memory and its
// bytes complete on the mbarrier at bar_cluster (a shared::cluster address, e.g. the pair leader's barrier).
__device__ __forceinline__ void tma_load_3d_cg2(void* dst, const CUtensorMap* map, int x, int y, int z,
                                                uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 1-D bulk copy global -> shared (both addresses 16-byte aligned, bytes a multiple of 16), completing on bar.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetches (no data returned, so they may run ahead of a dependency: L2 is the point of coherence, and a line
// written afterwards is updated there). Bulk: src and bytes multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}

// 3-D tiled tensor load (no multicast) into this CTA's shared memory, completing bytes on bar.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 2-D tiled tensor store shared -> global (bulk-group completion); elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups of this thread still read their shared-memory source.
template <int N> __device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups of this thread are still in flight (writes performed).
template <int N> __device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// One lane of a converged warp (elect.sync): the issuing lane for warp-uniform producer / MMA loops.
__device__ __forceinline__ bool elect_one() {
    uint32_t e;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(e));
    return e != 0;
}

// ---- programmatic dependent launch ------------------------------------------------------------------------------

// Block until every grid this one depends on has completed and its memory is visible (no-op without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Let the next grid in the stream start its prologue (it still waits in pdl_wait() for this grid to finish).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- named barriers (a subset of the CTA's warps) ----------------------------------------------------------------

__device__ __forceinline__ void named_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Arrive on named barrier `id` without waiting (the threads that wait on it see this thread's earlier writes).
__device__ __forceinline__ void named_arrive(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- m16n8k16 f16 x f16 -> f32 ----------------------------------------------------------------------------------

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- small bit helpers ------------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// (a & b) | c in one LOP3
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

}  // namespace vkb

namespace vkb {

// ---- explicit shared-memory loads on 32-bit shared addresses ------------------------------------------------------

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ float half_lo_f32(uint32_t h2) {
    float f;
    asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, lo; }" : "=f"(f) : "r"(h2));
    return f;
}
__device__ __forceinline__ float half_hi_f32(uint32_t h2) {
    float f;
    asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, hi; }" : "=f"(f) : "r"(h2));
    return f;
}

}  // namespace vkb
