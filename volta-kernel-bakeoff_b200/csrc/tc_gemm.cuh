// Prompt GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), Q4 weights, sm_100a.
//
//   y[m][n] = sum_k x[m][k] * w[n][k],  w = (code - 8) * scale rounded to fp16 (the reference's tc_q4 unpack,
//   src/stage4_tc.cuh:25-36: exact code, one fp16 multiply by the group scale), fp32 accumulation, fp16/fp32 out.
//
// One CTA computes a 128-row (weights) x NT-column (tokens) tile of y^T in TMEM. Three rings, each with its own
// depth, so that the slow stream (packed weights from HBM) runs far ahead of the fast one (activations from L2):
//   P ring  (shared memory) packed codes, 128 rows x PK K steps (PK = 8: 512 codes) per chunk, padded rows
//   X ring  (shared memory) activations, XK K steps of NT tokens x 64 k per stage (one 3-D TMA box), 128B-swizzled:
//           exactly the K-major UMMA B operand
// Stages are large on purpose: a TMA producer thread completes stages at a roughly fixed rate (~0.65-0.75k cycles
// per stage from L2 up to ~32 KB), so bytes per stage, not boxes per stage, set the streaming rate.
//   A ring  (tensor memory) dequantised fp16 weights, slots of 4 K steps (128 lanes x 128 columns): the UMMA A
//           operand read straight from TMEM (tcgen05.mma with [a-tmem], faster than A from shared memory), so
//           dequantised weights never touch shared memory; one afull/aempty handshake per slot (16 UMMAs) keeps the
//           MMA warp's per-instruction overhead (barrier waits, commits) off the tensor pipe's critical path
// Warp roles:
//   warp 0      TMA producer of the P ring (and the tile's scales, once), started before griddepcontrol.wait: the
//               weights never depend on the previous kernel in the stream
//   warp 1      allocates TMEM; one thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=NT, K=16) x4 per K
//               step and commits each step back to the X and A rings
//   warps 2, 11 TMA producers of the X ring (after griddepcontrol.wait), even and odd stages: one producer thread
//               completes stages at a fixed rate, two double it
//   warps 3-10  two groups of four warps dequantise half a slot each (K steps 0-1 / 2-3): one weight row per
//               thread (the warp's TMEM lane quarter), 64 codes -> 32 fp16 pairs -> tcgen05.st.32x32b.x32; then the
//               epilogue: tcgen05.ld of the accumulators, staged in shared memory per warp and written by TMA
//               stores (plain masked stores when y's rows are not 16-byte multiples)
// Waiting roles sleep in mbarrier.try_wait (suspend hint) so that they leave issue slots to the dequantising warps.
// No cluster multicast anywhere: the kernel also serves the row-split multi-GPU calls.
#pragma once

#include "ptx.cuh"

namespace vkb {

constexpr int TC_BM = 128;            // weight rows per CTA (UMMA M)
constexpr int TC_BK = 64;             // k per K step: one 128-byte swizzle row of fp16
// A packed chunk holds PK K steps (4 or 8: 32 * PK code bytes per row); its row pitch adds 16 bytes so that pitch / 16
// is odd and the dequantising warps' 16-byte reads are conflict free.
__host__ __device__ constexpr int tc_ppitch(int pk) { return 32 * pk + 16; }
__host__ __device__ constexpr int tc_pchunk(int pk) { return TC_BM * tc_ppitch(pk); }
constexpr int TC_ACOLS = 32;          // TMEM columns of one dequantised K step (128 lanes x 64 fp16)
constexpr int TC_SLOT = 4;            // K steps per A slot: one barrier handshake per 16 UMMAs
constexpr int TC_NDQ = 8;             // dequantising / epilogue warps (two groups of four)
constexpr int TC_XPROD2 = 3 + TC_NDQ;  // the second X producer warp (the first is warp 2)
constexpr int TC_THREADS = 32 * (4 + TC_NDQ);
constexpr int TC_EPI_BOX = 32;        // epilogue TMA store box: 32 weight rows x 32 tokens

struct TcArgs {
    void* y;            // [M][N]
    int M, N, K;
    int NT;             // tokens per CTA tile (multiple of 32, <= 256)
    int nk;             // K steps (K / 64)
    int na, nx, np;     // ring depths: A slots (TMEM), X stages, P chunks
    int a_col0;         // first TMEM column of the A ring (the accumulators occupy columns [0, NT))
    int x_off, p_off, s_off, bar_off;   // shared-memory region offsets (1024-aligned rings)
    int xk;             // K steps per X stage (one 3-D TMA box of xk 128B-swizzled NT x 64 tiles)
    int x_stage;        // bytes of one X stage (xk x NT x 128)
    int spitch;         // scale bytes per row
    int tmem_cols;
    int tma_store;      // 1: epilogue through shared memory + TMA stores (needs 16-byte y rows)
};

// ---- tcgen05 wrappers ----------------------------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// K-major, 128B-swizzled shared-memory matrix descriptor: 8-row atoms of 1024 bytes (SBO), version 1, layout 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                    // leading byte offset (unused for swizzled K-major): 16 B
    d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: next 8-row atom
    d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: f16 A and B, f32 D, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
    const uint32_t z = 0;   // disable-output-lane mask: every lane written
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accum), "r"(z)
        : "memory");
}

// A from tensor memory: tmem_a addresses 128 lanes x 8 columns (K = 16 fp16, two per 32-bit column, even k low).
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t accum) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum), "r"(z)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t gets lane (taddr.lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread t writes lane (taddr.lane + t); waits until done.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// The same without the wait: the registers are valid only after tmem_wait_ld(r) on the same array.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// tcgen05.wait::ld, with r as read-write operands so that no use of r moves above the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// One packed word (8 codes of one row, natural k order) -> 8 fp16 weights (code - 8) * scale in four consecutive
// registers of a row's 32-register K step (low half = even k).
__device__ __forceinline__ void dequant8_to(uint32_t v, uint32_t s2, uint32_t* r) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t b = prmt(v, 0u, 0x4040u | (j << 8) | j);                   // bytes [b_j, 0, b_j, 0]
        const uint32_t h = and_or(b, 0x00F0000Fu, 0x64006400u);                   // (1024 + lo, 1024 + 16 hi)
        const uint32_t c = h2_fma(h, 0x2C003C00u, 0xD480E408u);                    // exact (lo - 8, hi - 8)
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[j]) : "r"(c), "r"(s2));           // one rounding: code * scale
    }
}

template <typename OutT> __device__ __forceinline__ OutT tc_out(float v);
template <> __device__ __forceinline__ __half tc_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float tc_out<float>(float v) { return v; }

template <typename OutT, int PK>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_q4_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap ts,
             const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap ty, const TcArgs a) {
    constexpr int PPITCH = tc_ppitch(PK), PCHUNK = tc_pchunk(PK);
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* sm = smem_raw + pad;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + a.bar_off);
    uint64_t* pfull = bars;                   // [np] packed chunk landed
    uint64_t* pempty = pfull + a.np;          // [np] both dequant groups done with the chunk (8 warps)
    uint64_t* xfull = pempty + a.np;          // [nx] activation stage landed
    uint64_t* xempty = xfull + a.nx;          // [nx] MMAs of the stage done (tcgen05.commit)
    uint64_t* afull = xempty + a.nx;          // [na] dequantised slot written to TMEM (8 warps)
    uint64_t* aempty = afull + a.na;          // [na] MMAs of the slot done (tcgen05.commit)
    uint64_t* sfull = aempty + a.na;          // scales landed
    uint64_t* accum = sfull + 1;              // all MMAs done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * TC_BM, tok0 = blockIdx.y * a.NT;
    const int nk = a.nk, nch = nk / PK, nxs = nk / a.xk;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.np; ++i) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], TC_NDQ);
        }
        for (int i = 0; i < a.nx; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], 1);
        }
        for (int i = 0; i < a.na; ++i) {
            mbar_init(&afull[i], TC_NDQ);
            mbar_init(&aempty[i], 1);
        }
        mbar_init(sfull, 1);
        mbar_init(accum, 1);
        fence_mbar_init();
        // the weights do not depend on the previous grid: the scales and the first chunks start now, before the TMEM
        // allocation and the block-wide barrier (the thread that initialised the barriers issues them)
        prefetch_tmap(&tq);
        prefetch_tmap(&ts);
        mbar_arrive_expect_tx(sfull, (uint32_t)(TC_BM * a.spitch));
        tma_load_2d(sm + a.s_off, &ts, 0, row0, sfull);
        for (int c = 0; c < min(nch, a.np); ++c) {
            mbar_arrive_expect_tx(&pfull[c], (uint32_t)PCHUNK);
            tma_load_2d(sm + a.p_off + c * PCHUNK, &tq, c * PK * 4, row0, &pfull[c]);   // PK x 4 x 8 B of codes
        }
    }
    if (warp == 1) tmem_alloc(tmem_slot, (uint32_t)a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    // Producer and MMA roles run warp-uniform loops (every lane waits, one elected lane issues), the form the
    // tcgen05 / TMA issue path expects; `ok` stays warp-uniform.
    if (warp == 0) {
        // ===================== P ring producer (weights: no dependence on the previous grid) =====================
        // chunks 0 .. np-1 and the scales were issued at barrier set-up; refill the ring from chunk np on
        int b = 0, rnd = 1;
        for (int c = a.np; c < nch; ++c) {
            ok = __all_sync(0xffffffffu, wait_parity_sleep(&pempty[b], (rnd - 1) & 1));
            if (!ok) break;
            if (elect_one()) {
                mbar_arrive_expect_tx(&pfull[b], (uint32_t)PCHUNK);
                tma_load_2d(sm + a.p_off + b * PCHUNK, &tq, c * PK * 4, row0, &pfull[b]);   // PK x 4 x 8 B of codes
            }
            __syncwarp();
            if (++b == a.np) { b = 0; ++rnd; }
        }
        // drain: the last loads (and the scales) land before exit
        const int d = ok ? max(0, nch - a.np) : nch;
        for (int c = d; c < nch; ++c)
            if (!wait_parity_sleep(&pfull[c % a.np], (c / a.np) & 1, DEV_ERR_DRAIN_TIMEOUT)) break;
        wait_parity_sleep(sfull, 0, DEV_ERR_DRAIN_TIMEOUT);
    } else if (warp == 2 || warp == TC_XPROD2) {
        // ===================== X ring producers (activations: after the previous grid) =====================
        // warp 2 loads the even stages, warp TC_XPROD2 the odd ones (nx is even: each owns fixed ring slots)
        const int par = warp == 2 ? 0 : 1;
        if (elect_one()) prefetch_tmap(&tx);
        pdl_wait();
        int last = -1;
        for (int xs = par; xs < nxs; xs += 2) {
            const int b = xs % a.nx, rnd = xs / a.nx;
            if (rnd > 0) ok = __all_sync(0xffffffffu, wait_parity_sleep(&xempty[b], (rnd - 1) & 1));
            if (!ok) break;
            if (elect_one()) {
                mbar_arrive_expect_tx(&xfull[b], (uint32_t)a.x_stage);
                tma_load_3d(sm + a.x_off + b * a.x_stage, &tx, 0, tok0, xs * a.xk, &xfull[b]);
            }
            __syncwarp();
            last = xs;
        }
        // drain: this warp's loads that may still be in flight land before exit
        for (int xs = last; xs >= 0 && xs > last - a.nx; xs -= 2)
            if (!wait_parity_sleep(&xfull[xs % a.nx], (xs / a.nx) & 1, DEV_ERR_DRAIN_TIMEOUT)) break;
    } else if (warp == 1) {
        // ===================== MMA issuer =====================
        // per slot: wait for its A (TMEM) and the X stages its 4 K steps read, then 16 UMMAs (4 per K step), one A
        // handshake per slot. When the X ring holds at least two slots of K steps, all of a slot's X waits come first
        // and the 16 UMMAs issue back to back; otherwise (large token tiles, shallow X ring) the waits interleave
        // with the K steps, so that each X stage is released as soon as its own MMAs complete.
        const uint32_t idesc = umma_idesc_f16(a.NT);
        const uint32_t xtile = (uint32_t)a.NT * 128;
        const int nslots = nk / TC_SLOT;
        const bool hoist = a.nx * a.xk >= 2 * TC_SLOT;
        int ab = 0, arnd = 0, xb = 0, xrnd = 0, xj = 0;
        for (int sl = 0; sl < nslots && ok; ++sl) {
            ok = __all_sync(0xffffffffu, wait_parity_sleep(&afull[ab], arnd & 1));
            if (!ok) break;
            tc_fence_after();
            const uint32_t ta = tmem + (uint32_t)(a.a_col0 + ab * TC_SLOT * TC_ACOLS);
            if (hoist) {
                uint32_t sb[TC_SLOT];
                int rel[TC_SLOT];   // X stage to release after K step j (-1: none)
#pragma unroll
                for (int j = 0; j < TC_SLOT; ++j) {
                    if (xj == 0 && ok) ok = __all_sync(0xffffffffu, wait_parity_sleep(&xfull[xb], xrnd & 1));
                    sb[j] = smem_u32(sm + a.x_off + xb * a.x_stage) + xj * xtile;
                    rel[j] = xj + 1 == a.xk ? xb : -1;
                    if (++xj == a.xk) {
                        xj = 0;
                        if (++xb == a.nx) { xb = 0; ++xrnd; }
                    }
                }
                if (!ok) break;
                if (elect_one()) {
#pragma unroll
                    for (int j = 0; j < TC_SLOT; ++j) {
                        const int it = sl * TC_SLOT + j;
#pragma unroll
                        for (int kk = 0; kk < TC_BK / 16; ++kk)   // 16 k: 8 TMEM columns of A, 32 bytes of the B row
                            umma_f16_ts(tmem, ta + (uint32_t)(j * TC_ACOLS + 8 * kk), umma_desc_sw128(sb[j] + 32 * kk),
                                        idesc, (it | kk) != 0);
                        if (rel[j] >= 0) umma_commit(&xempty[rel[j]]);   // free the stage once these MMAs complete
                    }
                    umma_commit(&aempty[ab]);
                }
                __syncwarp();
            } else {
#pragma unroll
                for (int j = 0; j < TC_SLOT; ++j) {
                    if (xj == 0) {
                        ok = __all_sync(0xffffffffu, wait_parity_sleep(&xfull[xb], xrnd & 1));
                        if (!ok) break;
                    }
                    const int it = sl * TC_SLOT + j;
                    const uint32_t sb = smem_u32(sm + a.x_off + xb * a.x_stage) + xj * xtile;
                    const bool last_x = xj + 1 == a.xk;
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < TC_BK / 16; ++kk)
                            umma_f16_ts(tmem, ta + (uint32_t)(j * TC_ACOLS + 8 * kk), umma_desc_sw128(sb + 32 * kk),
                                        idesc, (it | kk) != 0);
                        if (last_x) umma_commit(&xempty[xb]);
                        if (j == TC_SLOT - 1) umma_commit(&aempty[ab]);
                    }
                    __syncwarp();
                    if (last_x) {
                        xj = 0;
                        if (++xb == a.nx) { xb = 0; ++xrnd; }
                    } else {
                        ++xj;
                    }
                }
                if (!ok) break;
            }
            if (++ab == a.na) { ab = 0; ++arnd; }
        }
        if (elect_one()) umma_commit(accum);   // arrives when every MMA issued above has completed
        __syncwarp();
    } else {
        // ===================== dequantise (two groups, half a slot each), then epilogue =====================
        const int dw = warp - 3;                  // 0..7
        const int grp = dw >> 2;                  // K steps 2 grp, 2 grp + 1 of every slot
        const int qtr = warp & 3;                 // TMEM lane quarter this warp may access
        const int r = qtr * 32 + lane;            // weight row of the tile = TMEM lane
        if (!wait_parity_sleep(sfull, 0)) ok = false;
        const uint32_t srow = smem_u32(sm + a.s_off + r * a.spitch);
        const uint32_t prow = smem_u32(sm + a.p_off) + r * PPITCH;
        const uint32_t tlane = tmem + ((uint32_t)(32 * qtr) << 16) + (uint32_t)(a.a_col0 + 2 * grp * TC_ACOLS);
        for (int c = 0; c < nch && ok; ++c) {
            const int pb = c % a.np;
            if (!wait_parity_sleep(&pfull[pb], (c / a.np) & 1)) { ok = false; break; }
            uint32_t sw[PK];                                          // scales of the chunk's 2 x PK groups
#pragma unroll
            for (int q4 = 0; q4 < PK / 4; ++q4) {
                const uint4 t = lds128(srow + (c * PK + 4 * q4) * 4);
                sw[4 * q4] = t.x; sw[4 * q4 + 1] = t.y; sw[4 * q4 + 2] = t.z; sw[4 * q4 + 3] = t.w;
            }
#pragma unroll
            for (int sc = 0; sc < PK / TC_SLOT; ++sc) {            // slots of this chunk
                const int sl = c * (PK / TC_SLOT) + sc;
                const int ab = sl % a.na;
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {                    // this group's two K steps of the slot
                    const int sub0 = sc * TC_SLOT + jj;             // sub-step within the chunk for grp 0
                    const uint32_t pa = prow + pb * PCHUNK + (sub0 + 2 * grp) * 32;
                    const uint4 w0 = lds128(pa), w1 = lds128(pa + 16);
                    const uint32_t sv = grp ? sw[sub0 + 2] : sw[sub0];  // groups of this K step (static indices)
                    const uint32_t s_lo = (sv & 0xFFFFu) * 0x00010001u, s_hi = (sv >> 16) * 0x00010001u;
                    uint32_t v[32];
                    dequant8_to(w0.x, s_lo, v + 0);
                    dequant8_to(w0.y, s_lo, v + 4);
                    dequant8_to(w0.z, s_lo, v + 8);
                    dequant8_to(w0.w, s_lo, v + 12);
                    dequant8_to(w1.x, s_hi, v + 16);
                    dequant8_to(w1.y, s_hi, v + 20);
                    dequant8_to(w1.z, s_hi, v + 24);
                    dequant8_to(w1.w, s_hi, v + 28);
                    if (sc == PK / TC_SLOT - 1 && jj == 1) {        // this warp's last read of the chunk
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&pempty[pb]);
                    }
                    if (jj == 0) {                                  // the slot's previous MMAs are done
                        if (sl >= a.na && !wait_parity_sleep(&aempty[ab], ((sl / a.na) - 1) & 1)) { ok = false; break; }
                        tc_fence_after();
                    }
                    tmem_st32(tlane + (uint32_t)(ab * TC_SLOT * TC_ACOLS + jj * TC_ACOLS), v);
                }
                if (!ok) break;
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[ab]);
            }
        }
    }
    // ===================== epilogue: all twelve warps =====================
    // warp w reads TMEM lanes 32 (w % 4).. (weight rows); the three warps of a lane quarter (w % 4 equal) take every
    // third 32-token chunk. Producers and the MMA warp join once their own loads have landed / MMAs are issued.
    pdl_wait();   // y may still be read or written by the previous grid
    if (ok && wait_parity_sleep(accum, 0)) {
        tc_fence_after();
        const int q = warp & 3, third = warp >> 2;
        constexpr int STEP = 3 * 32;
        const uint32_t tq_addr = tmem + ((uint32_t)(32 * q) << 16);
        if (a.tma_store) {
            // per-warp staging (2 buffers of 32 tokens x 32 rows) in the idle X/P rings: every load has landed and
            // been consumed before the last MMA completed
            OutT* stg = reinterpret_cast<OutT*>(sm) + (size_t)warp * 2 * TC_EPI_BOX * TC_EPI_BOX;
            auto put = [&](uint32_t (&v)[32], int c, int nb) {
                OutT* sb = stg + nb * TC_EPI_BOX * TC_EPI_BOX;
                if (lane == 0) bulk_wait_group_read<1>();   // the store that last used this buffer has read it
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 32; ++j) sb[j * TC_EPI_BOX + lane] = tc_out<OutT>(__uint_as_float(v[j]));
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&ty, row0 + 32 * q, tok0 + c, sb);   // clipped at N and M by the tensor map
                    bulk_commit_group();
                }
            };
            // two TMEM loads in flight: the next chunk loads while this one is converted and stored
            uint32_t va[32], vb[32];
            int c = 32 * third;
            if (c < a.NT) tmem_ld32_async(tq_addr + (uint32_t)c, va);
            for (; c < a.NT; c += 2 * STEP) {
                tmem_wait_ld(va);
                if (c + STEP < a.NT) tmem_ld32_async(tq_addr + (uint32_t)(c + STEP), vb);
                put(va, c, 0);
                if (c + STEP >= a.NT) break;
                tmem_wait_ld(vb);
                if (c + 2 * STEP < a.NT) tmem_ld32_async(tq_addr + (uint32_t)(c + 2 * STEP), va);
                put(vb, c + STEP, 1);
            }
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
        } else {
            const int n = row0 + 32 * q + lane;
            OutT* y = reinterpret_cast<OutT*>(a.y);
            for (int c = 32 * third; c < a.NT; c += STEP) {
                uint32_t v[32];
                tmem_ld32(tq_addr + (uint32_t)c, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int m = tok0 + c + j;
                    if (m < a.M && n < a.N) y[(size_t)m * a.N + n] = tc_out<OutT>(__uint_as_float(v[j]));
                }
            }
        }
    }
    // teardown: every MMA has completed (accum) before TMEM is released
    if (warp == 1 && !ok) wait_parity_sleep(accum, 0, DEV_ERR_DRAIN_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
    }
}

}  // namespace vkb
