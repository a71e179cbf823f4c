// Prompt GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), Q4 weights, sm_100a.
//
//   y[m][n] = sum_k x[m][k] * w[n][k],  w = (code - 8) * scale rounded to fp16 (the reference's tc_q4 unpack,
//   src/stage4_tc.cuh:25-36: exact code, one fp16 multiply by the group scale), fp32 accumulation, fp16/fp32 out.
//
// Persistent: one CTA per SM walks the output tiles t = blockIdx.x, + gridDim.x, ... (tile = 128 weight rows x NT
// tokens of y^T, accumulated in TMEM), so the next tile's loads and dequantisation overlap this tile's last MMAs and
// its epilogue. Three rings, each with its own depth, so that the slow stream (packed weights from HBM) runs far
// ahead of the fast one (activations from L2):
//   P ring  (shared memory) chunks of PK K steps (PK = 8: 512 codes per row): the packed codes, rows padded to an
//           odd number of 16-byte units, and the 2 PK fp16 scales of each row (48-byte rows), two TMA boxes per chunk
//   X ring  (shared memory) activations, XK K steps of NT tokens x 64 k per stage (one 3-D TMA box), 128B-swizzled:
//           exactly the K-major UMMA B operand
//   A ring  (tensor memory) dequantised fp16 weights, slots of 4 K steps (128 lanes x 128 columns): the UMMA A
//           operand read straight from TMEM (tcgen05.mma with [a-tmem], faster than A from shared memory); one
//           afull/aempty handshake per slot (16 UMMAs) keeps the MMA warp's per-handshake cost off the tensor pipe
// and one or two TMEM accumulators (two when NT <= 128: the epilogue of one tile overlaps the MMAs of the next).
// Warp roles (16 warps):
//   warp 0      P producer (the first chunks are issued by thread 0 right after the barriers exist); weights never
//               depend on the previous kernel in the stream, so none of this waits for griddepcontrol.wait
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=NT, K=16)
//   warps 2, 3  X producers (after griddepcontrol.wait), even and odd stages: one producer completes stages at a
//               fixed rate, two double it
//   warps 4-11  dequantise: two groups of four, half a slot each (K steps 0-1 / 2-3); one weight row per thread (the
//               warp's TMEM lane quarter), 128 codes -> 64 fp16 pairs -> one tcgen05.st.32x32b.x64
//   warps 12-15 epilogue: tcgen05.ld of a finished accumulator, coalesced direct stores of y, then the accumulator is
//               released; the dequantising warps join them for the CTA's last tile
// Producer / MMA / epilogue roles run warp-uniform loops (every lane waits, one elected lane issues). Waiting roles
// sleep in mbarrier.try_wait (suspend hint) so that they leave issue slots to the dequantising warps.
// Stages are large on purpose: a TMA producer thread completes stages at a roughly fixed rate (~0.65-0.75k cycles
// per stage from L2 up to ~32 KB), so bytes per stage, not boxes per stage, set the streaming rate.
// No cluster multicast anywhere: the kernel also serves the row-split multi-GPU calls.
#pragma once

#include "p2p.cuh"
#include "ptx.cuh"

namespace vkb {

constexpr int TC_BM = 128;            // weight rows per tile (UMMA M)
constexpr int TC_BK = 64;             // k per K step: one 128-byte swizzle row of fp16
constexpr int TC_ACOLS = 32;          // TMEM columns of one dequantised K step (128 lanes x 64 fp16)
constexpr int TC_SLOT = 4;            // K steps per A slot
constexpr int TC_SPITCH = 48;         // scale bytes per row in a chunk (up to 16 scales; 48 / 16 odd: conflict free)
constexpr int TC_NDQ = 8;             // dequantising warps (two groups of four)
constexpr int TC_NEPI = 4;            // epilogue warps (one per TMEM lane quarter)
constexpr int TC_WDQ0 = 4;            // first dequantising warp
constexpr int TC_WEPI0 = TC_WDQ0 + TC_NDQ;
constexpr int TC_THREADS = 32 * (TC_WEPI0 + TC_NEPI);

// A packed chunk holds PK K steps (4 or 8): 128 rows of 32 PK code bytes at a pitch of 32 PK + 16 (pitch / 16 odd:
// the dequantising warps' 16-byte reads are conflict free), then 128 rows of scales at TC_SPITCH.
// Q8 weights (wf = 1) take 64 code bytes per K step instead of 32: pitch 64 PK + 16 (again an odd number of 16-byte
// units).
__host__ __device__ constexpr int tc_ppitch(int pk, int wf = 0) { return (wf == 1 ? 64 : 32) * pk + 16; }
__host__ __device__ constexpr int tc_pchunk(int pk, int wf = 0) { return TC_BM * (tc_ppitch(pk, wf) + TC_SPITCH); }

struct TcArgs {
    void* y;            // [M][ldy], this call's columns from ycol0
    int M, N, K;
    int NT;             // tokens per tile (multiple of 16, <= 256; of 32 for a CTA pair)
    int nk;             // K steps per tile (K / 64)
    int tiles_n;        // row tiles (N / 128 rounded up); tile t: rows (t % tiles_n) * 128, tokens (t / tiles_n) NT
    int tiles;          // all tiles
    int na, nx, np;     // ring depths: A slots (TMEM), X stages, P chunks
    int nacc;           // TMEM accumulators (2 when NT <= 128 with one row block, else 1)
    int a_col0;         // first TMEM column of the A ring; accumulator b at column b * 128, its row block r at
                        // + r round_up(NT, 32)
    int xk;             // K steps per X stage (one 3-D TMA box of xk 128B-swizzled NT x 64 tiles)
    int x_stage;        // bytes of one X stage (xk x NT x 128)
    int x_off, p_off, bar_off;   // shared-memory region offsets (1024-aligned)
    int tmem_cols;
    int ldy, ycol0;     // output row stride and first column (row split: the full y, this rank's columns)
    int p2p;            // 1: push every tile into every peer's copy of y (pp.peer_base), epoch protocol (P2P kernels)
    P2PArgs pp;
    int splits, kunit;  // split-K kernels: CTAs sharing a tile's K range (a cluster), K steps per unit of that range
};

// ---- tcgen05 wrappers ----------------------------------------------------------------------------------------------

// TMEM allocation of one CTA (CG = 1) or of a CTA pair (CG = 2: the same warp of both CTAs issues it, with the same
// shared-memory slot; each CTA gets the columns in its own TMEM at the same address).
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    if constexpr (CG == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    } else {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
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

// kind::f16 instruction descriptor: f16 A and B, f32 D, both K-major, M = m (128, or 256 for a CTA pair), N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n, int m = TC_BM) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
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

// The same issued by the leader of a CTA pair (cta_group::2, M = 256): A is 128 rows of each CTA's TMEM at tmem_a, B
// is N/2 rows of each CTA's shared memory at the descriptor's address, D is each CTA's 128 rows x N in its own TMEM.
__device__ __forceinline__ void umma_f16_ts_cg2(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                                uint32_t accum) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum), "r"(z)
        : "memory");
}

// Commit of a pair's MMAs: one arrive on the mbarrier at this shared offset in both CTAs of the pair.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(smem_u32(bar)), "h"((uint16_t)3)
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

// 32 lanes x 64 consecutive 32-bit columns from registers (two K steps of one row); waits until done.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,"
        "%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]),
          "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]),
          "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]),
          "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]),
          "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// One Q8 word (4 int8 codes of one row, natural k order) -> 4 fp16 weights code * scale in two registers: the exact
// code through the offset-binary magic number ((0x6400 | (code + 128)) - 1152), then one fp16 rounding of code * scale
// (the rounding the Q4 kernel applies, so the prompt GEMM stays in the reference's fp16 class).
__device__ __forceinline__ void dequant4_q8_to(uint32_t v, uint32_t s2, uint32_t* r) {
    const uint32_t u = v ^ 0x80808080u;
    const uint32_t c01 = h2_sub(prmt(u, 0x64646464u, 0x4140u), 0x64806480u);   // exact (c0, c1)
    const uint32_t c23 = h2_sub(prmt(u, 0x64646464u, 0x4342u), 0x64806480u);   // exact (c2, c3)
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[0]) : "r"(c01), "r"(s2));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[1]) : "r"(c23), "r"(s2));
}

template <typename OutT> __device__ __forceinline__ OutT tc_out(float v);
template <> __device__ __forceinline__ __half tc_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float tc_out<float>(float v) { return v; }

// One warp's share of a finished accumulator: the 32-token chunks sub, sub + parts, ... of its TMEM lane quarter
// (tq_addr: lane quarter and accumulator column; n: this lane's weight row), two TMEM loads in flight, stored straight
// to y. 32-column loads may run past the tile's tokens (up to the next multiple of 32): still inside the TMEM
// allocation, and not stored.
template <typename OutT>
__device__ __forceinline__ void tc_epi_store(const TcArgs& a, uint32_t tq_addr, int n, int tok0, int sub, int parts) {
    OutT* y = reinterpret_cast<OutT*>(a.y);
    const int step = 32 * parts;
    const int ntok = min(a.NT, a.M - tok0);   // tokens of this tile (NT is a multiple of 16, not of 32)
    auto put = [&](const uint32_t (&v)[32], int c) {
        if (n >= a.N) return;
        OutT* yp = y + (size_t)(tok0 + c) * a.ldy + a.ycol0 + n;
        const int lim = ntok - c;
#pragma unroll
        for (int j = 0; j < 32; ++j, yp += a.ldy)
            if (j < lim) *yp = tc_out<OutT>(__uint_as_float(v[j]));
    };
    uint32_t va[32], vb[32];
    int c = 32 * sub;
    if (c < ntok) tmem_ld32_async(tq_addr + (uint32_t)c, va);
    for (; c < ntok; c += 2 * step) {
        tmem_wait_ld(va);
        if (c + step < ntok) tmem_ld32_async(tq_addr + (uint32_t)(c + step), vb);
        put(va, c);
        if (c + step >= ntok) break;
        tmem_wait_ld(vb);
        if (c + 2 * step < ntok) tmem_ld32_async(tq_addr + (uint32_t)(c + 2 * step), va);
        put(vb, c + step);
    }
}

// Split-K: one warp's share of a finished partial accumulator into this CTA's shared memory as fp32 [token][128 rows]
// at `part` (shared address): the TMEM chunks of tc_epi_store; each store covers 32 consecutive rows of one token.
__device__ __forceinline__ void tc_epi_stash(const TcArgs& a, uint32_t tq_addr, int rloc, int tok0, int sub, int parts,
                                             uint32_t part) {
    const int ntok = min(a.NT, a.M - tok0);
    uint32_t v[32];
    for (int c = 32 * sub; c < ntok; c += 32 * parts) {
        tmem_ld32(tq_addr + (uint32_t)c, v);
        const int lim = ntok - c;
        const uint32_t p0 = part + (uint32_t)((c * TC_BM + rloc) * 4);
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < lim)
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(p0 + (uint32_t)(j * TC_BM * 4)), "r"(v[j]) : "memory");
    }
}

// Four fp32 values from the shared memory of a CTA of the cluster (address from mapa_shared).
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// Push the finished tile (weight rows row0.., tokens tok0..) from this rank's y to every peer; thread t of nth.
// Out of line, so that the epilogue's register allocation does not carry it.
template <typename OutT>
__device__ __noinline__ void tc_push_tile(const TcArgs& a, int row0, int tok0, int t, int nth) {
    const int rows = min(a.NT, a.M - tok0), cols = min(TC_BM, a.N - row0);
    const size_t off = ((size_t)tok0 * a.ldy + a.ycol0 + row0) * sizeof(OutT);
    const size_t pitch = (size_t)a.ldy * sizeof(OutT);
    p2p_push(a.pp, rows, cols * (int)sizeof(OutT), off | pitch, [&](int r) { return off + (size_t)r * pitch; }, t,
             nth);
}

// CG = 2: a cluster of two CTAs (a pair) shares each 256-row tile. Each CTA dequantises its own 128 weight rows into
// its own TMEM and loads half of the tile's tokens into its shared memory; the pair leader (cluster rank 0) issues
// tcgen05.mma.cta_group::2 (M = 256), which reads A from both TMEMs and B from both shared memories, so each SM
// streams half of the activations it would stream alone: the shared-memory traffic per MMA halves. The leader's
// barriers count both CTAs (the peer's dequantising and epilogue warps arrive remotely, the peer's activation loads
// complete on the leader's barrier); the leader's commits arrive on both CTAs' barriers. No TMA multicast.
// WF: weight format, 0 = Q4 (the reference's tc_q4), 1 = Q8 (the tc_q8 it planned but never built): only the packed
// chunk layout and the dequantisation differ.
// SPLIT: split-K for tables with few row tiles (2560x6144 has 20): a cluster of a.splits CTAs shares one tile, CTA r
// taking its share of the K range (units of a.kunit K steps) through the unchanged pipeline. Each CTA stores its fp32
// partial accumulator in its own shared memory (the rings are idle by then), the cluster synchronises, and CTA r sums
// token slice r over the cluster's partials in rank order (distributed shared memory reads), so the result does not
// depend on timing: deterministic, unlike an atomic reduction. A second cluster barrier keeps every partial readable
// until all slices are done. One tile per cluster (the planner launches tiles x splits CTAs). With peer stores (the
// row split), each CTA then pushes its finished token slice to every peer; the row split uses the split count of the
// whole problem's one-GPU plan, so its result is the one-GPU result bit for bit.
// RB = 2 (opt-in, VKB_TC_RB=2): one CTA holds a 256-row tile as two 128-row blocks, each with its own accumulator
// (TMEM columns 0 and NT rounded up to 32), and every activation K step feeds the MMAs of both blocks: the activations
// are streamed from L2 once per 256 weight rows instead of once per 128 (that stream, N / 128 times the activations,
// takes two thirds of the one-block kernel's time at 12288x2560 x 512 tokens when its MMAs and dequantisation are
// compiled out). A slots hold one K step of both blocks (64 columns); dequantising group g (four warps) converts block
// g. Measured slower than one block at every shape (the MMA issue loop and the 2-slot A ring bound it first), so the
// planner never picks it.
template <typename OutT, int PK, bool P2P, int CG, int WF = 0, int RB = 1, bool SPLIT = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_q4_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap ts,
             const __grid_constant__ CUtensorMap tx, const __grid_constant__ TcArgs a) {
    static_assert(CG == 1 || (CG == 2 && !P2P), "peer stores use the one-CTA kernel");
    static_assert(WF == 0 || (WF == 1 && !P2P && CG == 1), "Q8 weights: the one-CTA kernel without peer stores");
    static_assert(RB == 1 || (RB == 2 && CG == 1 && !P2P && WF == 0), "two row blocks: the one-CTA Q4 kernel");
    static_assert(!SPLIT || (CG == 1 && RB == 1), "split-K: one-CTA tiles, one row block");
    constexpr int BMR = TC_BM * RB;                         // weight rows of a CTA's tile
    constexpr int SK = RB == 1 ? TC_SLOT : 1;               // K steps per A slot
    constexpr int SLOT_COLS = RB * SK * TC_ACOLS;           // TMEM columns per A slot (128, or 64 with two blocks)
    constexpr int PPITCH = tc_ppitch(PK, WF), PCHUNK = RB * tc_pchunk(PK, WF), SCOFF = BMR * PPITCH;
    constexpr int KSB = WF == 1 ? 64 : 32;   // code bytes per row per K step
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* sm = smem_raw + pad;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + a.bar_off);
    uint64_t* pfull = bars;                   // [np] packed chunk (codes + scales) landed
    uint64_t* pempty = pfull + a.np;          // [np] both dequant groups done with the chunk (8 warps)
    uint64_t* xfull = pempty + a.np;          // [nx] activation stage landed
    uint64_t* xempty = xfull + a.nx;          // [nx] MMAs of the stage done (tcgen05.commit)
    uint64_t* afull = xempty + a.nx;          // [na] dequantised slot written to TMEM (8 warps)
    uint64_t* aempty = afull + a.na;          // [na] MMAs of the slot done (tcgen05.commit)
    uint64_t* accfull = aempty + a.na;        // [nacc] a tile's MMAs done (tcgen05.commit)
    uint64_t* accempty = accfull + a.nacc;    // [nacc] the epilogue has read the accumulator (4 warps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + a.nacc);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's K steps [kofs, kofs + nk) of every tile (split-K: its rank's share of the units)
    int kofs = 0, nk = a.nk;
    uint32_t srank = 0;
    if constexpr (SPLIT) {
        srank = cluster_ctarank();
        const int nun = a.nk / a.kunit, lo = (int)srank * nun / a.splits, hi = ((int)srank + 1) * nun / a.splits;
        kofs = lo * a.kunit;
        nk = (hi - lo) * a.kunit;
    }
    const int nch = nk / PK, nxs = nk / a.xk, nslots = nk / SK;
    const int rbcol = (a.NT + 31) & ~31;   // TMEM columns between the row blocks' accumulators (32-aligned)
    // the CTA's place in its pair (CG = 2) and the pairs of the grid; a "unit" is a CTA (CG = 1) or a pair
    const uint32_t crank = CG == 2 ? cluster_ctarank() : 0u;
    const bool leader = crank == 0;
    const int units = CG == 2 || SPLIT ? (int)cluster_count_x() : (int)gridDim.x;
    const int unit = CG == 2 || SPLIT ? (int)cluster_id_x() : (int)blockIdx.x;
    // tiles of this unit: t = unit + i * units (a tile: 128 RB CG weight rows x NT tokens; this CTA's rows start at
    // row0_of(t), its tokens for the B operand at tok0_of(t) + crank NT / CG)
    const int ntl = unit < a.tiles ? (a.tiles - 1 - unit) / units + 1 : 0;
    auto tile_of = [&](int i) { return unit + i * units; };
    auto row0_of = [&](int t) { return (t % a.tiles_n) * (BMR * CG) + BMR * (int)crank; };
    auto tok0_of = [&](int t) { return (t / a.tiles_n) * a.NT; };
    // barrier helpers: waits that a peer CTA may have released acquire at cluster scope; arrivals that the MMA
    // issuer waits for go to the leader's barrier; commits of a pair's MMAs arrive in both CTAs
    auto wait_b = [&](uint64_t* bar, uint32_t par, unsigned err = DEV_ERR_WAIT_TIMEOUT) {
        if constexpr (CG == 2) return wait_parity_sleep_cl(bar, par, err);
        else return wait_parity_sleep(bar, par, err);
    };
    auto arrive_leader = [&](uint64_t* bar) {
        if constexpr (CG == 2) mbar_arrive_cluster(mapa_shared(smem_u32(bar), 0));
        else mbar_arrive(bar);
    };
    auto commit = [&](uint64_t* bar) {
        if constexpr (CG == 2) umma_commit_pair(bar);
        else umma_commit(bar);
    };
    const int total_ch = ntl * nch;

    auto issue_chunk = [&](int g, int b) {   // chunk g of this CTA's stream into ring slot b
        const int t = tile_of(g / nch), c = g % nch;
        uint8_t* dst = sm + a.p_off + b * PCHUNK;
        mbar_arrive_expect_tx(&pfull[b], (uint32_t)PCHUNK);
        tma_load_2d(dst, &tq, (kofs + c * PK) * (KSB / 8), row0_of(t), &pfull[b]);   // PK K steps of codes, 8-B units
        tma_load_2d(dst + SCOFF, &ts, (kofs + c * PK) * 2, row0_of(t), &pfull[b]);    // 2 PK (+ pad) fp16 scales
    };

    // peer stores: some thread of this CTA gave up a wait (its part of the call is missing); the word after the TMEM
    // address in the barrier block
    volatile int* cta_failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
    pdl_trigger();
    if (threadIdx.x == 0) {
        *cta_failed = 0;
        for (int i = 0; i < a.np; ++i) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], TC_NDQ);
        }
        for (int i = 0; i < a.nx; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], 1);
        }
        for (int i = 0; i < a.na; ++i) {
            mbar_init(&afull[i], TC_NDQ * CG);     // the leader's counts both CTAs' dequantising warps
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < a.nacc; ++i) {
            mbar_init(&accfull[i], 1);
            mbar_init(&accempty[i], TC_NEPI * CG);   // the leader's counts both CTAs' epilogue warps
        }
        fence_mbar_init();
        // the first chunks start now, before the TMEM allocation and the block-wide barrier
        prefetch_tmap(&tq);
        prefetch_tmap(&ts);
        for (int g = 0; g < min(total_ch, a.np); ++g) issue_chunk(g, g);
    }
    if (warp == 1) tmem_alloc<CG>(tmem_slot, (uint32_t)a.tmem_cols);
    tc_fence_before();
    if constexpr (CG == 2) cluster_sync();   // both CTAs' barriers exist before any remote arrive or pair load
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    // ---- epilogue of one tile, by one participant warp ----
    // A warp reads TMEM lanes 32 (w % 4).. (weight rows): the `parts` participants of a lane quarter take interleaved
    // 32-token chunks (sub: this warp's index among them) and store y directly (tc_epi_store; a warp's store covers
    // 32 consecutive outputs of one token: 64 or 128 contiguous bytes). With `arrive` the warp then
    // releases the accumulator to the MMA warp. With peer stores, the participants of a tile then push the finished
    // tile from this rank's y to every peer (p2p_push: 16-byte words) while the MMA warp works on the next tile; every
    // participant passes the tile's named barrier (id 2 for the epilogue warps alone, 3 for the last tile's three
    // participants per lane quarter), also after a failed wait (it then skips the work), so that no barrier waits for
    // a warp that left.
    // The epilogue warps empty every tile (with two accumulators, behind the next tile's MMAs); the dequantising
    // warps, idle by then, join for the CTA's last tile, whose epilogue nothing else overlaps. (Joining every tile
    // when there is one accumulator was measured slower: the epilogue code inside the dequantising loop, inline or
    // called, slows that loop by more than the shorter epilogue gains.)
    bool epi_began = false;
    auto epi_tile = [&](int i, int sub, int parts, bool arrive) {
        if (!epi_began) {
            epi_began = true;
            pdl_wait();   // y may still be read or written by the previous grid
            if constexpr (P2P && !SPLIT) {   // this rank's copy may now be written; wait until every peer's may be
                const uint32_t e = p2p_epoch(a.pp);
                if (warp == TC_WEPI0 && lane == 0) p2p_post_ready(a.pp, e);
                if (lane == 0 && !p2p_wait_ready(a.pp, e)) ok = false;
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            }
        }
        const int acc = i % a.nacc, t = tile_of(i), row0 = row0_of(t), tok0 = tok0_of(t);
        const int q = warp & 3;
        if (ok) ok = __all_sync(0xffffffffu, wait_b(&accfull[acc], (i / a.nacc) & 1));
        if (ok) {
            tc_fence_after();
#pragma unroll
            for (int rb = 0; rb < RB; ++rb) {   // row block rb: accumulator columns from rb rbcol, rows from 128 rb
                const uint32_t tq_addr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * 128 + rb * rbcol);
                if constexpr (SPLIT)
                    tc_epi_stash(a, tq_addr, 32 * q + lane, tok0, sub, parts, smem_u32(sm));
                else
                    tc_epi_store<OutT>(a, tq_addr, row0 + rb * TC_BM + 32 * q + lane, tok0, sub, parts);
            }
            // every TMEM read of this accumulator has completed: the MMA warp may overwrite it
            if (arrive) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_leader(&accempty[acc]);
            }
        }
        if constexpr (P2P && !SPLIT) {   // the tile is complete in this rank's copy: its participants push it to every peer
            // one barrier id per participant count: the epilogue warps' earlier tiles (128 threads) may still be
            // at their barrier when the dequantising warps reach the last tile's (384); two counts on one named
            // barrier at once is undefined (on B200 it raised an illegal-instruction fault)
            named_sync(parts == 1 ? 2u : 3u, 128u * (uint32_t)parts);
            if (ok) tc_push_tile<OutT>(a, row0, tok0, (warp >= TC_WEPI0 ? warp - TC_WEPI0 : warp - TC_WDQ0 + 4) * 32
                                       + lane, 128 * parts);
        }
    };

    if (warp == 0) {
        // ===================== P ring producer =====================
        for (int g = a.np; g < total_ch; ++g) {
            const int b = g % a.np, rnd = g / a.np;
            ok = __all_sync(0xffffffffu, wait_parity_sleep(&pempty[b], (rnd - 1) & 1));
            if (!ok) break;
            if (elect_one()) issue_chunk(g, b);
            __syncwarp();
        }
        // drain: the loads still in flight land before exit
        for (int g = ok ? max(0, total_ch - a.np) : total_ch; g < total_ch; ++g)
            if (!wait_parity_sleep(&pfull[g % a.np], (g / a.np) & 1, DEV_ERR_DRAIN_TIMEOUT)) break;
    } else if (warp == 2 || warp == 3) {
        // ===================== X ring producers (activations: after the previous grid) =====================
        // warp 2 loads the even stages of the CTA's stream, warp 3 the odd ones (nx is even: fixed ring slots)
        const int par = warp - 2;
        if (elect_one()) prefetch_tmap(&tx);
        pdl_wait();
        const int total_xs = ntl * nxs;
        int last = -1;
        for (int gs = par; gs < total_xs; gs += 2) {
            const int b = gs % a.nx, rnd = gs / a.nx;
            if (rnd > 0) ok = __all_sync(0xffffffffu, wait_b(&xempty[b], (rnd - 1) & 1));
            if (!ok) break;
            if (elect_one()) {
                const int t = tile_of(gs / nxs), xs = gs % nxs;
                if constexpr (CG == 1) {
                    mbar_arrive_expect_tx(&xfull[b], (uint32_t)a.x_stage);
                    tma_load_3d(sm + a.x_off + b * a.x_stage, &tx, 0, tok0_of(t), kofs + xs * a.xk, &xfull[b]);
                } else {   // this CTA's half of the tokens; both halves complete on the leader's barrier
                    if (leader) mbar_arrive_expect_tx(&xfull[b], (uint32_t)(2 * a.x_stage));
                    tma_load_3d_cg2(sm + a.x_off + b * a.x_stage, &tx, 0, tok0_of(t) + (int)crank * (a.NT / 2),
                                    xs * a.xk, mapa_shared(smem_u32(&xfull[b]), 0));
                }
            }
            __syncwarp();
            last = gs;
        }
        // drain: the loads still in flight land before exit (the leader's barrier counts the peer's loads too, and
        // the pair leaves only together)
        if (leader)
            for (int gs = last; gs >= 0 && gs > last - a.nx; gs -= 2)
                if (!wait_b(&xfull[gs % a.nx], (gs / a.nx) & 1, DEV_ERR_DRAIN_TIMEOUT)) break;
    } else if (warp == 1 && leader) {
        // ===================== MMA issuer (the pair leader's, CG = 2) =====================
        // Per slot: wait for its A (TMEM) and the X stages its SK K steps read, then 4 UMMAs per K step and row block
        // (16 per slot with one block), issued by one elected lane, the warp reconverged after each issue block.
        // tcgen05.mma issue blocks while the tensor pipe's queue is full (it holds about one instruction), so every
        // cycle this warp spends between two UMMAs is tensor-pipe idle time. Its waits therefore test the phase first
        // (mbarrier.test_wait, in wait_parity_sleep) and sleep in try_wait only when it is not complete (measured: a
        // sleeping try_wait on a completed phase cost ~150-300 cycles per wait, ~150 cycles per UMMA in all; testing
        // first took 5 % off 12288x2560 at 512 tokens; one lane running the loop alone, or issuing without elect.sync
        // and __syncwarp, was 4-30 % slower). When the X ring holds at least two slots of K steps all of a slot's X
        // waits come first and its UMMAs issue back to back; otherwise (large token tiles, shallow X ring) the waits
        // interleave with the K steps so that each X stage is released as soon as its own MMAs complete.
        {
            auto wait_m = [&](uint64_t* bar, uint32_t par) { return __all_sync(0xffffffffu, wait_b(bar, par)); };
            const uint32_t idesc = umma_idesc_f16(a.NT, TC_BM * CG);
            const uint32_t xtile = (uint32_t)(a.NT / CG) * 128;   // one K step of this CTA's tokens in a stage
            const bool hoist = a.nx * a.xk >= 2 * SK;
            // K step j of the slot at ta (X at sb, K step it of the tile): row block rb's A at slot column
            // (j RB + rb) 32, its accumulator at td + rb rbcol
            auto issue_k = [&](uint32_t td, uint32_t ta, uint32_t sb, int j, int it) {
#pragma unroll
                for (int kk = 0; kk < TC_BK / 16; ++kk) {   // 16 k: 8 TMEM columns of A, 32 B of a B row
#pragma unroll
                    for (int rb = 0; rb < RB; ++rb) {
                        const uint32_t tdr = td + (uint32_t)(rb * rbcol);
                        const uint32_t tar = ta + (uint32_t)((j * RB + rb) * TC_ACOLS + 8 * kk);
                        if constexpr (CG == 2)
                            umma_f16_ts_cg2(tdr, tar, umma_desc_sw128(sb + 32 * kk), idesc, (it | kk) != 0);
                        else
                            umma_f16_ts(tdr, tar, umma_desc_sw128(sb + 32 * kk), idesc, (it | kk) != 0);
                    }
                }
            };
            int ab = 0, arnd = 0, xb = 0, xrnd = 0, xj = 0;
            for (int i = 0; i < ntl && ok; ++i) {
                const int acc = i % a.nacc;
                if (i >= a.nacc) ok = wait_m(&accempty[acc], ((i / a.nacc) - 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t td = tmem + (uint32_t)(acc * 128);
                for (int sl = 0; sl < nslots && ok; ++sl) {
                    ok = wait_m(&afull[ab], arnd & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t ta = tmem + (uint32_t)(a.a_col0 + ab * SLOT_COLS);
                    if (hoist) {
                        uint32_t sb[SK];
                        int rel[SK];   // X stage to release after K step j (-1: none)
#pragma unroll
                        for (int j = 0; j < SK; ++j) {
                            if (xj == 0 && ok) ok = wait_m(&xfull[xb], xrnd & 1);
                            sb[j] = smem_u32(sm + a.x_off + xb * a.x_stage) + xj * xtile;
                            rel[j] = xj + 1 == a.xk ? xb : -1;
                            if (++xj == a.xk) {
                                xj = 0;
                                if (++xb == a.nx) { xb = 0; ++xrnd; }
                            }
                        }
                        if (!ok) break;
                        tc_fence_after();
                        if (elect_one()) {
#pragma unroll
                            for (int j = 0; j < SK; ++j) {
                                issue_k(td, ta, sb[j], j, sl * SK + j);
                                if (rel[j] >= 0) commit(&xempty[rel[j]]);   // free the stage after these MMAs
                            }
                            commit(&aempty[ab]);
                        }
                        __syncwarp();
                    } else {
#pragma unroll
                        for (int j = 0; j < SK; ++j) {
                            if (xj == 0) {
                                ok = wait_m(&xfull[xb], xrnd & 1);
                                if (!ok) break;
                                tc_fence_after();
                            }
                            const uint32_t sb = smem_u32(sm + a.x_off + xb * a.x_stage) + xj * xtile;
                            const bool last_x = xj + 1 == a.xk;
                            if (elect_one()) {
                                issue_k(td, ta, sb, j, sl * SK + j);
                                if (last_x) commit(&xempty[xb]);
                                if (j == SK - 1) commit(&aempty[ab]);
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
                if (!ok) break;
                if (elect_one()) commit(&accfull[acc]);   // the tile's MMAs are done: its accumulator is final
                __syncwarp();
            }
        }
    } else if (warp >= TC_WDQ0 && warp < TC_WEPI0) {
        // ===================== dequantise (two groups: half a slot each, or one row block each) ==============
        const int dw = warp - TC_WDQ0;            // 0..7
        const int grp = dw >> 2;                  // RB = 1: K steps 2 grp, 2 grp + 1 of every slot; RB = 2: block grp
        const int qtr = warp & 3;                 // TMEM lane quarter this warp may access
        if constexpr (RB == 2) {
            // one K step per slot; group grp converts row block grp (tile row 128 grp + TMEM lane)
            const int r = grp * TC_BM + qtr * 32 + lane;
            const uint32_t prow = smem_u32(sm + a.p_off) + r * PPITCH;
            const uint32_t srow = smem_u32(sm + a.p_off) + SCOFF + r * TC_SPITCH;
            const uint32_t tlane = tmem + ((uint32_t)(32 * qtr) << 16) + (uint32_t)(a.a_col0 + grp * TC_ACOLS);
            for (int g = 0; g < total_ch && ok; ++g) {   // chunk g of the CTA's stream (tile g / nch)
                const int pb = g % a.np;
                if (!wait_parity_sleep(&pfull[pb], (g / a.np) & 1)) { ok = false; break; }
                uint32_t sw[PK];                                      // scales of the chunk's 2 PK groups
#pragma unroll
                for (int q4 = 0; q4 < PK / 4; ++q4) {
                    const uint4 t = lds128(srow + pb * PCHUNK + 16 * q4);
                    sw[4 * q4] = t.x; sw[4 * q4 + 1] = t.y; sw[4 * q4 + 2] = t.z; sw[4 * q4 + 3] = t.w;
                }
#pragma unroll
                for (int sc = 0; sc < PK; ++sc) {                     // K step sc of the chunk = one slot
                    const int sl = g * PK + sc, ab = sl % a.na;
                    const uint32_t pa = prow + pb * PCHUNK + sc * KSB;
                    const uint4 w0 = lds128(pa), w1 = lds128(pa + 16);
                    if (sc == PK - 1) {                               // this warp's last read of the chunk
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&pempty[pb]);
                    }
                    const uint32_t lo = (sw[sc] & 0xFFFFu) * 0x00010001u, hi = (sw[sc] >> 16) * 0x00010001u;
                    uint32_t v[32];
                    dequant8_to(w0.x, lo, v + 0);
                    dequant8_to(w0.y, lo, v + 4);
                    dequant8_to(w0.z, lo, v + 8);
                    dequant8_to(w0.w, lo, v + 12);
                    dequant8_to(w1.x, hi, v + 16);
                    dequant8_to(w1.y, hi, v + 20);
                    dequant8_to(w1.z, hi, v + 24);
                    dequant8_to(w1.w, hi, v + 28);
                    if (sl >= a.na && !wait_b(&aempty[ab], ((sl / a.na) - 1) & 1)) { ok = false; break; }
                    tc_fence_after();                                 // the slot's previous MMAs are done
                    tmem_st32(tlane + (uint32_t)(ab * SLOT_COLS), v);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) arrive_leader(&afull[ab]);
                }
            }
        } else {
            const int r = qtr * 32 + lane;            // weight row of the tile = TMEM lane
            const uint32_t prow = smem_u32(sm + a.p_off) + r * PPITCH;
            const uint32_t srow = smem_u32(sm + a.p_off) + SCOFF + r * TC_SPITCH;
            const uint32_t tlane = tmem + ((uint32_t)(32 * qtr) << 16) + (uint32_t)(a.a_col0 + 2 * grp * TC_ACOLS);
            for (int g = 0; g < total_ch && ok; ++g) {   // chunk g of the CTA's stream (tile g / nch)
                const int pb = g % a.np;
                if (!wait_parity_sleep(&pfull[pb], (g / a.np) & 1)) { ok = false; break; }
                uint32_t sw[PK];                                          // scales of the chunk's 2 PK groups
#pragma unroll
                for (int q4 = 0; q4 < PK / 4; ++q4) {
                    const uint4 t = lds128(srow + pb * PCHUNK + 16 * q4);
                    sw[4 * q4] = t.x; sw[4 * q4 + 1] = t.y; sw[4 * q4 + 2] = t.z; sw[4 * q4 + 3] = t.w;
                }
#pragma unroll
                for (int sc = 0; sc < PK / TC_SLOT; ++sc) {            // slots of this chunk
                    const int sl = g * (PK / TC_SLOT) + sc;             // slot of the CTA's stream
                    const int ab = sl % a.na;
                    // this group's two K steps of the slot: both loads first, then both conversions, one TMEM store
                    const int sub0 = sc * TC_SLOT + 2 * grp;            // first of the two sub-steps within the chunk
                    const uint32_t pa = prow + pb * PCHUNK + sub0 * KSB;
                    uint4 w0 = lds128(pa), w1 = lds128(pa + 16), w2 = lds128(pa + 32), w3 = lds128(pa + 48);
                    const uint32_t sa = grp ? sw[sc * TC_SLOT + 2] : sw[sc * TC_SLOT];       // static indices
                    const uint32_t sb = grp ? sw[sc * TC_SLOT + 3] : sw[sc * TC_SLOT + 1];
                    if (WF == 0 && sc == PK / TC_SLOT - 1) {            // this warp's last read of the chunk
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&pempty[pb]);
                    }
                    uint32_t v[64];
                    const uint32_t a_lo = (sa & 0xFFFFu) * 0x00010001u, a_hi = (sa >> 16) * 0x00010001u;
                    const uint32_t b_lo = (sb & 0xFFFFu) * 0x00010001u, b_hi = (sb >> 16) * 0x00010001u;
                    if constexpr (WF == 0) {   // Q4: 32 code bytes per K step (w0-w1: step A, w2-w3: step B)
                        dequant8_to(w0.x, a_lo, v + 0);
                        dequant8_to(w0.y, a_lo, v + 4);
                        dequant8_to(w0.z, a_lo, v + 8);
                        dequant8_to(w0.w, a_lo, v + 12);
                        dequant8_to(w1.x, a_hi, v + 16);
                        dequant8_to(w1.y, a_hi, v + 20);
                        dequant8_to(w1.z, a_hi, v + 24);
                        dequant8_to(w1.w, a_hi, v + 28);
                        dequant8_to(w2.x, b_lo, v + 32);
                        dequant8_to(w2.y, b_lo, v + 36);
                        dequant8_to(w2.z, b_lo, v + 40);
                        dequant8_to(w2.w, b_lo, v + 44);
                        dequant8_to(w3.x, b_hi, v + 48);
                        dequant8_to(w3.y, b_hi, v + 52);
                        dequant8_to(w3.z, b_hi, v + 56);
                        dequant8_to(w3.w, b_hi, v + 60);
                    } else {   // Q8: 64 code bytes per K step; w0-w3 hold step A, step B is loaded after A is converted
                        const uint4 wa[4] = {w0, w1, w2, w3};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {   // 16 codes per uint4: groups of 32 = two uint4
                            const uint32_t s2 = i < 2 ? a_lo : a_hi;
                            dequant4_q8_to(wa[i].x, s2, v + 8 * i);
                            dequant4_q8_to(wa[i].y, s2, v + 8 * i + 2);
                            dequant4_q8_to(wa[i].z, s2, v + 8 * i + 4);
                            dequant4_q8_to(wa[i].w, s2, v + 8 * i + 6);
                        }
                        w0 = lds128(pa + 64); w1 = lds128(pa + 80); w2 = lds128(pa + 96); w3 = lds128(pa + 112);
                        const uint4 wb[4] = {w0, w1, w2, w3};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t s2 = i < 2 ? b_lo : b_hi;
                            dequant4_q8_to(wb[i].x, s2, v + 32 + 8 * i);
                            dequant4_q8_to(wb[i].y, s2, v + 32 + 8 * i + 2);
                            dequant4_q8_to(wb[i].z, s2, v + 32 + 8 * i + 4);
                            dequant4_q8_to(wb[i].w, s2, v + 32 + 8 * i + 6);
                        }
                        if (sc == PK / TC_SLOT - 1) {                   // this warp's last read of the chunk
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&pempty[pb]);
                        }
                    }
                    if (sl >= a.na && !wait_b(&aempty[ab], ((sl / a.na) - 1) & 1)) { ok = false; break; }
                    tc_fence_after();                                   // the slot's previous MMAs are done
                    tmem_st64(tlane + (uint32_t)(ab * TC_SLOT * TC_ACOLS), v);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) arrive_leader(&afull[ab]);
                }
            }
        }
    }
    // ===================== epilogue =====================
    if (warp >= TC_WEPI0) {   // every tile
        for (int i = 0; i < ntl && (ok || P2P); ++i) epi_tile(i, 0, i == ntl - 1 ? 3 : 1, true);
    } else if (warp >= TC_WDQ0 && ntl > 0 && (ok || P2P)) {   // the last tile
        epi_tile(ntl - 1, 1 + ((warp - TC_WDQ0) >> 2), 3, false);
    }
    // split-K: the cluster's partials -> y, CTA r summing token slice r over the ranks in order
    if constexpr (SPLIT) {
        cluster_sync();   // every CTA's partial is in its shared memory
        pdl_wait();       // y may still be read or written by the previous grid
        uint32_t e = 0;
        if constexpr (P2P) {   // this rank's copy may now be written
            e = p2p_epoch(a.pp);
            if (threadIdx.x == 0) p2p_post_ready(a.pp, e);
        }
        const int t = tile_of(0), row0 = row0_of(t), tok0 = tok0_of(t), ntok = min(a.NT, a.M - tok0);
        const int lo = (int)srank * ntok / a.splits, hi = ((int)srank + 1) * ntok / a.splits;
        if (ntl > 0) {
            OutT* y = reinterpret_cast<OutT*>(a.y);
            const int n = row0 + 4 * lane;
            for (int tk = lo + warp; tk < hi; tk += TC_THREADS / 32) {
                const uint32_t off = smem_u32(sm) + (uint32_t)((tk * TC_BM + 4 * lane) * 4);
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int r = 0; r < a.splits; ++r) {
                    const float4 v = ld_cluster_f4(mapa_shared(off, (uint32_t)r));
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
                OutT* yp = y + (size_t)(tok0 + tk) * a.ldy + a.ycol0 + n;
                if (n < a.N) yp[0] = tc_out<OutT>(acc.x);
                if (n + 1 < a.N) yp[1] = tc_out<OutT>(acc.y);
                if (n + 2 < a.N) yp[2] = tc_out<OutT>(acc.z);
                if (n + 3 < a.N) yp[3] = tc_out<OutT>(acc.w);
            }
        }
        cluster_sync();   // no CTA releases its shared memory while a peer still reads its partial
        if constexpr (P2P) {
            // the CTA's token slice of the tile is complete in this rank's copy (the barrier above orders every
            // thread's stores): push it to every peer once every peer's CTA of this index accepts writes
            bool rd = ok;
            if (lane == 0 && rd) rd = p2p_wait_ready(a.pp, e);
            rd = __shfl_sync(0xffffffffu, rd ? 1 : 0, 0) != 0;
            ok = ok && rd;
            if (rd && ntl > 0 && hi > lo) {
                const int cols = min(TC_BM, a.N - row0);
                const size_t pitch = (size_t)a.ldy * sizeof(OutT);
                const size_t off = ((size_t)(tok0 + lo) * a.ldy + a.ycol0 + row0) * sizeof(OutT);
                p2p_push(a.pp, hi - lo, cols * (int)sizeof(OutT), off | pitch,
                         [&](int r) { return off + (size_t)r * pitch; }, threadIdx.x, TC_THREADS);
            }
        }
    }
    // teardown: every MMA has completed (the epilogue waited on each accumulator) before TMEM is released
    if (warp == 1 && !ok && ntl > 0) wait_b(&accfull[(ntl - 1) % a.nacc], ((ntl - 1) / a.nacc) & 1,
                                            DEV_ERR_DRAIN_TIMEOUT);
    if (P2P && !ok) *cta_failed = 1;
    tc_fence_before();
    // a pair leaves together: no remote arrive, pair load or MMA touches a CTA that has released its TMEM or exited
    if constexpr (CG == 2) cluster_sync();
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<CG>(tmem, (uint32_t)a.tmem_cols);
    }
    // every store of this CTA precedes the barrier above; thread 0's system-scope fence in p2p_finish releases them
    // all (cumulativity), so no per-thread fence is needed
    if (P2P && threadIdx.x == 0) p2p_finish(a.pp, *cta_failed == 0);
}

}  // namespace vkb
