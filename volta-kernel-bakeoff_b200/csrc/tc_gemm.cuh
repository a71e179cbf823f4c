// Prompt GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), Q4 weights, sm_100a.
//
//   y[m][n] = sum_k x[m][k] * w[n][k],  w = (code - 8) * scale rounded to fp16 (the reference's tc_q4 unpack,
//   src/stage4_tc.cuh:25-36: exact code, one fp16 multiply by the group scale), fp32 accumulation, fp16/fp32 out.
//
// One CTA computes a 128-row (weights) x NT-column (tokens) tile of y^T in TMEM:
//   warp 0      TMA producer: per 64-value K step, the packed codes of 128 rows (128 x 32 B) and the activations of
//               NT tokens (NT x 128 B, 128B-swizzled: exactly the K-major UMMA B layout); the tile's scales once.
//   warp 1      allocates TMEM, and one thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=NT, K=16) x4 per
//               step, committing each stage back to the producer.
//   warps 2-9   dequantise each step's codes into the 128B-swizzled K-major A tile (one 16-byte chunk = 8 k per
//               store), fence.proxy.async, and signal the MMA; at the end they read the accumulators with tcgen05.ld
//               and store y.
// No cluster multicast anywhere: the kernel also runs on row-split multi-GPU calls.
#pragma once

#include "ptx.cuh"

namespace vkb {

constexpr int TC_BM = 128;           // weight rows per CTA (UMMA M)
constexpr int TC_BK = 64;            // k per stage: one 128-byte swizzle row of fp16
constexpr int TC_NDQ = 8;            // dequantising / epilogue warps
constexpr int TC_THREADS = 32 * (2 + TC_NDQ);

struct TcArgs {
    void* y;            // [M][N]
    int M, N, K;
    int NT;             // tokens per CTA tile (multiple of 16, <= 256)
    int nstage;
    int a_off, b_off, p_off, stage_bytes;   // inside a stage: A tile, B tile, packed codes
    int s_off;          // scale block (128 rows x K/16 bytes + pad)
    int spitch;         // scale bytes per row
    int bar_off;
    int tmem_cols;
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

// One packed word (8 codes of one row, natural k order) -> 8 fp16 weights (code - 8) * scale, as one 16-byte chunk.
__device__ __forceinline__ uint4 dequant8(uint32_t v, uint32_t s2) {
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t b = prmt(v, 0u, 0x4040u | (j << 8) | j);                   // bytes [b_j, 0, b_j, 0]
        const uint32_t h = and_or(b, 0x00F0000Fu, 0x64006400u);                   // (1024 + lo, 1024 + 16 hi)
        const uint32_t c = h2_fma(h, 0x2C003C00u, 0xD480E408u);                    // exact (lo - 8, hi - 8)
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[j]) : "r"(c), "r"(s2));           // one rounding: code * scale
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
}

template <typename OutT> __device__ __forceinline__ OutT tc_out(float v);
template <> __device__ __forceinline__ __half tc_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float tc_out<float>(float v) { return v; }

template <typename OutT>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_q4_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap ts,
             const __grid_constant__ CUtensorMap tx, const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* sm = smem_raw + pad;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + a.bar_off);
    uint64_t* full = bars;                    // [nstage] TMA: packed codes + activations landed
    uint64_t* afull = bars + a.nstage;        // [nstage] dequantised A tile written
    uint64_t* empty = bars + 2 * a.nstage;    // [nstage] MMAs of the stage done (tcgen05.commit)
    uint64_t* sfull = bars + 3 * a.nstage;    // scales landed
    uint64_t* accum = sfull + 1;              // all MMAs done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * TC_BM, tok0 = blockIdx.y * a.NT;
    const int nk = a.K / TC_BK;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&afull[i], TC_NDQ);
            mbar_init(&empty[i], 1);
        }
        mbar_init(sfull, 1);
        mbar_init(accum, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, (uint32_t)a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (warp == 0) {
        // ===================== TMA producer =====================
        if (lane == 0) {
            prefetch_tmap(&tq);
            prefetch_tmap(&ts);
            prefetch_tmap(&tx);
            const uint32_t ptx_bytes = TC_BM * 32, xtx_bytes = (uint32_t)a.NT * 128;
            mbar_arrive_expect_tx(sfull, (uint32_t)(TC_BM * a.spitch));
            tma_load_2d(sm + a.s_off, &ts, 0, row0, sfull);
            const int pre = min(nk, a.nstage);
            for (int it = 0; it < pre; ++it) {   // weights first: they do not depend on the previous grid
                uint8_t* st = sm + it * a.stage_bytes;
                mbar_arrive_expect_tx(&full[it], ptx_bytes + xtx_bytes);
                tma_load_2d(st + a.p_off, &tq, it * 4, row0, &full[it]);   // 4 x 8-byte elements = 64 codes
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it)
                tma_load_2d(sm + it * a.stage_bytes + a.b_off, &tx, it * TC_BK, tok0, &full[it]);
            int stg = pre % a.nstage, rnd = pre / a.nstage;
            for (int it = pre; it < nk; ++it) {
                if (!wait_parity(&empty[stg], (rnd - 1) & 1)) { ok = false; break; }
                uint8_t* st = sm + stg * a.stage_bytes;
                mbar_arrive_expect_tx(&full[stg], ptx_bytes + xtx_bytes);
                tma_load_2d(st + a.p_off, &tq, it * 4, row0, &full[stg]);
                tma_load_2d(st + a.b_off, &tx, it * TC_BK, tok0, &full[stg]);
                if (++stg == a.nstage) { stg = 0; ++rnd; }
            }
            // drain: the last nstage loads (and the scales) land before exit
            int d = max(0, nk - a.nstage);
            int dstg = d % a.nstage, drnd = d / a.nstage;
            for (int it = d; it < nk; ++it) {
                if (!wait_parity(&full[dstg], drnd & 1, DEV_ERR_DRAIN_TIMEOUT)) break;
                if (++dstg == a.nstage) { dstg = 0; ++drnd; }
            }
            wait_parity(sfull, 0, DEV_ERR_DRAIN_TIMEOUT);
        }
    } else if (warp == 1) {
        // ===================== MMA issuer =====================
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(a.NT);
            int stg = 0, rnd = 0;
            for (int it = 0; it < nk; ++it) {
                if (!wait_parity(&afull[stg], rnd & 1) || !wait_parity(&full[stg], rnd & 1)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(sm + stg * a.stage_bytes + a.a_off);
                const uint32_t sb = smem_u32(sm + stg * a.stage_bytes + a.b_off);
#pragma unroll
                for (int kk = 0; kk < TC_BK / 16; ++kk)   // 16 k = 32 bytes further along the swizzled row
                    umma_f16(tmem, umma_desc_sw128(sa + 32 * kk), umma_desc_sw128(sb + 32 * kk), idesc,
                             (it | kk) != 0);
                umma_commit(&empty[stg]);
                if (++stg == a.nstage) { stg = 0; ++rnd; }
            }
            umma_commit(accum);   // arrives when every MMA issued above has completed
        }
    } else {
        // ===================== dequantise, then epilogue =====================
        const int dt = threadIdx.x - 64;          // 0..255
        const int r = dt >> 1, h = dt & 1;        // row of the tile, which 16 bytes of its 32-byte K step
        if (!wait_parity(sfull, 0)) ok = false;
        const uint8_t* srow = sm + a.s_off + r * a.spitch;
        int stg = 0, rnd = 0;
        for (int it = 0; it < nk && ok; ++it) {
            if (!wait_parity(&full[stg], rnd & 1)) { ok = false; break; }
            uint8_t* st = sm + stg * a.stage_bytes;
            const uint4 w = lds128(smem_u32(st + a.p_off + r * 32 + 16 * h));
            const uint16_t sbits = *reinterpret_cast<const uint16_t*>(srow + 2 * (2 * it + h));
            const uint32_t s2 = (uint32_t)sbits * 0x00010001u;
            const uint32_t abase = smem_u32(st + a.a_off) + (r >> 3) * 1024 + (r & 7) * 128;
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = 4 * h + j;   // 16-byte chunk (8 k values) of the 128-byte row
                sts128(abase + ((c ^ (r & 7)) << 4), dequant8(wv[j], s2));
            }
            fence_proxy_async_smem();   // generic-proxy stores -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[stg]);
            if (++stg == a.nstage) { stg = 0; ++rnd; }
        }
        // epilogue: warp w reads TMEM lanes 32*(w % 4).. (weight rows), columns of its half of the token tile
        pdl_wait();   // y may still be read or written by the previous grid
        if (ok && wait_parity(accum, 0)) {
            tc_fence_after();
            // 32-column chunks of the token tile alternate between the two warps that own each lane quarter; every
            // chunk lies inside the allocation (tmem_cols is a power of two >= NT and >= 32)
            const int q = warp & 3, half = (warp - 2) >> 2;
            const int n = row0 + 32 * q + lane;
            OutT* y = reinterpret_cast<OutT*>(a.y);
            for (int c = 32 * half; c < a.NT; c += 64) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int m = tok0 + c + j;
                    if (c + j < a.NT && m < a.M && n < a.N)
                        y[(size_t)m * a.N + n] = tc_out<OutT>(__uint_as_float(v[j]));
                }
            }
        }
    }
    // teardown: every MMA has completed (accum) before TMEM is released
    if (warp == 1 && lane == 0 && !ok) wait_parity(accum, 0, DEV_ERR_DRAIN_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
    }
}

}  // namespace vkb
