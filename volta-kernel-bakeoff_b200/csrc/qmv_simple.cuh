// The general-shape decode kernel: any K % 32 == 0, any pointer alignment the formats allow, 1..8 tokens, dense or
// MoE. One warp per (output row, slot); lanes stride over 8-value chunks with vector loads; exact codes, fp32 sums (the
// reference's fused_q4 structure, src/bakeoff.cu:70-113). It is the path for shapes the TMA kernel does not take
// (K % 256 != 0 or unaligned buffers).
#pragma once

#include "qmv.cuh"

namespace vkb {

// Eight consecutive codes 8c..8c+7 of a row (exact integers).
template <int F>
__device__ __forceinline__ void codes8(const void* q, size_t row, int K, int c, bool q8_vec, int (&v)[8]) {
    if constexpr (F == FMT_Q4) {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(q) + row * (K / 8) + c);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = (int)((w >> (4 * j)) & 15u) - 8;
    } else if constexpr (F == FMT_Q8) {
        const int8_t* p = reinterpret_cast<const int8_t*>(q) + row * K + 8 * c;
        if (q8_vec) {   // 8-byte aligned rows
            const uint2 w = __ldg(reinterpret_cast<const uint2*>(p));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[j] = (int)(int8_t)(w.x >> (8 * j));
                v[4 + j] = (int)(int8_t)(w.y >> (8 * j));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = (int)__ldg(p + j);
        }
    } else {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(q) + row * (K / 16) + (c >> 1)) >> (16 * (c & 1));
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = (int)((w >> (2 * j)) & 3u) - 2;
    }
}

// Eight consecutive fp16 activations as fp32 (one 16-byte load when x is 16-byte aligned).
__device__ __forceinline__ void x8(const __half* x, bool x_vec, float (&f)[8]) {
    if (x_vec) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(x));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            f[2 * j] = half_lo_f32(w[j]);
            f[2 * j + 1] = half_hi_f32(w[j]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = __half2float(__ldg(x + j));
    }
}

// Dense: grid.y = 1, M tokens per warp. MoE: grid.y = T*topk slots, one token per warp (idx != nullptr). Lanes take
// 8-value chunks (one code word / 16 bytes of x each); per chunk the 8 products are summed in fp32, scaled by the
// group's scale and added to the lane's sum; a warp shuffle reduces the lanes.
template <int F, typename OutT>
__global__ void __launch_bounds__(256) qmv_simple_kernel(const void* __restrict__ q, const __half* __restrict__ s,
                                                         const __half* __restrict__ x, OutT* __restrict__ y,
                                                         const int32_t* __restrict__ idx, int N, int K, int M,
                                                         int topk, int E_local, int e0, int zero_foreign) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int row = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    if (row >= N) return;   // whole warps leave together
    size_t wrow = row;
    int slot = 0, ntok = M, tok0 = 0;
    if (idx != nullptr) {
        slot = blockIdx.y;
        const int e = __ldg(idx + slot) - e0;
        if (e < 0 || e >= E_local) {   // another rank's expert: zero for the expert-parallel combine, or untouched
            if (zero_foreign && lane == 0) y[(size_t)slot * N + row] = to_out<OutT>(0.f);
            return;
        }
        wrow = (size_t)e * N + row;
        ntok = 1;
        tok0 = slot / topk;
    }
    const bool x_vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    const bool q8_vec = (reinterpret_cast<uintptr_t>(q) & 7u) == 0;
    float acc[QMV_MAXTOK];
#pragma unroll
    for (int m = 0; m < QMV_MAXTOK; ++m) acc[m] = 0.f;
    const int KG = K / 32;
    for (int c = lane; c < K / 8; c += 32) {
        const float sc = __half2float(__ldg(s + wrow * KG + (c >> 2)));
        int v[8];
        codes8<F>(q, wrow, K, c, q8_vec, v);
#pragma unroll
        for (int m = 0; m < QMV_MAXTOK; ++m) {
            if (m < ntok) {
                float xf[8];
                x8(x + (size_t)(tok0 + m) * K + 8 * c, x_vec, xf);
                float part = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) part = fmaf((float)v[j], xf[j], part);
                acc[m] = fmaf(part, sc, acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < QMV_MAXTOK; ++m) {
        float v = acc[m];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
        if (lane == 0 && m < ntok) {
            const size_t yrow = idx != nullptr ? (size_t)slot : (size_t)m;
            y[yrow * N + row] = to_out<OutT>(v);
        }
    }
}

// MoE on the general path: block (row block, local expert e) gathers the slots of expert e0 + e from the index list
// (shared memory), then each warp takes rows of the block and reads each row's codes once for up to 8 of those slots
// at a time. Grid y = E_local (+ 1 block row that zeroes the foreign slots when zero_foreign). Slot order inside an
// expert does not matter: every slot is computed on its own.
constexpr int QMV_SIMPLE_MOE_ROWS = 64;   // rows per block (8 warps x 8 rows)

template <int F, typename OutT>
__global__ void __launch_bounds__(256) qmv_simple_moe_kernel(const void* __restrict__ q, const __half* __restrict__ s,
                                                             const __half* __restrict__ x, OutT* __restrict__ y,
                                                             const int32_t* __restrict__ idx, int N, int K, int T,
                                                             int topk, int E_local, int e0, int zero_foreign) {
    extern __shared__ int sm_slots[];
    __shared__ int nsl;
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nslots = T * topk;
    const int r0 = blockIdx.x * QMV_SIMPLE_MOE_ROWS, r1 = min(N, r0 + QMV_SIMPLE_MOE_ROWS);
    if ((int)blockIdx.y == E_local) {   // zero the slots of experts outside the pool (expert-parallel combine)
        for (int i = warp; i < nslots; i += 8) {
            const int e = __ldg(idx + i) - e0;
            if (e >= 0 && e < E_local) continue;
            for (int r = r0 + lane; r < r1; r += 32) y[(size_t)i * N + r] = to_out<OutT>(0.f);
        }
        return;
    }
    const int e = blockIdx.y;
    if (threadIdx.x == 0) nsl = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < nslots; i += blockDim.x)
        if (__ldg(idx + i) - e0 == e) sm_slots[atomicAdd(&nsl, 1)] = i;
    __syncthreads();
    const int ns = nsl;
    if (ns == 0) return;
    const bool x_vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    const bool q8_vec = (reinterpret_cast<uintptr_t>(q) & 7u) == 0;
    const int KG = K / 32;
    for (int row = r0 + warp; row < r1; row += 8) {
        const size_t wrow = (size_t)e * N + row;
        for (int p0 = 0; p0 < ns; p0 += QMV_MAXTOK) {
            const int ntok = min(QMV_MAXTOK, ns - p0);
            float acc[QMV_MAXTOK];
#pragma unroll
            for (int m = 0; m < QMV_MAXTOK; ++m) acc[m] = 0.f;
            for (int c = lane; c < K / 8; c += 32) {
                const float sc = __half2float(__ldg(s + wrow * KG + (c >> 2)));
                int v[8];
                codes8<F>(q, wrow, K, c, q8_vec, v);
#pragma unroll
                for (int m = 0; m < QMV_MAXTOK; ++m) {
                    if (m < ntok) {
                        float xf[8];
                        x8(x + (size_t)(sm_slots[p0 + m] / topk) * K + 8 * c, x_vec, xf);
                        float part = 0.f;
#pragma unroll
                        for (int j = 0; j < 8; ++j) part = fmaf((float)v[j], xf[j], part);
                        acc[m] = fmaf(part, sc, acc[m]);
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < QMV_MAXTOK; ++m) {
                float v = acc[m];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
                if (lane == 0 && m < ntok) y[(size_t)sm_slots[p0 + m] * N + row] = to_out<OutT>(v);
            }
        }
    }
}

}  // namespace vkb
