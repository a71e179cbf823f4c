// The general-shape decode kernel: any K % 32 == 0, any pointer alignment the formats allow, 1..8 tokens, dense or
// MoE. One warp per (output row, slot); lanes stride over the 32-value groups; exact codes, fp32 sums (the reference's
// fused_q4 structure, src/bakeoff.cu:70-113). It is the path for shapes the TMA kernel does not take (K % 256 != 0
// or unaligned buffers), so it favours simplicity over speed.
#pragma once

#include "qmv.cuh"

namespace vkb {

template <int F>
__device__ __forceinline__ int code_at(const void* q, size_t row, int K, int k) {
    if constexpr (F == FMT_Q4) {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(q) + row * (K / 8) + k / 8);
        return (int)((w >> (4 * (k & 7))) & 15u) - 8;
    } else if constexpr (F == FMT_Q8) {
        return (int)__ldg(reinterpret_cast<const int8_t*>(q) + row * K + k);
    } else {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(q) + row * (K / 16) + k / 16);
        return (int)((w >> (2 * (k & 15))) & 3u) - 2;
    }
}

// Dense: grid.y = 1, M tokens per warp. MoE: grid.y = T*topk slots, one token per warp (idx != nullptr).
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
    float acc[QMV_MAXTOK];
#pragma unroll
    for (int m = 0; m < QMV_MAXTOK; ++m) acc[m] = 0.f;
    const int KG = K / 32;
    for (int grp = lane; grp < KG; grp += 32) {
        const float sc = __half2float(__ldg(s + wrow * KG + grp));
        float part[QMV_MAXTOK];
#pragma unroll
        for (int m = 0; m < QMV_MAXTOK; ++m) part[m] = 0.f;
        for (int i = 0; i < 32; ++i) {
            const int k = 32 * grp + i;
            const float c = (float)code_at<F>(q, wrow, K, k);
#pragma unroll
            for (int m = 0; m < QMV_MAXTOK; ++m)
                if (m < ntok) part[m] = fmaf(c, __half2float(__ldg(x + (size_t)(tok0 + m) * K + k)), part[m]);
        }
#pragma unroll
        for (int m = 0; m < QMV_MAXTOK; ++m) acc[m] = fmaf(part[m], sc, acc[m]);
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

}  // namespace vkb
