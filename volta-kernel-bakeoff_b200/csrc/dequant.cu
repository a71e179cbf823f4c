// Packed weights -> a dense fp16 (or bf16) copy, w[n][k] = code * scale with one rounding: the reference's dequant_q4
// (src/bakeoff.cu:52-68), which feeds its "dq4+cublas" control (a cuBLAS GEMM on the dequantised weights,
// src/bakeoff.cu:687-690), here for Q4, Q8 and 2-bit.
//
// HBM-bound (0.3-1.1 B read and 2 B written per weight). Lane l of a warp takes 8 consecutive values (a 16-byte
// output chunk): the warp's loads of codes (4 / 8 / 2 B per lane) and its stores (512 B) are contiguous, and the
// 4 lanes of one 32-value group read the same scale. fp32 product, round to nearest even: for fp16 the same value as
// the prompt GEMM's single fp16 multiply of the exact code by the scale.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vkb.h"
#include "vkb_internal.h"

namespace vkb {

template <int F, bool BF16>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ q, const __half* __restrict__ s,
                                                      uint4* __restrict__ w, long long chunks) {
    for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < chunks;
         c += (long long)gridDim.x * blockDim.x) {
        const float sc = __half2float(s[c >> 2]);   // 4 chunks of 8 per group of 32
        int code[8];
        if constexpr (F == VKB_FMT_Q4) {   // one word: code i in nibble i, stored as code + 8
            const uint32_t v = reinterpret_cast<const uint32_t*>(q)[c];
#pragma unroll
            for (int i = 0; i < 8; ++i) code[i] = (int)((v >> (4 * i)) & 15u) - 8;
        } else if constexpr (F == VKB_FMT_Q8) {   // eight int8 codes
            const uint2 v = reinterpret_cast<const uint2*>(q)[c];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                code[i] = (int)(int8_t)(v.x >> (8 * i));
                code[4 + i] = (int)(int8_t)(v.y >> (8 * i));
            }
        } else {   // 2-bit: half of a word, code i in bits 2i, 2i + 1, stored as code + 2
            const uint32_t v = reinterpret_cast<const uint16_t*>(q)[c];
#pragma unroll
            for (int i = 0; i < 8; ++i) code[i] = (int)((v >> (2 * i)) & 3u) - 2;
        }
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = (float)code[2 * i] * sc, b = (float)code[2 * i + 1] * sc;
            if constexpr (BF16) {
                o[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
                       ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
            } else {
                o[i] = (uint32_t)__half_as_ushort(__float2half_rn(a)) |
                       ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
            }
        }
        w[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

template <int F>
static void launch_dequant(const void* q, const void* s, void* w, long long chunks, bool bf16, cudaStream_t st) {
    const int threads = 256;
    const long long want = (chunks + threads - 1) / threads;
    const int grid = (int)(want < 148 * 16 ? want : 148 * 16);   // a grid-stride loop over 16 CTAs per SM at most
    if (bf16)
        dequant_kernel<F, true><<<grid, threads, 0, st>>>((const uint8_t*)q, (const __half*)s, (uint4*)w, chunks);
    else
        dequant_kernel<F, false><<<grid, threads, 0, st>>>((const uint8_t*)q, (const __half*)s, (uint4*)w, chunks);
}

}  // namespace vkb

using namespace vkb;

extern "C" int vkb_dequant(int fmt, const void* q, const void* s, void* w, int N, int K, int out_bf16,
                           vkb_stream_t stream) {
    if (!q || !s || !w || N < 1 || K < 32) return VKB_EINVAL;
    if (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8 && fmt != VKB_FMT_Q2) return VKB_EINVAL;
    if (K % 32 != 0 || (fmt == VKB_FMT_Q2 && K % 64 != 0)) return VKB_EUNSUPPORTED;
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q);
    const uintptr_t need = fmt == VKB_FMT_Q8 ? 7u : fmt == VKB_FMT_Q4 ? 3u : 1u;
    if ((qa & need) || (reinterpret_cast<uintptr_t>(s) & 1u) || (reinterpret_cast<uintptr_t>(w) & 15u))
        return VKB_EUNSUPPORTED;
    const long long chunks = (long long)N * (K / 8);
    cudaStream_t st = (cudaStream_t)stream;
    const bool bf16 = out_bf16 != 0;
    if (fmt == VKB_FMT_Q4) launch_dequant<VKB_FMT_Q4>(q, s, w, chunks, bf16, st);
    else if (fmt == VKB_FMT_Q8) launch_dequant<VKB_FMT_Q8>(q, s, w, chunks, bf16, st);
    else launch_dequant<VKB_FMT_Q2>(q, s, w, chunks, bf16, st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : -(int)e;
}
