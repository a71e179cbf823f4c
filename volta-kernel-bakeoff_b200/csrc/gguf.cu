// GGUF Q4_0 / Q8_0 blocks -> the split layout of vkb.h, on the GPU (weights uploaded as GGUF blocks are repacked once,
// in device memory). The host functions vkb_gguf_to_vkb / vkb_vkb_to_gguf (formats.cpp) state the same conversion.
//
//   Q4_0 block (18 B): fp16 d, 16 bytes qs: element j in the low nibble of qs[j], element j + 16 in the high nibble
//   Q8_0 block (34 B): fp16 d, 32 int8
//   split Q4: 16 bytes per block, element 2j in the low nibble of byte j, 2j + 1 in the high one; Q8: the 32 int8 as
//   they are; scales: one fp16 per block, row-major [N][K/32] -- the block order.
//
// One thread per block: a warp covers 32 consecutive blocks (576 / 1088 contiguous bytes), read as 16-bit words
// (GGUF blocks are only 2-byte aligned), and writes 16- or 32-byte aligned code vectors. Memory-bound, run once.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vkb.h"
#include "vkb_internal.h"

namespace vkb {

__global__ void __launch_bounds__(256) gguf_q4_0_kernel(const uint16_t* __restrict__ blocks, uint4* __restrict__ q,
                                                        uint16_t* __restrict__ s, long long nb) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nb; i += (long long)gridDim.x * blockDim.x) {
        const uint16_t* b = blocks + i * 9;   // 18 bytes
        s[i] = b[0];
        uint32_t qs[4];                      // the 16 bytes of qs as 4 little-endian words
#pragma unroll
        for (int w = 0; w < 4; ++w) qs[w] = (uint32_t)b[1 + 2 * w] | ((uint32_t)b[2 + 2 * w] << 16);
        // byte j of qs: lo = element j, hi = element j + 16. Output byte j: element 2j (lo) | element 2j + 1 (hi).
        uint32_t o[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int e0 = 2 * j, e1 = 2 * j + 1;   // elements of output byte j
            const uint32_t n0 = e0 < 16 ? (qs[e0 >> 2] >> (8 * (e0 & 3))) & 15u : (qs[(e0 - 16) >> 2] >> (8 * ((e0 - 16) & 3) + 4)) & 15u;
            const uint32_t n1 = e1 < 16 ? (qs[e1 >> 2] >> (8 * (e1 & 3))) & 15u : (qs[(e1 - 16) >> 2] >> (8 * ((e1 - 16) & 3) + 4)) & 15u;
            o[j >> 2] |= (n0 | (n1 << 4)) << (8 * (j & 3));
        }
        q[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void __launch_bounds__(256) gguf_q8_0_kernel(const uint16_t* __restrict__ blocks, uint4* __restrict__ q,
                                                        uint16_t* __restrict__ s, long long nb) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nb; i += (long long)gridDim.x * blockDim.x) {
        const uint16_t* b = blocks + i * 17;   // 34 bytes
        s[i] = b[0];
        uint32_t w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = (uint32_t)b[1 + 2 * k] | ((uint32_t)b[2 + 2 * k] << 16);
        q[2 * i] = make_uint4(w[0], w[1], w[2], w[3]);
        q[2 * i + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

}  // namespace vkb

using namespace vkb;

extern "C" int vkb_gguf_to_vkb_device(int fmt, const void* blocks, int N, int K, void* q, void* scales,
                                      vkb_stream_t stream) {
    if (!blocks || !q || !scales || N < 1 || K < 32) return VKB_EINVAL;
    if (K % 32 != 0 || (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8)) return VKB_EUNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(blocks) | reinterpret_cast<uintptr_t>(scales)) & 1u) return VKB_EUNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(q) & 15u) return VKB_EUNSUPPORTED;
    const long long nb = (long long)N * (K / 32);
    const int threads = 256;
    const long long want = (nb + threads - 1) / threads;
    const int grid = (int)(want < 8192 ? want : 8192);
    cudaStream_t st = (cudaStream_t)stream;
    if (fmt == VKB_FMT_Q4)
        gguf_q4_0_kernel<<<grid, threads, 0, st>>>((const uint16_t*)blocks, (uint4*)q, (uint16_t*)scales, nb);
    else
        gguf_q8_0_kernel<<<grid, threads, 0, st>>>((const uint16_t*)blocks, (uint4*)q, (uint16_t*)scales, nb);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : -(int)e;
}
