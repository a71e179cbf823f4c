/*
 * vkb_host.h -- host-side helpers of libvkb.so: weight quantisation and packing into the bakeoff's formats, and the
 * seeded synthetic inputs of the benchmarks. Pure CPU functions (no CUDA calls); return 0 on success.
 *
 * These replace the reference harness's host weight model: make_weights / pack_q4 (reference src/bakeoff.cu:195-219),
 * the raw Q8 copy with its pair-swap sabotage (:486-490), and pack_q2_rowmajor (src/stage3_lut.cuh:90-97). The
 * quantiser is the Q4_0 / Q8_0 / 2-bit rule of the benchmark configuration (block of 32, one fp16 scale).
 */
#ifndef VKB_HOST_H
#define VKB_HOST_H

#include <stddef.h>
#include <stdint.h>

#include "vkb.h"

#ifdef __cplusplus
extern "C" {
#endif

#define VKB_HOST_EINVAL 2

/* fp32 w[N][K] -> integer codes[N][K] (-8..7, -127..127 or -2..1) and fp16 scales[N][K/32] (as raw uint16 bits). */
int vkb_quantize(int fmt, const float* w, int N, int K, int8_t* codes, uint16_t* scales);
/* codes[N][K] -> the packed layout of vkb.h (Q4 uint32 [N][K/8], Q8 int8 [N][K], Q2 uint32 [N][K/16]).
 * sabotage != 0 breaks the packing the way the reference's BAKEOFF_SABOTAGE does, so every check must fail. */
int vkb_pack(int fmt, const int8_t* codes, int N, int K, int sabotage, void* out);
/* Bytes of packed codes for an N x K matrix. */
size_t vkb_packed_bytes(int fmt, int N, int K);
/* n normal draws N(0, stddev^2) from std::mt19937(seed) with Box-Muller written out (library-independent). */
int vkb_synth_normal(uint32_t seed, size_t n, float stddev, float* out);
/* fp32 -> fp16 bits, round to nearest even. */
int vkb_f32_to_f16(const float* in, size_t n, uint16_t* out);
/* T tokens x k distinct expert ids in [0, E) from std::mt19937(seed) (partial Fisher-Yates). */
int vkb_synth_topk(uint32_t seed, int T, int E, int k, int32_t* idx);

/* ---- GGUF interop (Q4_0 / Q8_0) -------------------------------------------------------------------------------------
 * The reference stores its own layout but states value parity with GGUF's Q4_0 / Q8_0 (reference src/bakeoff.cu:5-7):
 * one fp16 scale d per 32 consecutive values of a row, value = (q - 8) d (Q4_0) or q d (Q8_0). GGUF stores each
 * block of 32 together, in row order, K / 32 blocks per row:
 *   Q4_0  18 bytes: fp16 d, then 16 bytes qs; element j of the block in the low nibble of qs[j], element j + 16 in
 *         the high nibble (j = 0..15), stored q = code + 8
 *   Q8_0  34 bytes: fp16 d, then 32 int8 q
 * These convert blocks [N][K/32] to this library's split layout (packed codes as vkb_pack writes them, scales
 * [N][K/32]) and back, bit-exactly: the values, the scales and the codes are unchanged. K % 32 == 0. Q2 has no GGUF
 * counterpart here (VKB_HOST_EINVAL). vkb_gguf_to_vkb_device (libvkb.so, vkb.h) does the GGUF -> split direction on
 * the GPU for weights already in device memory. */
size_t vkb_gguf_bytes(int fmt, int N, int K);
int vkb_gguf_to_vkb(int fmt, const void* blocks, int N, int K, void* q, uint16_t* scales);
int vkb_vkb_to_gguf(int fmt, const void* q, const uint16_t* scales, int N, int K, void* blocks);

#ifdef __cplusplus
}
#endif

#endif /* VKB_HOST_H */
