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

#ifdef __cplusplus
}
#endif

#endif /* VKB_HOST_H */
