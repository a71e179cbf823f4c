// Host-side weight formats: quantisation of fp32 weights to Q4_0 / Q8_0 / 2-bit blocks of 32, packing of integer
// codes into the bakeoff's layouts (with its sabotage mode), and the seeded synthetic inputs the benchmarks use.
//
// Packing follows the reference's host model byte for byte:
//   Q4  pack_q4            reference src/bakeoff.cu:210-219   (sabotage swaps the two nibbles of every byte)
//   Q8  raw int8 codes     reference src/bakeoff.cu:486-490   (sabotage swaps every pair of codes)
//   Q2  pack_q2_rowmajor   reference src/stage3_lut.cuh:90-97 (sabotage swaps the two codes of every pair)
// The quantiser is the rule BASELINE's configs state (absent from the reference, whose weights are random codes):
//   Q4: d = fp16(absmax / 8),   q = clamp(round(w / d) + 8, 0, 15), value = d * (q - 8)
//   Q8: d = fp16(absmax / 127), q = clamp(round(w / d), -127, 127)
//   Q2: d = fp16(absmax / 2),   q = clamp(round(w / d), -2, 1)
// round() is C's roundf (halves away from zero); an all-zero block gets d = 0 and codes 0.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>

#include "../../include/vkb_host.h"

namespace {

inline uint16_t half_bits(float v) {
    const __half h = __float2half_rn(v);
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}
inline float half_val(uint16_t b) {
    __half h;
    memcpy(&h, &b, 2);
    return __half2float(h);
}

}  // namespace

extern "C" {

int vkb_quantize(int fmt, const float* w, int N, int K, int8_t* codes, uint16_t* scales) {
    if (!w || !codes || !scales || N < 1 || K < 32 || K % 32) return VKB_HOST_EINVAL;
    const float div = fmt == VKB_FMT_Q4 ? 8.f : fmt == VKB_FMT_Q8 ? 127.f : 2.f;
    const int lo = fmt == VKB_FMT_Q4 ? -8 : fmt == VKB_FMT_Q8 ? -127 : -2;
    const int hi = fmt == VKB_FMT_Q4 ? 7 : fmt == VKB_FMT_Q8 ? 127 : 1;
    if (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8 && fmt != VKB_FMT_Q2) return VKB_HOST_EINVAL;
    const size_t G = (size_t)N * K / 32;
    for (size_t g = 0; g < G; ++g) {
        const float* b = w + 32 * g;
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(b[i]));
        const uint16_t dh = half_bits(amax / div);
        scales[g] = dh;
        const float d = half_val(dh);
        const float id = d != 0.f ? 1.f / d : 0.f;
        for (int i = 0; i < 32; ++i) {
            int q = (int)roundf(b[i] * id);
            q = std::min(hi, std::max(lo, q));
            codes[32 * g + i] = (int8_t)q;
        }
    }
    return 0;
}

int vkb_pack(int fmt, const int8_t* codes, int N, int K, int sabotage, void* out) {
    if (!codes || !out || N < 1 || K < 32 || K % 32) return VKB_HOST_EINVAL;
    const size_t n = (size_t)N * K;
    if (fmt == VKB_FMT_Q4) {
        uint32_t* o = static_cast<uint32_t*>(out);
        memset(o, 0, n / 2);
        for (size_t i = 0; i < n; i += 2) {
            uint32_t a = (uint32_t)(codes[i] + 8) & 15u, b = (uint32_t)(codes[i + 1] + 8) & 15u;
            if (sabotage) std::swap(a, b);
            o[i / 8] |= (a | (b << 4)) << (8 * ((i / 2) % 4));
        }
        return 0;
    }
    if (fmt == VKB_FMT_Q8) {
        int8_t* o = static_cast<int8_t*>(out);
        memcpy(o, codes, n);
        if (sabotage)
            for (size_t i = 0; i + 1 < n; i += 2) std::swap(o[i], o[i + 1]);
        return 0;
    }
    if (fmt == VKB_FMT_Q2) {
        if (K % 64) return VKB_HOST_EINVAL;
        uint32_t* o = static_cast<uint32_t*>(out);
        memset(o, 0, n / 4);
        for (size_t i = 0; i < n; ++i) {
            const size_t src = sabotage ? (i ^ 1) : i;
            o[i / 16] |= ((uint32_t)(codes[src] + 2) & 3u) << (2 * (i % 16));
        }
        return 0;
    }
    return VKB_HOST_EINVAL;
}

size_t vkb_packed_bytes(int fmt, int N, int K) {
    const size_t n = (size_t)N * K;
    return fmt == VKB_FMT_Q4 ? n / 2 : fmt == VKB_FMT_Q8 ? n : fmt == VKB_FMT_Q2 ? n / 4 : 0;
}

// Seeded normal draws: std::mt19937(seed), Box-Muller on pairs of 32-bit draws u = (r + 0.5) / 2^32, computed in
// double, multiplied by stddev and rounded to float. Written out here (not std::normal_distribution) so the draws do
// not depend on the C++ library.
int vkb_synth_normal(uint32_t seed, size_t n, float stddev, float* out) {
    if (!out) return VKB_HOST_EINVAL;
    std::mt19937 rng(seed);
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        const double u1 = ((double)rng() + 0.5) / 4294967296.0;
        const double u2 = ((double)rng() + 0.5) / 4294967296.0;
        const double r = std::sqrt(-2.0 * std::log(u1));
        out[i] = (float)(r * std::cos(two_pi * u2) * stddev);
        if (i + 1 < n) out[i + 1] = (float)(r * std::sin(two_pi * u2) * stddev);
    }
    return 0;
}

int vkb_f32_to_f16(const float* in, size_t n, uint16_t* out) {
    if (!in || !out) return VKB_HOST_EINVAL;
    for (size_t i = 0; i < n; ++i) out[i] = half_bits(in[i]);
    return 0;
}

// k distinct expert ids per token drawn from std::mt19937(seed): a partial Fisher-Yates shuffle of 0..E-1 per token
// using rejection-free draws rng() % (E - j). Deterministic given (seed, T, E, k).
int vkb_synth_topk(uint32_t seed, int T, int E, int k, int32_t* idx) {
    if (!idx || T < 1 || E < 1 || k < 1 || k > E) return VKB_HOST_EINVAL;
    std::mt19937 rng(seed);
    int32_t* perm = new int32_t[E];
    for (int t = 0; t < T; ++t) {
        for (int e = 0; e < E; ++e) perm[e] = e;
        for (int j = 0; j < k; ++j) {
            const int r = j + (int)(rng() % (uint32_t)(E - j));
            std::swap(perm[j], perm[r]);
            idx[(size_t)t * k + j] = perm[j];
        }
    }
    delete[] perm;
    return 0;
}

}  // extern "C"

// ---- GGUF Q4_0 / Q8_0 blocks <-> split codes + scales ---------------------------------------------------------------
// Block layouts (GGUF's published format): Q4_0 = fp16 d + 16 bytes, element j in the low nibble of byte j and element
// j + 16 in its high nibble, stored q = code + 8; Q8_0 = fp16 d + 32 int8. The split layout's Q4 word w of a row holds
// elements 8w..8w+7, element i in nibble i (stored code + 8); Q8 is one int8 per element.

extern "C" size_t vkb_gguf_bytes(int fmt, int N, int K) {
    if (N < 1 || K < 32 || K % 32) return 0;
    const size_t blocks = (size_t)N * (K / 32);
    return fmt == VKB_FMT_Q4 ? blocks * 18 : fmt == VKB_FMT_Q8 ? blocks * 34 : 0;
}

extern "C" int vkb_gguf_to_vkb(int fmt, const void* blocks, int N, int K, void* q, uint16_t* scales) {
    if (!blocks || !q || !scales || N < 1 || K < 32 || K % 32) return VKB_HOST_EINVAL;
    if (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8) return VKB_HOST_EINVAL;
    const size_t nb = (size_t)N * (K / 32);
    const uint8_t* b = static_cast<const uint8_t*>(blocks);
    const size_t bsz = fmt == VKB_FMT_Q4 ? 18 : 34;
    for (size_t i = 0; i < nb; ++i, b += bsz) {
        memcpy(&scales[i], b, 2);
        if (fmt == VKB_FMT_Q4) {
            uint8_t nib[32];
            for (int j = 0; j < 16; ++j) {
                nib[j] = b[2 + j] & 15u;
                nib[j + 16] = b[2 + j] >> 4;
            }
            uint8_t* o = static_cast<uint8_t*>(q) + i * 16;   // 32 codes, two per byte, even element low
            for (int j = 0; j < 16; ++j) o[j] = (uint8_t)(nib[2 * j] | (nib[2 * j + 1] << 4));
        } else {
            memcpy(static_cast<int8_t*>(q) + i * 32, b + 2, 32);
        }
    }
    return 0;
}

extern "C" int vkb_vkb_to_gguf(int fmt, const void* q, const uint16_t* scales, int N, int K, void* blocks) {
    if (!blocks || !q || !scales || N < 1 || K < 32 || K % 32) return VKB_HOST_EINVAL;
    if (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8) return VKB_HOST_EINVAL;
    const size_t nb = (size_t)N * (K / 32);
    uint8_t* b = static_cast<uint8_t*>(blocks);
    const size_t bsz = fmt == VKB_FMT_Q4 ? 18 : 34;
    for (size_t i = 0; i < nb; ++i, b += bsz) {
        memcpy(b, &scales[i], 2);
        if (fmt == VKB_FMT_Q4) {
            const uint8_t* in = static_cast<const uint8_t*>(q) + i * 16;
            uint8_t nib[32];
            for (int j = 0; j < 16; ++j) {
                nib[2 * j] = in[j] & 15u;
                nib[2 * j + 1] = in[j] >> 4;
            }
            for (int j = 0; j < 16; ++j) b[2 + j] = (uint8_t)(nib[j] | (nib[j + 16] << 4));
        } else {
            memcpy(b + 2, static_cast<const int8_t*>(q) + i * 32, 32);
        }
    }
    return 0;
}
