// bakeoff -- the contender harness of the quantised matmul path, on libvkb.so (B200, sm_100a).
//
//   bakeoff            sweep: one CSV row per (contender, table, token count):
//                      contender,shape,N,K,M,us,weight_GBps,tflops,copies
//   bakeoff --check    every contender against a CPU double-precision reference of the same quantised weights:
//                      check,contender,shape,M,max_err_rel,worst_m,worst_n,verdict   (exit 1 on any FAIL)
//
// Environment (the reference harness's switches, src/bakeoff.cu:656-657, :845):
//   BAKEOFF_SABOTAGE=1   --check packs every weight matrix wrongly: every packed-weight contender must FAIL, the
//                        cuBLAS controls (which get unpacked fp16/bf16 weights) must stay ok
//   BAKEOFF_SHAPE=name   sweep one weight table only (the MoE part is skipped), for a profiler
//   BAKEOFF_M=m          sweep one token count only
//   BAKEOFF_CONTENDER=c  sweep the contenders whose name starts with c only (and allocate only their weights)
//
// Contenders: vkb_q4 / vkb_q8 / vkb_q2 (decode GEMV, 1-8 tokens), vkb_q4_f32in (the same with fp32 activations),
// vkb_glu_q4_f32in (gate + up + SwiGLU, fp32 activations), vkb_tc_q4 / vkb_tc_q8 (prompt GEMM on tcgen05, Q4 or Q8
// weights, any token count),
// vkb_moe_q4 (MoE, one launch over a device index list), and the controls cublas_fp16 (the reference's
// cublasGemmEx fp16 x fp16 -> fp32, src/bakeoff.cu:249-253), cublas_bf16 (bf16 x bf16 -> bf16) and dq4+cublas (the
// packed Q4 weights dequantised on the GPU by vkb_dequant, then cublas_fp16: the reference's row, src/bakeoff.cu:687-690). Timing follows the
// reference's time_us (src/bakeoff.cu:283-298: 20 warm-up calls, the median of 5 repetitions of 50 calls), with the 50
// calls captured in a CUDA graph on a created stream so that host launch cost is not measured, and the weights
// cycled over copies that span at least 4x the L2 (every call reads HBM).
//
// Error yardstick (src/bakeoff.cu:221-235, :566-579): |y - ref| / sum_k |x_k w_k|, sampled on 256 outputs plus the
// first and last row of every token. Tolerances: 1e-4 for the exact-code kernels with fp32 output, 2e-3 for the fp16
// class (tensor-core prompt GEMM, cuBLAS fp16), 8e-3 for cuBLAS bf16 (weights rounded to 8 mantissa bits); the fp16
// output variants are checked with the benchmark's own bound |y - ref| <= 1e-2 + 1e-3 |ref| as well.
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "vkb.h"
#include "vkb_host.h"

#define CK(x)                                                                                                   \
    do {                                                                                                        \
        cudaError_t e_ = (x);                                                                                   \
        if (e_ != cudaSuccess) {                                                                                \
            fprintf(stderr, "CUDA error %s at %s:%d: %s\n", cudaGetErrorString(e_), __FILE__, __LINE__, #x);    \
            exit(2);                                                                                            \
        }                                                                                                       \
    } while (0)
#define CB(x)                                                                                                   \
    do {                                                                                                        \
        cublasStatus_t s_ = (x);                                                                                \
        if (s_ != CUBLAS_STATUS_SUCCESS) {                                                                      \
            fprintf(stderr, "cuBLAS error %d at %s:%d: %s\n", (int)s_, __FILE__, __LINE__, #x);                \
            exit(2);                                                                                            \
        }                                                                                                       \
    } while (0)

// A library call: < 0 is a CUDA error (fatal, as the reference's CK), > 0 means "unsupported, nothing launched".
static bool VK(int rc, const char* what) {
    if (rc < 0) {
        fprintf(stderr, "%s: %s\n", what, vkb_strerror(rc));
        exit(2);
    }
    return rc == 0;
}

static cudaStream_t g_st;
static cublasHandle_t g_hb;

// ---- host weights -------------------------------------------------------------------------------------------------

struct Weights {          // one quantised matrix, kept on the host for the reference
    int fmt, N, K;
    std::vector<int8_t> code;      // [N][K]
    std::vector<uint16_t> scale;   // fp16 bits [N][K/32]
};

static uint16_t f16(float v) { return __half_as_ushort(__float2half_rn(v)); }
static float f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// Codes uniform over the format's range, scales uniform (the reference's make_weights / make_q2 value model,
// src/bakeoff.cu:202-210, src/stage2.cuh:237-243).
static Weights make_weights(int fmt, int N, int K, std::mt19937& rng) {
    Weights w{fmt, N, K, std::vector<int8_t>((size_t)N * K), std::vector<uint16_t>((size_t)N * K / 32)};
    const int lo = fmt == VKB_FMT_Q4 ? -8 : fmt == VKB_FMT_Q8 ? -127 : -2;
    const int span = fmt == VKB_FMT_Q4 ? 16 : fmt == VKB_FMT_Q8 ? 255 : 4;
    for (auto& c : w.code) c = (int8_t)(lo + (int)(rng() % (uint32_t)span));
    const float s0 = fmt == VKB_FMT_Q2 ? 0.01f : 0.004f, s1 = fmt == VKB_FMT_Q2 ? 0.04f : 0.02f;
    const float mul = fmt == VKB_FMT_Q8 ? 0.06f : 1.f;
    for (auto& s : w.scale) s = f16((s0 + (s1 - s0) * (float)(rng() >> 8) * (1.f / 16777216.f)) * mul);
    return w;
}

static std::vector<uint8_t> packed(const Weights& w, bool sabotage) {
    std::vector<uint8_t> p(vkb_packed_bytes(w.fmt, w.N, w.K));
    if (vkb_pack(w.fmt, w.code.data(), w.N, w.K, sabotage ? 1 : 0, p.data()) != 0) {
        fprintf(stderr, "vkb_pack failed\n");
        exit(2);
    }
    return p;
}

// fp16 (or bf16) copy of the weights, one rounding of code * scale: the cuBLAS controls' input.
static std::vector<uint16_t> dequant(const Weights& w, bool bf16) {
    std::vector<uint16_t> o((size_t)w.N * w.K);
    for (size_t i = 0; i < o.size(); ++i) {
        const float v = (float)w.code[i] * f32(w.scale[i / 32]);
        o[i] = bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : f16(v);
    }
    return o;
}

// sum_k x w and sum_k |x w| in double (the reference's ref_value / ref_scale, src/bakeoff.cu:221-235)
static double ref_dot(const Weights& w, const uint16_t* x, int n, double* mag) {
    double a = 0, m = 0;
    const int8_t* c = w.code.data() + (size_t)n * w.K;
    const uint16_t* s = w.scale.data() + (size_t)n * (w.K / 32);
    for (int k = 0; k < w.K; ++k) {
        const double t = (double)f32(x[k]) * (double)c[k] * (double)f32(s[k / 32]);
        a += t;
        m += std::fabs(t);
    }
    *mag = m;
    return a;
}

template <typename T> static T* dalloc(size_t n) {
    T* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    return p;
}
template <typename T> static T* dupload(const std::vector<T>& v) {
    T* p = dalloc<T>(v.size());
    CK(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
    return p;
}

static size_t g_l2 = 0;
// copies of a buffer set so that cycling them streams at least 4x the L2 from HBM
static int copies_for(size_t bytes) { return (int)std::max<size_t>(2, 4 * g_l2 / std::max<size_t>(bytes, 1) + 1); }

// ---- cuBLAS controls ------------------------------------------------------------------------------------------------

// y[M][N] = x[M][K] . W[N][K]^T, W row-major: C (N x M, column-major) = op_T(W as K x N) * X (K x M)
static void cublas_f16(const void* w, const void* x, float* y, int N, int K, int M) {
    const float one = 1.f, zero = 0.f;
    CB(cublasGemmEx(g_hb, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &one, w, CUDA_R_16F, K, x, CUDA_R_16F, K, &zero, y,
                    CUDA_R_32F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT_TENSOR_OP));
}
static void cublas_bf16(const void* w, const void* x, void* y, int N, int K, int M) {
    const float one = 1.f, zero = 0.f;
    CB(cublasGemmEx(g_hb, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &one, w, CUDA_R_16BF, K, x, CUDA_R_16BF, K, &zero, y,
                    CUDA_R_16BF, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT_TENSOR_OP));
}

// ---- timing ---------------------------------------------------------------------------------------------------------

// Median microseconds per call of fn(i): 20 warm-up calls, then 5 repetitions of a captured graph of 50 calls,
// i counting on so that the caller cycles its weight copies. Returns < 0 if fn reported "unsupported".
static double time_us(const std::function<bool(int)>& fn) {
    int i = 0;
    for (; i < 20; ++i)
        if (!fn(i)) return -1;
    CK(cudaStreamSynchronize(g_st));
    cudaGraph_t g;
    cudaGraphExec_t ge;
    CK(cudaStreamBeginCapture(g_st, cudaStreamCaptureModeThreadLocal));
    bool ok = true;
    for (int k = 0; k < 50; ++k, ++i) ok &= fn(i);
    CK(cudaStreamEndCapture(g_st, &g));
    if (!ok) {
        CK(cudaGraphDestroy(g));
        return -1;
    }
    CK(cudaGraphInstantiate(&ge, g, 0));
    CK(cudaGraphLaunch(ge, g_st));   // warm the graph
    cudaEvent_t a, b;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b));
    std::vector<double> t;
    for (int rep = 0; rep < 5; ++rep) {
        CK(cudaEventRecord(a, g_st));
        CK(cudaGraphLaunch(ge, g_st));
        CK(cudaEventRecord(b, g_st));
        CK(cudaEventSynchronize(b));
        float ms = 0;
        CK(cudaEventElapsedTime(&ms, a, b));
        t.push_back(ms * 1000.0 / 50);
    }
    CK(cudaEventDestroy(a));
    CK(cudaEventDestroy(b));
    CK(cudaGraphExecDestroy(ge));
    CK(cudaGraphDestroy(g));
    std::sort(t.begin(), t.end());
    return t[2];
}

struct Shape { const char* name; int N, K; };
// The reference's weight tables (src/bakeoff.cu:300-311): names and sizes are the benchmark's vocabulary.
static const Shape SHAPES[] = {
    {"flashnext_expert_gate_up", 640, 2560}, {"flashnext_expert_down", 2560, 640}, {"flashnext_attn_q", 12288, 2560},
    {"flashnext_attn_out", 2560, 6144},      {"qwen36_expert_gate_up", 512, 2048}, {"qwen36_expert_down", 2048, 512},
    {"qwen36_attn_qkv", 8192, 2048},         {"qwen3_1p7b_mlp_up", 6144, 2048},   {"qwen3_1p7b_mlp_down", 2048, 6144},
};
static const int MS[] = {1, 2, 4, 8, 16, 32, 64, 128, 256, 512};

static int gemv_f32(int fmt, const void* q, const void* s, const void* x, float* y, int N, int K, int M) {
    return vkb_gemv(fmt, q, s, x, y, 1, N, K, M, (vkb_stream_t)g_st);
}
static int gemv_f16(int fmt, const void* q, const void* s, const void* x, void* y, int N, int K, int M) {
    return vkb_gemv(fmt, q, s, x, y, 0, N, K, M, (vkb_stream_t)g_st);
}

// ---- the sweep ------------------------------------------------------------------------------------------------------

static void run_sweep() {
    std::mt19937 rng(42);
    printf("contender,shape,N,K,M,us,weight_GBps,tflops,copies\n");
    const char* only = getenv("BAKEOFF_SHAPE");
    const int only_m = getenv("BAKEOFF_M") ? atoi(getenv("BAKEOFF_M")) : 0;
    const char* only_c = getenv("BAKEOFF_CONTENDER");
    auto want = [&](const char* who) { return !only_c || !strncmp(who, only_c, strlen(only_c)); };
    const bool any_gemv = !only_m || only_m <= 8;
    static const char* gname[] = {"vkb_q4", "vkb_q8", "vkb_q2"};
    for (const Shape& sh : SHAPES) {
        if (only && strcmp(sh.name, only)) continue;
        const size_t NK = (size_t)sh.N * sh.K;
        struct Set { int fmt; size_t bytes; int c; std::vector<void*> q, s; };
        std::vector<Set> sets;
        for (int fmt : {VKB_FMT_Q4, VKB_FMT_Q8, VKB_FMT_Q2}) {
            const Weights w = make_weights(fmt, sh.N, sh.K, rng);
            const auto p = packed(w, false);
            Set st{fmt, p.size() + w.scale.size() * 2, 0, {}, {}};
            if ((any_gemv && want(gname[fmt])) ||
                (fmt == VKB_FMT_Q4 && (want("vkb_tc_q4") || want("dq4+cublas") || (any_gemv && want("vkb_q4_f32in")))) ||
                (fmt == VKB_FMT_Q8 && want("vkb_tc_q8")))
                st.c = copies_for(st.bytes);
            for (int i = 0; i < st.c; ++i) {
                st.q.push_back(dupload(p));
                st.s.push_back(dupload(w.scale));
            }
            sets.push_back(std::move(st));
        }
        const Weights w4 = make_weights(VKB_FMT_Q4, sh.N, sh.K, rng);
        const int cf = (want("cublas_fp16") || want("cublas_bf16")) ? copies_for(NK * 2) : 0;
        std::vector<void*> df, db;
        if (cf) {
            const auto wf = dequant(w4, false), wb = dequant(w4, true);
            for (int i = 0; i < cf; ++i) {
                df.push_back(dupload(wf));
                db.push_back(dupload(wb));
            }
        }
        for (int M : MS) {
            if (only_m && M != only_m) continue;
            const uint16_t hx = f16(0.5f), hb = __bfloat16_as_ushort(__float2bfloat16_rn(0.5f));
            void* dx = dupload(std::vector<uint16_t>((size_t)M * sh.K, hx));
            void* dxb = dupload(std::vector<uint16_t>((size_t)M * sh.K, hb));
            float* dy = dalloc<float>((size_t)M * sh.N);
            void* dyh = dalloc<uint16_t>((size_t)M * sh.N);
            const double flop = 2.0 * M * NK;
            auto report = [&](const char* who, double us, size_t wbytes, int copies) {
                if (us < 0) return;   // unsupported here
                printf("%s,%s,%d,%d,%d,%.2f,%.1f,%.3f,%d\n", who, sh.name, sh.N, sh.K, M, us, wbytes / us / 1e3,
                       flop / us / 1e6, copies);
                fflush(stdout);
            };
            if (want("cublas_fp16"))
                report("cublas_fp16", time_us([&](int i) { cublas_f16(df[i % cf], dx, dy, sh.N, sh.K, M); return true; }),
                       NK * 2, cf);
            if (want("cublas_bf16"))
                report("cublas_bf16", time_us([&](int i) { cublas_bf16(db[i % cf], dxb, dyh, sh.N, sh.K, M); return true; }),
                       NK * 2, cf);
            if (want("dq4+cublas") && sets[0].c > 0) {   // the reference's control: dequantise, then a cuBLAS fp16 GEMM
                const Set& s4d = sets[0];
                void* wtmp = dalloc<uint16_t>(NK);
                report("dq4+cublas", time_us([&](int i) {
                           if (!VK(vkb_dequant(VKB_FMT_Q4, s4d.q[i % s4d.c], s4d.s[i % s4d.c], wtmp, sh.N, sh.K, 0,
                                               (vkb_stream_t)g_st), "vkb_dequant"))
                               return false;
                           cublas_f16(wtmp, dx, dy, sh.N, sh.K, M);
                           return true;
                       }), s4d.bytes, s4d.c);
                CK(cudaFree(wtmp));
            }
            const Set& s4 = sets[0];
            if (want("vkb_tc_q4"))
                report("vkb_tc_q4", time_us([&](int i) {
                           return VK(vkb_gemm_q4_tc(s4.q[i % s4.c], s4.s[i % s4.c], dx, dyh, sh.N, sh.K, M,
                                                    (vkb_stream_t)g_st), "vkb_gemm_q4_tc");
                       }), s4.bytes, s4.c);
            const Set& s8 = sets[1];
            if (want("vkb_tc_q8"))
                report("vkb_tc_q8", time_us([&](int i) {
                           return VK(vkb_gemm_q8_tc(s8.q[i % s8.c], s8.s[i % s8.c], dx, dyh, sh.N, sh.K, M,
                                                    (vkb_stream_t)g_st), "vkb_gemm_q8_tc");
                       }), s8.bytes, s8.c);
            if (M <= 8)
                for (const Set& st : sets)
                    if (want(gname[st.fmt]))
                        report(gname[st.fmt], time_us([&](int i) {
                                   return VK(gemv_f16(st.fmt, st.q[i % st.c], st.s[i % st.c], dx, dyh, sh.N, sh.K, M),
                                             "vkb_gemv");
                               }), st.bytes, st.c);
            if (M <= 8 && want("vkb_q4_f32in")) {   // fp32 activations in (the reference's fused_q4_v3_fp32in row)
                float* dxf = dupload(std::vector<float>((size_t)M * sh.K, 0.5f));
                report("vkb_q4_f32in", time_us([&](int i) {
                           return VK(vkb_gemv_q4_f32in(s4.q[i % s4.c], s4.s[i % s4.c], dxf, dxb, dy, sh.N, sh.K, M,
                                                       (vkb_stream_t)g_st), "vkb_gemv_q4_f32in");
                       }), s4.bytes, s4.c);
                CK(cudaFree(dxf));
            }
            CK(cudaFree(dx));
            CK(cudaFree(dxb));
            CK(cudaFree(dy));
            CK(cudaFree(dyh));
        }
        for (auto& st : sets)
            for (int i = 0; i < st.c; ++i) {
                CK(cudaFree(st.q[i]));
                CK(cudaFree(st.s[i]));
            }
        for (int i = 0; i < cf; ++i) {
            CK(cudaFree(df[i]));
            CK(cudaFree(db[i]));
        }
    }
    // gate + up + SwiGLU on Qwen3-1.7B's MLP (gate and up 6144x2048 stacked), fp32 activations in, one call per
    // step (the reference's gate_up_glu_fp32in row, src/bakeoff.cu:767-786); bytes: the stacked table
    if ((!only || !strcmp(only, "qwen3_1p7b_mlp_gate_up")) && want("vkb_glu_q4_f32in")) {
        const int N = 6144, K = 2048;
        const Weights w = make_weights(VKB_FMT_Q4, 2 * N, K, rng);
        const auto p = packed(w, false);
        const size_t qb = p.size() + w.scale.size() * 2;
        const int c = copies_for(qb);
        std::vector<void*> q(c), sc(c);
        for (int i = 0; i < c; ++i) {
            q[i] = dupload(p);
            sc[i] = dupload(w.scale);
        }
        for (int M : {1, 2, 4, 8}) {
            if (only_m && M != only_m) continue;
            float* dxf = dupload(std::vector<float>((size_t)M * K, 0.5f));
            void* dxh = dalloc<uint16_t>((size_t)M * K);
            float* dys = dalloc<float>((size_t)M * 2 * N);
            float* dout = dalloc<float>((size_t)M * N);
            const double us = time_us([&](int i) {
                return VK(vkb_gate_up_glu_q4_f32in(q[i % c], sc[i % c], dxf, dxh, dys, dout, N, K, M,
                                                   (vkb_stream_t)g_st), "vkb_gate_up_glu_q4_f32in");
            });
            printf("vkb_glu_q4_f32in,qwen3_1p7b_mlp_gate_up,%d,%d,%d,%.2f,%.1f,%.3f,%d\n", 2 * N, K, M, us, qb / us / 1e3,
                   2.0 * M * 2 * N * K / us / 1e6, c);
            fflush(stdout);
            CK(cudaFree(dxf));
            CK(cudaFree(dxh));
            CK(cudaFree(dys));
            CK(cudaFree(dout));
        }
        for (int i = 0; i < c; ++i) {
            CK(cudaFree(q[i]));
            CK(cudaFree(sc[i]));
        }
    }
    if (only || !want("vkb_moe_q4")) return;
    // MoE decode: a pool of experts, k distinct experts per token, one launch (the benchmark's MoE configurations)
    struct MoeCase { const char* name; int E, topk, N, K; };
    static const MoeCase MOE[] = {{"qwen36_expert_gate_up", 128, 8, 512, 2048}, {"qwen36_expert_down", 128, 8, 2048, 512},
                                  {"flashnext_expert_gate_up", 160, 10, 640, 2560},
                                  {"flashnext_expert_down", 160, 10, 2560, 640}};
    for (const MoeCase& mc : MOE) {
        const Weights w = make_weights(VKB_FMT_Q4, mc.N * mc.E, mc.K, rng);   // E experts stacked
        const auto p = packed(w, false);
        const size_t pool = p.size() + w.scale.size() * 2, per = pool / mc.E;
        const int c = copies_for(pool);
        std::vector<void*> q, s;
        for (int i = 0; i < c; ++i) {
            q.push_back(dupload(p));
            s.push_back(dupload(w.scale));
        }
        for (int T : {1, 8, 64}) {
            if (only_m && T != only_m) continue;
            std::vector<int32_t> idx((size_t)T * mc.topk);
            vkb_synth_topk(7, T, mc.E, mc.topk, idx.data());
            std::vector<bool> used(mc.E, false);
            for (int e : idx) used[e] = true;
            const size_t touched = (size_t)std::count(used.begin(), used.end(), true) * per;
            int32_t* didx = dupload(idx);
            void* dx = dupload(std::vector<uint16_t>((size_t)T * mc.K, f16(0.5f)));
            void* dy = dalloc<uint16_t>((size_t)T * mc.topk * mc.N);
            const double us = time_us([&](int i) {
                return VK(vkb_moe(VKB_FMT_Q4, q[i % c], s[i % c], didx, T, mc.topk, dx, dy, 0, mc.E, 0, mc.N, mc.K,
                                  (vkb_stream_t)g_st), "vkb_moe");
            });
            if (us >= 0)
                printf("vkb_moe_q4,%s_pool%d_top%d,%d,%d,%d,%.2f,%.1f,%.3f,%d\n", mc.name, mc.E, mc.topk, mc.N, mc.K, T,
                       us, touched / us / 1e3, 2.0 * T * mc.topk * mc.N * mc.K / us / 1e6, c);
            fflush(stdout);
            CK(cudaFree(didx));
            CK(cudaFree(dx));
            CK(cudaFree(dy));
        }
        for (int i = 0; i < c; ++i) {
            CK(cudaFree(q[i]));
            CK(cudaFree(s[i]));
        }
    }
}

// ---- correctness ----------------------------------------------------------------------------------------------------

static int g_failures = 0;

struct Worst { double err = 0, abs_excess = 0; int m = 0, n = 0; };

// Sampled error of y (fp32 or fp16 [M][N]) against the reference: 256 random outputs plus the first and last row of
// every token. f16_bound also applies |y - ref| <= 1e-2 + 1e-3 |ref|.
static Worst sample_err(const Weights& w, const std::vector<uint16_t>& x, const void* y_host, bool y_f16, int M,
                        std::mt19937& rng, bool* f16_ok) {
    Worst r;
    *f16_ok = true;
    for (int t = 0; t < 256 + 2 * M; ++t) {
        int m, n;
        if (t < 2 * M) {
            m = t / 2;
            n = (t & 1) ? w.N - 1 : 0;
        } else {
            m = (int)(rng() % (uint32_t)M);
            n = (int)(rng() % (uint32_t)w.N);
        }
        double mag;
        const double ref = ref_dot(w, x.data() + (size_t)m * w.K, n, &mag);
        const double got = y_f16 ? (double)f32(((const uint16_t*)y_host)[(size_t)m * w.N + n])
                                 : (double)((const float*)y_host)[(size_t)m * w.N + n];
        const double err = std::fabs(got - ref) / (mag + 1e-12);
        if (err > r.err) { r.err = err; r.m = m; r.n = n; }
        if (std::fabs(got - ref) > 1e-2 + 1e-3 * std::fabs(ref)) *f16_ok = false;
    }
    return r;
}

static void verdict(const std::string& who, const std::string& label, int M, const Worst& r, bool ok) {
    g_failures += !ok;
    printf("check,%s,%s,%d,%.3g,%d,%d,%s\n", who.c_str(), label.c_str(), M, r.err, r.m, r.n, ok ? "ok" : "FAIL");
    fflush(stdout);
}

// One contender call writing y[M][N] (fp32 when f32) -- returns false when unsupported (nothing launched).
using Call = std::function<bool(void* y)>;

static void check_one(const std::string& who, const std::string& label, const Weights& w,
                      const std::vector<uint16_t>& x, int M, bool f32out, double tol, const Call& call,
                      std::mt19937& rng) {
    const size_t n = (size_t)M * w.N, bytes = n * (f32out ? 4 : 2);
    void* dy = dalloc<uint8_t>(bytes);
    CK(cudaMemsetAsync(dy, 0, bytes, g_st));
    if (!call(dy)) {
        CK(cudaFree(dy));
        return;
    }
    CK(cudaStreamSynchronize(g_st));
    std::vector<uint8_t> y(bytes);
    CK(cudaMemcpy(y.data(), dy, bytes, cudaMemcpyDeviceToHost));
    CK(cudaFree(dy));
    bool f16_ok;
    const Worst r = sample_err(w, x, y.data(), !f32out, M, rng, &f16_ok);
    verdict(who, label, M, r, r.err <= tol && (f32out || f16_ok));
}

static std::vector<uint16_t> make_x(int M, int K, int kind, std::mt19937& rng) {
    // kind 0: x in [-1, 1]; 1 ("bigx"): plus 64 neighbouring channels at +-20000..60000 (fits fp16, overflows short
    // fp16 sums); 2 ("tinyx"): x in [-1e-3, 1e-3] (src/bakeoff.cu:493-512)
    std::vector<uint16_t> x((size_t)M * K);
    auto u = [&]() { return (float)(rng() >> 8) * (1.f / 16777216.f); };
    for (auto& v : x) v = f16((2.f * u() - 1.f) * (kind == 2 ? 1e-3f : 1.f));
    if (kind == 1) {
        const int k0 = K / 3 / 64 * 64;
        for (int m = 0; m < M; ++m)
            for (int k = k0; k < std::min(K, k0 + 64); ++k)
                x[(size_t)m * K + k] = f16(((rng() & 1) ? 1.f : -1.f) * (20000.f + 40000.f * u()));
    }
    return x;
}

static void check_tables(bool sabotage, std::mt19937& rng) {
    for (const Shape& sh : SHAPES) {
        for (int fmt : {VKB_FMT_Q4, VKB_FMT_Q8, VKB_FMT_Q2}) {
            const Weights w = make_weights(fmt, sh.N, sh.K, rng);
            void* dq = dupload(packed(w, sabotage));
            void* ds = dupload(w.scale);
            void* dwf = fmt == VKB_FMT_Q4 ? dupload(dequant(w, false)) : nullptr;
            void* dwq = fmt == VKB_FMT_Q4 ? dalloc<uint16_t>((size_t)sh.N * sh.K) : nullptr;   // vkb_dequant's output
            struct XCase { int M, kind; };
            std::vector<XCase> xcases;
            for (int M : {1, 2, 4, 8}) xcases.push_back({M, 0});
            if (fmt != VKB_FMT_Q2)   // prompt GEMM: Q4 and Q8 weights
                for (int M : {64, 65, 128, 256, 512}) xcases.push_back({M, 0});
            for (int M : {1, 2, 4, 8}) {
                xcases.push_back({M, 1});
                xcases.push_back({M, 2});
            }
            static const char* gname[] = {"vkb_q4", "vkb_q8", "vkb_q2"};
            for (const XCase& xc : xcases) {
                const int M = xc.M;
                const std::string label =
                    std::string(sh.name) + (xc.kind == 1 ? "+bigx" : xc.kind == 2 ? "+tinyx" : "");
                const auto x = make_x(M, sh.K, xc.kind, rng);
                void* dx = dupload(x);
                if (M <= 8) {
                    check_one(gname[fmt], label, w, x, M, true, 1e-4, [&](void* y) {
                        return VK(gemv_f32(fmt, dq, ds, dx, (float*)y, sh.N, sh.K, M), "vkb_gemv");
                    }, rng);
                    if (xc.kind != 1)   // bigx sums exceed the fp16 range: fp32 output only
                        check_one(std::string(gname[fmt]) + "_f16out", label, w, x, M, false, 1e-3, [&](void* y) {
                            return VK(gemv_f16(fmt, dq, ds, dx, y, sh.N, sh.K, M), "vkb_gemv");
                        }, rng);
                }
                if (fmt == VKB_FMT_Q4) {
                    check_one("vkb_tc_q4", label, w, x, M, true, 2e-3, [&](void* y) {
                        return VK(vkb_gemm_q4_tc_f32(dq, ds, dx, (float*)y, sh.N, sh.K, M, (vkb_stream_t)g_st),
                                  "vkb_gemm_q4_tc");
                    }, rng);
                    if (xc.kind != 1)
                        check_one("vkb_tc_q4_f16out", label, w, x, M, false, 2e-3, [&](void* y) {
                            return VK(vkb_gemm_q4_tc(dq, ds, dx, y, sh.N, sh.K, M, (vkb_stream_t)g_st),
                                      "vkb_gemm_q4_tc");
                        }, rng);
                    check_one("cublas_fp16", label, w, x, M, true, 2e-3, [&](void* y) {   // the control
                        cublas_f16(dwf, dx, (float*)y, sh.N, sh.K, M);
                        return true;
                    }, rng);
                    check_one("dq4+cublas", label, w, x, M, true, 2e-3, [&](void* y) {   // packed -> GPU dequant
                        if (!VK(vkb_dequant(VKB_FMT_Q4, dq, ds, dwq, sh.N, sh.K, 0, (vkb_stream_t)g_st), "vkb_dequant"))
                            return false;
                        cublas_f16(dwq, dx, (float*)y, sh.N, sh.K, M);
                        return true;
                    }, rng);
                }
                if (fmt == VKB_FMT_Q8 && xc.kind != 1) {   // the Q8 prompt GEMM (tc_q8, planned by the reference)
                    check_one("vkb_tc_q8", label, w, x, M, true, 2e-3, [&](void* y) {
                        return VK(vkb_gemm_q8_tc_f32(dq, ds, dx, (float*)y, sh.N, sh.K, M, (vkb_stream_t)g_st),
                                  "vkb_gemm_q8_tc");
                    }, rng);
                }
                CK(cudaFree(dx));
            }
            CK(cudaFree(dq));
            CK(cudaFree(ds));
            if (dwf) CK(cudaFree(dwf));
            if (dwq) CK(cudaFree(dwq));
        }
    }
}

// MoE: a pool of E experts stacked [E][N][K], T tokens x k distinct experts from a device index list; every slot
// y[t][j] against the reference of expert idx[t][j] (a wrong expert or a wrong slot fails).
static void check_moe(bool sabotage, std::mt19937& rng) {
    struct MoeCase { const char* name; int E, topk, N, K; };
    static const MoeCase MOE[] = {{"qwen36_expert_gate_up", 128, 8, 512, 2048}, {"qwen36_expert_down", 128, 8, 2048, 512},
                                  {"flashnext_expert_gate_up", 160, 10, 640, 2560},
                                  {"flashnext_expert_down", 160, 10, 2560, 640}};
    for (const MoeCase& mc : MOE) {
        const Weights w = make_weights(VKB_FMT_Q4, mc.N * mc.E, mc.K, rng);
        void* dq = dupload(packed(w, sabotage));
        void* ds = dupload(w.scale);
        for (int T : {1, 8, 64}) {
            std::vector<int32_t> idx((size_t)T * mc.topk);
            vkb_synth_topk(rng(), T, mc.E, mc.topk, idx.data());
            const auto x = make_x(T, mc.K, 0, rng);
            int32_t* didx = dupload(idx);
            void* dx = dupload(x);
            const size_t ny = (size_t)T * mc.topk * mc.N;
            float* dy = dalloc<float>(ny);
            CK(cudaMemsetAsync(dy, 0, ny * 4, g_st));
            if (VK(vkb_moe(VKB_FMT_Q4, dq, ds, didx, T, mc.topk, dx, dy, 1, mc.E, 0, mc.N, mc.K, (vkb_stream_t)g_st),
                   "vkb_moe")) {
                CK(cudaStreamSynchronize(g_st));
                std::vector<float> y(ny);
                CK(cudaMemcpy(y.data(), dy, ny * 4, cudaMemcpyDeviceToHost));
                Worst r;
                for (int t = 0; t < T; ++t)
                    for (int j = 0; j < mc.topk; ++j)
                        for (int s = 0; s < 34; ++s) {
                            const int n = s == 0 ? 0 : s == 1 ? mc.N - 1 : (int)(rng() % (uint32_t)mc.N);
                            double mag;
                            const int row = idx[(size_t)t * mc.topk + j] * mc.N + n;
                            const double ref = ref_dot(w, x.data() + (size_t)t * mc.K, row, &mag);
                            const double err =
                                std::fabs(y[((size_t)t * mc.topk + j) * mc.N + n] - ref) / (mag + 1e-12);
                            if (err > r.err) { r.err = err; r.m = t; r.n = n; }
                        }
                verdict("vkb_moe_q4", std::string(mc.name) + "_pool" + std::to_string(mc.E) + "_top" +
                        std::to_string(mc.topk), T, r, r.err <= 1e-4);
            }
            CK(cudaFree(didx));
            CK(cudaFree(dx));
            CK(cudaFree(dy));
        }
        CK(cudaFree(dq));
        CK(cudaFree(ds));
    }
}

// Rows that are not a multiple of any tile (1031), every output checked, sentinels around y: nothing is written past
// the M x N output. Then an unsupported token count: nothing launched, nothing written (src/bakeoff.cu:580-640).
static void check_odd_rows(bool sabotage, std::mt19937& rng) {
    const int N = 1031, K = 2048, PAD = 1024;
    const float SENT = -12345.f;
    const Weights w = make_weights(VKB_FMT_Q4, N, K, rng);
    void* dq = dupload(packed(w, sabotage));
    void* ds = dupload(w.scale);
    for (int M : {1, 2, 3, 5, 8, 9, 100}) {
        const auto x = make_x(M, K, 0, rng);
        void* dx = dupload(x);
        std::vector<float> xf(x.size());   // the same activations as fp32 (the fp32-in entry, src/bakeoff.cu:421-423)
        for (size_t i = 0; i < x.size(); ++i) xf[i] = f32(x[i]);
        float* dxf = dupload(xf);
        void* dxh = dalloc<uint16_t>(x.size());
        const std::vector<float> init((size_t)M * N + 2 * PAD, SENT);
        float* dbuf = dupload(init);
        for (int who = 0; who < 3; ++who) {   // decode GEMV, prompt GEMM, decode with fp32 activations
            if (who != 1 && M > 8) continue;
            CK(cudaMemcpy(dbuf, init.data(), init.size() * 4, cudaMemcpyHostToDevice));
            const bool ran = who == 0 ? VK(gemv_f32(VKB_FMT_Q4, dq, ds, dx, dbuf + PAD, N, K, M), "vkb_gemv")
                             : who == 1 ? VK(vkb_gemm_q4_tc_f32(dq, ds, dx, dbuf + PAD, N, K, M, (vkb_stream_t)g_st),
                                             "vkb_gemm_q4_tc")
                                        : VK(vkb_gemv_q4_f32in(dq, ds, dxf, dxh, dbuf + PAD, N, K, M,
                                                               (vkb_stream_t)g_st), "vkb_gemv_q4_f32in");
            CK(cudaStreamSynchronize(g_st));
            std::vector<float> out(init.size());
            CK(cudaMemcpy(out.data(), dbuf, out.size() * 4, cudaMemcpyDeviceToHost));
            int spill = 0;
            for (int i = 0; i < PAD; ++i) spill += (out[i] != SENT) + (out[PAD + (size_t)M * N + i] != SENT);
            Worst r;
            for (int m = 0; m < M; ++m)
                for (int n = 0; n < N; ++n) {
                    double mag;
                    const double ref = ref_dot(w, x.data() + (size_t)m * K, n, &mag);
                    const double err = std::fabs(out[PAD + (size_t)m * N + n] - ref) / (mag + 1e-12);
                    if (err > r.err) { r.err = err; r.m = m; r.n = n; }
                }
            verdict(who == 0 ? "vkb_q4" : who == 1 ? "vkb_tc_q4" : "vkb_q4_f32in", "odd_rows_1031x2048", M, r,
                    ran && spill == 0 && r.err <= (who == 1 ? 2e-3 : 1e-4));
        }
        CK(cudaFree(dx));
        CK(cudaFree(dxf));
        CK(cudaFree(dxh));
        CK(cudaFree(dbuf));
    }
    {   // unsupported token count for the decode GEMV (9 > 8): returns "unsupported", writes nothing
        const int M = 9;
        void* dx = dupload(std::vector<uint16_t>((size_t)M * K, f16(0.5f)));
        const std::vector<float> init((size_t)M * N, SENT);
        float* dy = dupload(init);
        const int rc = gemv_f32(VKB_FMT_Q4, dq, ds, dx, dy, N, K, M);
        CK(cudaStreamSynchronize(g_st));
        std::vector<float> out(init.size());
        CK(cudaMemcpy(out.data(), dy, out.size() * 4, cudaMemcpyDeviceToHost));
        bool untouched = true;
        for (float v : out) untouched &= v == SENT;
        const bool ok = rc == VKB_EUNSUPPORTED && untouched;
        g_failures += !ok;
        printf("check,vkb_q4_unsupported_M,odd_rows_1031x2048,%d,0,%d,0,%s\n", M, rc, ok ? "ok" : "FAIL");
        CK(cudaFree(dx));
        CK(cudaFree(dy));
    }
    {   // the same through the fp32-in entry on a big table (the reference's check, src/bakeoff.cu:448-470): nothing
        // launched, so neither the output nor the fp16 scratch (where a conversion would land) is touched
        const int M = 9, NB = 4096;
        const Weights wb = make_weights(VKB_FMT_Q4, NB, K, rng);
        void* dqb = dupload(packed(wb, sabotage));
        void* dsb = dupload(wb.scale);
        float* dxf = dupload(std::vector<float>((size_t)M * K, 0.5f));
        const std::vector<uint16_t> hs((size_t)M * K, f16(-7.f));
        void* dxh = dupload(hs);
        const std::vector<float> init((size_t)M * NB, SENT);
        float* dy = dupload(init);
        const int rc = vkb_gemv_q4_f32in(dqb, dsb, dxf, dxh, dy, NB, K, M, (vkb_stream_t)g_st);
        CK(cudaStreamSynchronize(g_st));
        std::vector<float> out(init.size());
        std::vector<uint16_t> hout(hs.size());
        CK(cudaMemcpy(out.data(), dy, out.size() * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(hout.data(), dxh, hout.size() * 2, cudaMemcpyDeviceToHost));
        bool untouched = true;
        for (float v : out) untouched &= v == SENT;
        for (uint16_t v : hout) untouched &= v == hs[0];
        const bool ok = rc == VKB_EUNSUPPORTED && untouched;
        g_failures += !ok;
        printf("check,vkb_q4_f32in_unsupported_M,big_4096x2048,%d,0,%d,0,%s\n", M, rc, ok ? "ok" : "FAIL");
        CK(cudaFree(dqb));
        CK(cudaFree(dsb));
        CK(cudaFree(dxf));
        CK(cudaFree(dxh));
        CK(cudaFree(dy));
    }
    CK(cudaFree(dq));
    CK(cudaFree(ds));
}

// Qwen3-1.7B's MLP gate + up + SwiGLU (gate and up 6144x2048, stacked), the reference's check (src/bakeoff.cu:370-406):
// the stacked product against the double reference on 256 sampled outputs (both halves; 1e-4 here, the exact-code
// class -- the reference's own kernel is fp16-class, 2e-3) and out against silu(gate) * up recomputed in double from
// that product (1e-5), one row per token count: max_err_rel is the product's error, worst_m the SwiGLU error.
static void check_glu(bool sabotage, std::mt19937& rng) {
    const int N = 6144, K = 2048;
    const Weights w = make_weights(VKB_FMT_Q4, 2 * N, K, rng);
    void* dq = dupload(packed(w, sabotage));
    void* ds = dupload(w.scale);
    for (int M : {1, 2, 4, 8}) {
        const auto x = make_x(M, K, 0, rng);
        std::vector<float> xf(x.size());
        for (size_t i = 0; i < x.size(); ++i) xf[i] = f32(x[i]);
        float* dxf = dupload(xf);
        void* dxh = dalloc<uint16_t>(x.size());
        float* dys = dalloc<float>((size_t)M * 2 * N);
        float* dout = dalloc<float>((size_t)M * N);
        const bool ran = VK(vkb_gate_up_glu_q4_f32in(dq, ds, dxf, dxh, dys, dout, N, K, M, (vkb_stream_t)g_st),
                            "vkb_gate_up_glu_q4_f32in");
        CK(cudaStreamSynchronize(g_st));
        std::vector<float> ys((size_t)M * 2 * N), out((size_t)M * N);
        CK(cudaMemcpy(ys.data(), dys, ys.size() * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(out.data(), dout, out.size() * 4, cudaMemcpyDeviceToHost));
        Worst mm, glu;
        for (int i = 0; i < 256; ++i) {
            const int m = (int)(rng() % (uint32_t)M), n = (int)(rng() % (uint32_t)N);
            for (int part = 0; part < 2; ++part) {
                const int row = n + part * N;
                double mag;
                const double ref = ref_dot(w, x.data() + (size_t)m * K, row, &mag);
                const double e = std::fabs(ys[(size_t)m * 2 * N + row] - ref) / (mag + 1e-12);
                if (e > mm.err) { mm.err = e; mm.m = m; mm.n = row; }
            }
            const double g = ys[(size_t)m * 2 * N + n], u = ys[(size_t)m * 2 * N + N + n];
            const double want = g / (1.0 + std::exp(-g)) * u;
            const double e = std::fabs(out[(size_t)m * N + n] - want) / (std::fabs(want) + 1e-6);
            if (e > glu.err) { glu.err = e; glu.m = m; glu.n = n; }
        }
        // one verdict for both parts, in the reference's columns (src/bakeoff.cu:401-403): max_err_rel = the stacked
        // product's error, worst_m = the SwiGLU error, worst_n = 0
        const bool ok = ran && mm.err <= 1e-4 && glu.err <= 1e-5;
        g_failures += !ok;
        printf("check,vkb_glu_q4_f32in,qwen3_1p7b_mlp_gate_up,%d,%.3g,%.3g,0,%s\n", M, mm.err, glu.err,
               ok ? "ok" : "FAIL");
        fflush(stdout);
        CK(cudaFree(dxf));
        CK(cudaFree(dxh));
        CK(cudaFree(dys));
        CK(cudaFree(dout));
    }
    CK(cudaFree(dq));
    CK(cudaFree(ds));
}

static int run_check(bool sabotage) {
    std::mt19937 rng(1234);
    printf("check,contender,shape,M,max_err_rel,worst_m,worst_n,verdict\n");
    check_tables(sabotage, rng);
    check_moe(sabotage, rng);
    check_odd_rows(sabotage, rng);
    check_glu(sabotage, rng);
    unsigned int bits = 0;
    const int rc = vkb_device_status(&bits);
    if (rc != 0 || bits != 0) {
        fprintf(stderr, "device status %u (rc %d)\n", bits, rc);
        ++g_failures;
    }
    fprintf(stderr, "%d failure(s)%s\n", g_failures, sabotage ? " (sabotage mode: failures expected)" : "");
    return g_failures ? 1 : 0;
}

int main(int argc, char** argv) {
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, 0));
    g_l2 = (size_t)prop.l2CacheSize;
    fprintf(stderr, "device: %s (sm_%d%d), %d SMs, L2 %d MB, libvkb %d\n", prop.name, prop.major, prop.minor,
            prop.multiProcessorCount, prop.l2CacheSize >> 20, vkb_version());
    CK(cudaStreamCreateWithFlags(&g_st, cudaStreamNonBlocking));
    CB(cublasCreate(&g_hb));
    CB(cublasSetStream(g_hb, g_st));
    void* ws = dalloc<uint8_t>(64u << 20);   // a fixed cuBLAS workspace, so graph capture never allocates
    CB(cublasSetWorkspace(g_hb, ws, 64u << 20));
    int rc = 0;
    if (argc > 1 && !strcmp(argv[1], "--check")) {
        const char* sab = getenv("BAKEOFF_SABOTAGE");
        rc = run_check(sab && sab[0] == '1');
    } else {
        run_sweep();
    }
    CB(cublasDestroy(g_hb));
    CK(cudaFree(ws));
    CK(cudaStreamDestroy(g_st));
    return rc;
}
