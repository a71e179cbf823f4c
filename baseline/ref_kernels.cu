// The reference's own GPU kernels, rebuilt for sm_100a, for the same-GPU comparison section of bench.py (never linked
// into libvkb.so, never on a product path).
//
// src/bakeoff.cu (which includes stage2..5.cuh) is compiled where it lies by baseline/Makefile, with its main()
// renamed; nothing from the reference is copied into this repository. The calls below go through the reference's own
// launchers and pick rules, unchanged:
//   fused_q4_v2w   fused_q4_v2_any(M, true, ...)        src/stage2.cuh:213-224    Q4, 1/2/4/8 tokens
//   fused_q8       fused_q8_any                         src/bakeoff.cu:272-280    Q8, 1/2/4/8 tokens
//   q2w_alu_v3     launch_q2w_alu_v3                    src/stage3_lut.cuh:183-185 2-bit, 1 token
//   fused_q4_v3    fused_q4_v3_any (its pick rule)      src/stage5_gap8.cuh:188-205 Q4, 1/2/4/8 tokens
//   tc_q4          launch_tc_q4                         src/stage2.cuh:226-229    prompt, M % 64 == N % 64 == 0
//   tc_q4_v2       launch_tc_q4_v2 (its pick rule)      src/stage4_tc.cuh:182-200 prompt, M, N, K % 64 == 0
//   moe_fused_q4   moe_fused_q4<<<((N+3)/4, E), 128>>>  src/bakeoff.cu:157-186, :826-830  E <= 16 experts, one token each
// The launchers issue their kernels on the default stream. This file is compiled with --default-stream per-thread,
// so that stream is the calling thread's per-thread stream, which can be captured: ref_time_us captures 50 calls in a
// CUDA graph and replays it, the reference's time_us (src/bakeoff.cu:283-298: 20 warm-up calls, the median of 5 x 50
// calls) without host launch cost -- the same method bench.py uses for this library's kernels -- and cycles the
// weight copies the caller passes (>= 4x L2, so every call reads HBM; the reference's own 96 MB sits inside B200's
// L2). Every output is fp32 [M][N], the reference's float* y.
//
// Errors: the reference's CK macro exits the process on a CUDA error (src/bakeoff.cu:43-46); bench.py therefore runs
// this library in a child process.
#define main bakeoff_main
#include "bakeoff.cu"
#undef main

enum { RK_FUSED_Q4_V2W = 0, RK_FUSED_Q8 = 1, RK_Q2W_ALU_V3 = 2, RK_FUSED_Q4_V3 = 3, RK_TC_Q4 = 4, RK_TC_Q4_V2 = 5 };

// One call of the reference launcher `kind`; false when the launcher does not take (M, N, K) (nothing launched).
static bool ref_call(int kind, int M, const void* q, const void* s, const void* x, float* y, int N, int K) {
    const uint32_t* q4 = static_cast<const uint32_t*>(q);
    const half* sh = static_cast<const half*>(s);
    const half* xh = static_cast<const half*>(x);
    switch (kind) {
        case RK_FUSED_Q4_V2W: return fused_q4_v2_any(M, true, q4, sh, xh, y, N, K);
        case RK_FUSED_Q8: return fused_q8_any(M, static_cast<const uint2*>(q), sh, xh, y, N, K);
        case RK_Q2W_ALU_V3:
            if (M != 1) return false;
            launch_q2w_alu_v3(q4, sh, xh, y, N, K);
            return true;
        case RK_FUSED_Q4_V3: return fused_q4_v3_any(M, q4, sh, xh, y, N, K);
        case RK_TC_Q4:
            if (!tc_q4_ok(M, N)) return false;
            launch_tc_q4(q4, sh, xh, y, N, K, M);
            return true;
        case RK_TC_Q4_V2:
            if (!tc_q4_v2_ok(M, N, K)) return false;
            launch_tc_q4_v2(q4, sh, xh, y, N, K, M);
            return true;
        default: return false;
    }
}

// E experts, one token each, one launch: expert e reads q[e], s[e], its token x + e * x_stride (halves), writes
// y + e * N (the reference's MoePtrs, filled by the host per call).
static bool ref_moe_call(int E, const void* const* q, const void* const* s, const void* x, long long x_stride, float* y,
                         int N, int K) {
    if (E < 1 || E > 16) return false;
    MoePtrs p{};
    for (int e = 0; e < E; ++e) {
        p.q[e] = static_cast<const uint32_t*>(q[e]);
        p.s[e] = static_cast<const half*>(s[e]);
        p.x[e] = static_cast<const half*>(x) + e * x_stride;
        p.y[e] = y + (size_t)e * N;
    }
    moe_fused_q4<<<dim3((N + 3) / 4, E), 128>>>(p, N, K);
    return true;
}

template <typename F>
static double graph_time_us(F call) {
    for (int i = 0; i < 20; ++i)
        if (!call(i)) return -1.0;
    CK(cudaStreamSynchronize(cudaStreamPerThread));
    cudaGraph_t g;
    cudaGraphExec_t ge;
    CK(cudaStreamBeginCapture(cudaStreamPerThread, cudaStreamCaptureModeThreadLocal));
    for (int k = 0; k < 50; ++k) call(20 + k);
    CK(cudaStreamEndCapture(cudaStreamPerThread, &g));
    CK(cudaGraphInstantiate(&ge, g, 0));
    CK(cudaGraphLaunch(ge, cudaStreamPerThread));
    cudaEvent_t a, b;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b));
    std::vector<double> t;
    for (int rep = 0; rep < 5; ++rep) {
        CK(cudaEventRecord(a, cudaStreamPerThread));
        CK(cudaGraphLaunch(ge, cudaStreamPerThread));
        CK(cudaEventRecord(b, cudaStreamPerThread));
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

extern "C" {

// One call of the reference kernel `kind` (RK_*), synchronised; 0 launched, 1 unsupported.
int ref_kernel_run(int kind, int M, const void* q, const void* s, const void* x, float* y, int N, int K) {
    const bool ok = ref_call(kind, M, q, s, x, y, N, K);
    CK(cudaStreamSynchronize(cudaStreamPerThread));
    return ok ? 0 : 1;
}

// Median microseconds per call of the reference kernel `kind`, call i using weight copy i % copies; < 0: unsupported.
double ref_kernel_time_us(int kind, int M, const void* const* q, const void* const* s, int copies, const void* x,
                          float* y, int N, int K) {
    if (copies < 1) return -1.0;
    return graph_time_us([&](int i) { return ref_call(kind, M, q[i % copies], s[i % copies], x, y, N, K); });
}

// The reference's one-launch MoE: q, s hold copies x E expert pointers (copy c, expert e at c * E + e).
int ref_moe_run(int E, const void* const* q, const void* const* s, const void* x, long long x_stride, float* y, int N,
                int K) {
    const bool ok = ref_moe_call(E, q, s, x, x_stride, y, N, K);
    CK(cudaStreamSynchronize(cudaStreamPerThread));
    return ok ? 0 : 1;
}

double ref_moe_time_us(int E, const void* const* q, const void* const* s, int copies, const void* x,
                       long long x_stride, float* y, int N, int K) {
    if (copies < 1) return -1.0;
    return graph_time_us([&](int i) {
        const int c = i % copies;
        return ref_moe_call(E, q + (size_t)c * E, s + (size_t)c * E, x, x_stride, y, N, K);
    });
}

}  // extern "C"
