// TEST INFRASTRUCTURE ONLY (never linked into libvkb.so, never on a product path).
//
// Builds the reference's own host-side model straight from its source file, src/bakeoff.cu (which includes
// stage2..5.cuh), by compiling it here with its main() renamed, and exposes the pieces the parity tests, the golden
// fixture generator and the CPU baseline need through a C ABI:
//   make_weights / pack_q4 / ref_value / ref_scale     reference src/bakeoff.cu:201-235
//   make_q2 / ref_q2                                   reference src/stage2.cuh:237-244, :261-270
//   pack_q2_rowmajor                                   reference src/stage3_lut.cuh:90-97
// The reference source is NOT copied into this repository: oracle/Makefile compiles it where it lies, into
// oracle/_ref/ (git-ignored; it travels with the working tree to the GPU box as a built library).
#define main bakeoff_main
#include "bakeoff.cu"
#undef main

#include <thread>

extern "C" {

void* ref_rng_new(unsigned seed) { return new std::mt19937(seed); }
void ref_rng_free(void* r) { delete static_cast<std::mt19937*>(r); }
unsigned ref_rng_next(void* r) { return (*static_cast<std::mt19937*>(r))(); }

static HostQ to_hostq(int N, int K, const int8_t* codes, const uint16_t* scales) {
    HostQ h{N, K, std::vector<int8_t>(codes, codes + (size_t)N * K), std::vector<half>((size_t)N * K / GROUP)};
    memcpy(h.scale.data(), scales, h.scale.size() * 2);
    return h;
}

// make_weights(N, K, bits, rng): codes [N][K], scales [N][K/32] (fp16 bits)
void ref_make_weights(void* rng, int N, int K, int bits, int8_t* codes, uint16_t* scales) {
    HostQ h = make_weights(N, K, bits, *static_cast<std::mt19937*>(rng));
    memcpy(codes, h.code.data(), h.code.size());
    memcpy(scales, h.scale.data(), h.scale.size() * 2);
}

void ref_make_q2(void* rng, int N, int K, int8_t* codes, uint16_t* scales) {
    HostQ2 h = make_q2(N, K, *static_cast<std::mt19937*>(rng));
    memcpy(codes, h.code.data(), h.code.size());
    memcpy(scales, h.scale_rowmajor.data(), h.scale_rowmajor.size() * 2);
}

// the check's activations: U[-1, 1] floats rounded to fp16, times mul (1 or 1e-3 for +tinyx), src/bakeoff.cu:504-506
void ref_uniform_x(void* rng, size_t n, float mul, uint16_t* out) {
    std::uniform_real_distribution<float> xd(-1.f, 1.f);
    auto& g = *static_cast<std::mt19937*>(rng);
    for (size_t i = 0; i < n; ++i) {
        half v = __float2half(xd(g) * mul);
        memcpy(out + i, &v, 2);
    }
}

// the +bigx channels, src/bakeoff.cu:507-513
void ref_bigx(void* rng, int M, int K, uint16_t* x) {
    auto& g = *static_cast<std::mt19937*>(rng);
    std::uniform_real_distribution<float> big(20000.f, 60000.f);
    const int k0 = K / 3 / 64 * 64;
    for (int m = 0; m < M; ++m)
        for (int k = k0; k < std::min(K, k0 + 64); ++k) {
            half v = __float2half((g() & 1 ? 1.f : -1.f) * big(g));
            memcpy(x + (size_t)m * K + k, &v, 2);
        }
}

void ref_pack_q4(int N, int K, const int8_t* codes, const uint16_t* scales, int sabotage, uint32_t* out) {
    HostQ h = to_hostq(N, K, codes, scales);
    std::vector<uint32_t> p = pack_q4(h, sabotage != 0);
    memcpy(out, p.data(), p.size() * 4);
}

void ref_pack_q2_rowmajor(int N, int K, const int8_t* codes, const uint16_t* scales, int sabotage, uint32_t* out) {
    HostQ2 h{N, K, std::vector<int8_t>(codes, codes + (size_t)N * K), std::vector<half>((size_t)N * K / GROUP)};
    memcpy(h.scale_rowmajor.data(), scales, h.scale_rowmajor.size() * 2);
    std::vector<uint32_t> q;
    pack_q2_rowmajor(h, sabotage != 0, q);
    memcpy(out, q.data(), q.size() * 4);
}

// ref_value / ref_scale for every (m, n): out_val, out_scale [M][N] (either may be null)
void ref_values(int N, int K, int M, const int8_t* codes, const uint16_t* scales, const uint16_t* x, double* out_val,
                double* out_scale) {
    HostQ h = to_hostq(N, K, codes, scales);
    std::vector<half> xv((size_t)M * K);
    memcpy(xv.data(), x, xv.size() * 2);
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            if (out_val) out_val[(size_t)m * N + n] = ref_value(h, xv, m, n);
            if (out_scale) out_scale[(size_t)m * N + n] = ref_scale(h, xv, m, n);
        }
}

void ref_q2_values(int N, int K, const int8_t* codes, const uint16_t* scales, const uint16_t* x, double* out_val,
                   double* out_mag) {
    HostQ2 h{N, K, std::vector<int8_t>(codes, codes + (size_t)N * K), std::vector<half>((size_t)N * K / GROUP)};
    memcpy(h.scale_rowmajor.data(), scales, h.scale_rowmajor.size() * 2);
    std::vector<half> xv(K);
    memcpy(xv.data(), x, (size_t)K * 2);
    for (int n = 0; n < N; ++n) {
        double mag;
        const double v = ref_q2(h, xv, n, &mag);
        if (out_val) out_val[n] = v;
        if (out_mag) out_mag[n] = mag;
    }
}

// The reference's CPU path timed as the CPU baseline: ref_value for the outputs [row0, row0 + nrows) x M tokens of an
// N x K table, split over `threads` std::threads by output row. Returns the checksum sum(y) so the work is not
// optimised away; out (optional) receives [M][nrows].
double ref_gemv_mt(int N, int K, int M, const int8_t* codes, const uint16_t* scales, const uint16_t* x, int row0,
                   int nrows, int threads, double* out) {
    HostQ h = to_hostq(N, K, codes, scales);
    std::vector<half> xv((size_t)M * K);
    memcpy(xv.data(), x, xv.size() * 2);
    if (threads < 1) threads = 1;
    std::vector<double> part(threads, 0.0);
    std::vector<std::thread> pool;
    for (int w = 0; w < threads; ++w)
        pool.emplace_back([&, w] {
            double sum = 0;
            for (int r = row0 + w; r < row0 + nrows; r += threads)
                for (int m = 0; m < M; ++m) {
                    const double v = ref_value(h, xv, m, r);
                    sum += v;
                    if (out) out[(size_t)m * nrows + (r - row0)] = v;
                }
            part[w] = sum;
        });
    for (auto& t : pool) t.join();
    double s = 0;
    for (double p : part) s += p;
    return s;
}

// The benchmark's synthetic weights and activations without libvkb.so (bench.py's reference arm loads only this
// library): n normal draws from std::mt19937(seed), Box-Muller on pairs of 32-bit draws u = (r + 0.5) / 2^32 computed
// in double, times stddev, rounded to float -- the definition the benchmark states for its inputs (BASELINE: fp32
// N(0, 0.02) weights and fp16 N(0, 1) activations from a seed). tests/test_oracle.py pins it bit for bit against the
// library's vkb_synth_normal.
void oracle_synth_normal(unsigned seed, size_t n, float stddev, float* out) {
    std::mt19937 rng(seed);
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        const double u1 = ((double)rng() + 0.5) / 4294967296.0;
        const double u2 = ((double)rng() + 0.5) / 4294967296.0;
        const double r = std::sqrt(-2.0 * std::log(u1));
        out[i] = (float)(r * std::cos(two_pi * u2) * stddev);
        if (i + 1 < n) out[i + 1] = (float)(r * std::sin(two_pi * u2) * stddev);
    }
}

}  // extern "C"
