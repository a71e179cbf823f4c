// Quantised matrix-vector product for 1..8 tokens (decode), dense or MoE, on sm_100a.
//
//   y[m][n] = sum_k x[m][k] * code[n][k] * scale[n][k/32]
//
// Weight formats are the bakeoff's, byte for byte (reference src/bakeoff.cu:5-8, :210-219, :486-490;
// src/stage3_lut.cuh:4, :90-97):
//   Q4  u32 [N][K/8]   word w of a row holds codes 8w..8w+7, code i in nibble i, stored as code + 8
//   Q8  i8  [N][K]     one two's-complement code per value
//   Q2  u32 [N][K/16]  word w holds codes 16w..16w+15, code i in bits 2i..2i+1, stored as code + 2
//   scales fp16 [N][K/32]; x fp16 [T][K]; y fp16 or fp32.
//
// Design (one CTA per SM, persistent over 16-row tiles):
//   * warp NW (the producer) streams 16-row x KS-column stages of codes and scales into a shared-memory ring, one 2-D
//     TMA box each (8-byte elements, so a box row can span a whole stage row of up to 1.5 KB). The boxes are 16 (Q8: 32) bytes
//     wider than the data they need, which pads every shared-memory row by that much and makes the consumers'
//     fragment reads bank-conflict free (the pad is zero-filled past the end of a row, or the next stage's first
//     bytes inside it). Few, large TMA requests are what keep HBM busy: 16-row x 128-byte boxes ran at under half
//     the bandwidth of these on B200. The weight stages are issued
//     before griddepcontrol.wait, so under programmatic dependent launch the next call's weight stream overlaps the
//     previous call's tail. The activations (after the wait): dense calls' small blocks are loaded by the consumers
//     themselves in fragment order (see qmv_xstage_max); larger blocks and MoE segments come in as 1-D bulk copies.
//   * warps 0..NW-1 split each stage's K range and run the m16n8k16 tensor-core MMA with the weights as A (16 rows)
//     and the tokens as B (8 columns). The codes enter the MMA exactly: the fp16 magic-number trick (0x6400 | n is
//     the half 1024 + n) turns two codes into one f16x2 with one LOP3 and one HSUB2/HFMA2, and every 32-value group is
//     accumulated on its own (two k16 steps) and then scaled in fp32, so the result is the exact-code fp32-sum class
//     of the reference's fused kernels (tolerance 1e-4 of sum|x*w|), not the fp16-rounded-weight class.
//   * inside one k16 step the order of k is free as long as A and B agree; each format picks the order that makes its
//     unpack cheapest, and the activations are either staged in that order or permuted to match with PRMT as loaded.
//   * per-tile partial sums of the NW warps are added in shared memory and written by warp 0.
#pragma once

#include "p2p.cuh"
#include "ptx.cuh"

namespace vkb {

enum : int { FMT_Q4 = 0, FMT_Q8 = 1, FMT_Q2 = 2 };

template <int F> struct FmtTraits;
template <> struct FmtTraits<FMT_Q4> { static constexpr int BITS = 4; };
template <> struct FmtTraits<FMT_Q8> { static constexpr int BITS = 8; };
template <> struct FmtTraits<FMT_Q2> { static constexpr int BITS = 2; };

constexpr int QMV_NW = 16;         // consumer warps per CTA
constexpr int QMV_KS_UNIT = 256;   // stage widths are multiples of this (8 groups; a 128-byte multiple of every format)
constexpr int QMV_ROWS = 16;       // weight rows per tile (the MMA's M)
constexpr int QMV_MAXTOK = 8;      // tokens per MMA column group (the MMA's N)

// QMV_MOE_P2P: MoE whose outputs are also pushed into every peer's copy of y (expert parallelism, peer stores).
// QMV_GLU: gate + up + SwiGLU over a stacked [2N][K] table (rows 0..N-1 gate, N..2N-1 up). Tiles come in pairs: tile
// 2j = gate rows 16j.., tile 2j + 1 = up rows N + 16j.. (a CTA's range is pair aligned, so adjacent warp groups take
// the two halves); the gate tile's reducer hands its sums to the up tile's reducer through shared memory, which
// writes out = silu(gate) * up (and the stacked products, when asked). Stages and reductions are the dense GEMV's.
enum : int { QMV_DENSE = 0, QMV_MOE = 1, QMV_MOE_P2P = 2, QMV_GLU = 3 };

// Division by a divisor fixed at launch, without the ~150-cycle integer division sequence on the kernels' prologue
// path (a MoE call's whole prologue comes after its dependency): q = (umulhi(x, mul) + x) >> shift with the host's
// round-up multiplier mul = floor(2^32 (2^shift - d) / d) + 1, shift = ceil(log2 d); exact for 0 <= x < 2^31.
struct FastDiv {
    uint32_t mul, shift;
};
__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    return FastDiv{(uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1), l};
}
__device__ __forceinline__ int fdiv(int x, FastDiv f) {
    return (int)((__umulhi((uint32_t)x, f.mul) + (uint32_t)x) >> f.shift);
}

struct QmvArgs {
    const __half* x;         // [T][K] (fp32 [T][K] for the XF32 kernels)
    float* ys;               // QMV_GLU: the stacked products [T][2N] (gate, then up) or null
    void* y;                 // dense: [T][N]; MoE: [T*topk][N]
    const int32_t* idx;      // MoE: [T*topk] global expert ids
    int N, K;                // rows per matrix (per expert), inner dimension
    int T;                   // dense: tokens (M); MoE: tokens
    int topk;                // MoE: slots per token
    int E_local, e0;         // MoE: experts held in this pool, id of the first one
    int zero_foreign;        // MoE: write zeros into the slots of experts outside the pool (expert-parallel combine)
    P2PArgs pp;              // QMV_MOE_P2P: every rank's copy of y (pp.peer_base) and flags of the epoch protocol
    int KS, nchunks;         // stage width in k values, stages per row tile
    int cpitch, spitch;      // shared bytes per row of a stage: codes (KS*bits/8 + pad), scales (KS/16 + 16)
    int nstage;              // ring depth
    int stage_bytes;         // shared bytes per stage (1024-aligned)
    int xpitch;              // shared bytes per staged activation row
    int xrows;               // staged activation rows per buffer (<= 8)
    int xres;                // MoE over T <= 8 tokens: all T rows staged once (one buffer); else per segment (two)
    int tilesN;              // ceil(N / 16)
    int wg;                  // consumer warp groups (1, 2 or 4), with nstage >= wg * nchunks
    int ring_off, x_off, red_off, bar_off, moe_off;   // shared-memory carve-up (bytes from the aligned base)
    FastDiv dv_tiles, dv_topk, dv_grid;               // by tilesN, topk (MoE; else 1), the launch's grid size
};

// ---- per-format unpack: one 32-bit word of codes -> the four f16x2 A registers this thread feeds the MMA ----------

// Q4, word t of a group: (c0,c4) (c1,c5) | (c2,c6) (c3,c7); exact code values.
__device__ __forceinline__ void unpack_q4(uint32_t v, uint32_t (&a)[4]) {
    const uint32_t M = 0x64006400u;
    const uint32_t vs = v >> 8;
    a[0] = h2_sub(and_or(v, 0x000F000Fu, M), 0x64086408u);                 // 1024 + n - 1032
    a[1] = h2_fma(and_or(v, 0x00F000F0u, M), 0x2C002C00u, 0xD480D480u);    // (1024 + 16n)/16 - 72
    a[2] = h2_sub(and_or(vs, 0x000F000Fu, M), 0x64086408u);
    a[3] = h2_fma(and_or(vs, 0x00F000F0u, M), 0x2C002C00u, 0xD480D480u);
}

// Q8, words 2t and 2t+1 of a group: (c0,c1) (c2,c3) | (c4,c5) (c6,c7).
__device__ __forceinline__ void unpack_q8(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    const uint32_t u0 = w0 ^ 0x80808080u, u1 = w1 ^ 0x80808080u;   // offset binary: c + 128
    a[0] = h2_sub(prmt(u0, 0x64646464u, 0x4140u), 0x64806480u);    // 1024 + c + 128 - 1152
    a[1] = h2_sub(prmt(u0, 0x64646464u, 0x4342u), 0x64806480u);
    a[2] = h2_sub(prmt(u1, 0x64646464u, 0x4140u), 0x64806480u);
    a[3] = h2_sub(prmt(u1, 0x64646464u, 0x4342u), 0x64806480u);
}

// Q2, half h of word p (already shifted right by 8h): (c0,c8) (c1,c9) | (c2,c10) (c3,c11) of that half.
__device__ __forceinline__ void unpack_q2(uint32_t vs, uint32_t (&a)[4]) {
    const uint32_t M = 0x64006400u;
    a[0] = h2_sub(and_or(vs, 0x00030003u, M), 0x64026402u);                // 1024 + u - 1026
    a[1] = h2_fma(and_or(vs, 0x000C000Cu, M), 0x34003400u, 0xDC08DC08u);   // (1024 + 4u)/4 - 258
    a[2] = h2_fma(and_or(vs, 0x00300030u, M), 0x2C002C00u, 0xD420D420u);   // (1024 + 16u)/16 - 66
    a[3] = h2_fma(and_or(vs, 0x00C000C0u, M), 0x24002400u, 0xCC80CC80u);   // (1024 + 64u)/64 - 18
}

// Byte offset, inside a row of a stage, of the word(s) lane-in-quad t reads for stage-local group G.
template <int F>
__device__ __forceinline__ uint32_t code_off(int G, int t) {
    if constexpr (F == FMT_Q4) return 16 * G + 4 * t;          // word t of the group's 16 bytes
    else if constexpr (F == FMT_Q8) return 32 * G + 8 * t;     // words 2t, 2t+1 of the group's 32 bytes
    else return 8 * G + 4 * (t >> 1);                          // word t/2 of the group's 8 bytes
}

// The four A registers (two k16 steps) of one row for group G of the stage at shared address st.
template <int F>
__device__ __forceinline__ void load_a(uint32_t a, int t, uint32_t (&r)[4]) {
    if constexpr (F == FMT_Q4) {
        unpack_q4(lds32(a), r);
    } else if constexpr (F == FMT_Q8) {
        const uint2 w = lds64(a);
        unpack_q8(w.x, w.y, r);
    } else {
        unpack_q2(lds32(a) >> (8 * (t & 1)), r);
    }
}

// The B registers (two k16 steps) of this thread's token for the group whose activations start at shared address xa
// (xa already includes the thread's t offset). Padding token columns read a real row: their MMA columns are never
// stored, and the MMA keeps columns independent. PX: the rows are staged in fragment order (stage_x_chunk), so the
// four registers are one 16-byte load; otherwise they are in k order and permuted here.
template <int F, bool PX>
__device__ __forceinline__ void load_b(uint32_t xa, uint32_t (&b)[4]) {
    if constexpr (PX) {
        const uint4 v = lds128(xa);
        b[0] = v.x; b[1] = v.y; b[2] = v.z; b[3] = v.w;
    } else if constexpr (F == FMT_Q2) {
        const uint2 xa0 = lds64(xa), xb0 = lds64(xa + 16);
        b[0] = prmt(xa0.x, xb0.x, 0x5410u);   // (x0, x8)
        b[1] = prmt(xa0.x, xb0.x, 0x7632u);   // (x1, x9)
        b[2] = prmt(xa0.y, xb0.y, 0x5410u);   // (x2, x10)
        b[3] = prmt(xa0.y, xb0.y, 0x7632u);   // (x3, x11)
    } else {
        const uint4 v = lds128(xa);
        if constexpr (F == FMT_Q4) {
            b[0] = prmt(v.x, v.z, 0x5410u);   // (x0, x4)
            b[1] = prmt(v.x, v.z, 0x7632u);   // (x1, x5)
            b[2] = prmt(v.y, v.w, 0x5410u);   // (x2, x6)
            b[3] = prmt(v.y, v.w, 0x7632u);   // (x3, x7)
        } else {
            b[0] = v.x; b[1] = v.y; b[2] = v.z; b[3] = v.w;
        }
    }
}

// Per-thread byte offset of its activations inside a 32-value group (see load_b).
template <int F, bool PX>
__device__ __forceinline__ uint32_t x_lane_off(int t) {
    if constexpr (F == FMT_Q2 && !PX) return 32 * (t >> 1) + 8 * (t & 1);
    else return 16 * t;
}

// Fragment-order staging: 16-byte chunk c of a staged row is lane-in-quad (c & 3)'s four B registers of group c / 4,
// built from 8 activations in k order (lo, hi: f16x2 words 0-1 and 2-3 of the format's source pairs). Q4 takes
// activations 8c..8c+7 and pairs (x0,x4) (x1,x5) (x2,x6) (x3,x7); Q2 takes 4 of each half of its 16-value block
// (block c / 2, offset 4 (c & 1)) and pairs (x0,x8) (x1,x9) (x2,x10) (x3,x11); Q8 keeps k order.
template <int F>
__device__ __forceinline__ uint4 frag_order(uint2 lo, uint2 hi) {
    if constexpr (F == FMT_Q8) return make_uint4(lo.x, lo.y, hi.x, hi.y);
    else return make_uint4(prmt(lo.x, hi.x, 0x5410u), prmt(lo.x, hi.x, 0x7632u), prmt(lo.y, hi.y, 0x5410u),
                           prmt(lo.y, hi.y, 0x7632u));
}
// element offset, in a [K] row, of chunk c's first 4 source activations; the other 4 are chunk_hi further
template <int F>
__device__ __forceinline__ int chunk_src(int c) {
    if constexpr (F == FMT_Q2) return 16 * (c >> 1) + 4 * (c & 1);
    else return 8 * c;
}
template <int F>
__device__ __forceinline__ constexpr int chunk_hi() { return F == FMT_Q2 ? 8 : 4; }

// Dense calls with more activations than this (tokens x K) use the XB kernels: their rows come in by the producer's
// bulk copy in k order and the consumers permute each group's registers as they load them; smaller ones are loaded
// by the consumer threads themselves, in fragment order. Measured on B200 (µs, 50-call graphs): 8 x 6144 activations
// staged by the consumers took 2048x6144 2-bit from 4.7 to 5.7 and Q8 from 6.05 to 6.6, while 2 x 6144 took Q4
// 2560x6144 from 6.2 to 5.6; permuting the bulk copy in place once was slower than both (shared-memory traffic), and
// one kernel holding both loops ran both slower than the single-loop kernels. Q4 calls keep the consumers' staging up
// to twice as many values: at 32768 every Q4 case that moved got faster (2560x6144 at 4 tokens 6.37 -> 5.77 µs,
// 12288x2560 at 8 tokens 8.50 -> 8.22, 2048x6144 at 4 tokens 4.80 -> 4.67), while Q8 and 2-bit had one case faster
// and one slower each.
constexpr int QMV_XSTAGE_MAX = 16384;
__host__ __device__ constexpr int qmv_xstage_max(int fmt) {
    return fmt == FMT_Q4 ? 2 * QMV_XSTAGE_MAX : QMV_XSTAGE_MAX;
}

// One group: two k16 MMAs into a fresh fragment, then the per-row fp32 scales. ca: row g's codes in the stage;
// row g+8 is 8 * cp further.
template <int F, bool PX>
__device__ __forceinline__ void qmv_group(uint32_t ca, uint32_t cp, int G, int t, uint32_t xa, float s0, float s1,
                                          float (&acc)[4]) {
    uint32_t b[4], ar[4], ar8[4];
    load_b<F, PX>(xa, b);
    const uint32_t a = ca + code_off<F>(G, t);
    load_a<F>(a, t, ar);
    load_a<F>(a + 8 * cp, t, ar8);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_16816(d, ar[0], ar8[0], ar[1], ar8[1], b[0], b[1]);
    mma_16816(d, ar[2], ar8[2], ar[3], ar8[3], b[2], b[3]);
    acc[0] = fmaf(d[0], s0, acc[0]);
    acc[1] = fmaf(d[1], s0, acc[1]);
    acc[2] = fmaf(d[2], s1, acc[2]);
    acc[3] = fmaf(d[3], s1, acc[3]);
}

// This warp's groups [G0, G1) of one stage, stopping at K.
//   ca, cp: shared address of row g's codes in the stage, code row pitch
//   sc, sp: shared address of row g's scales in the stage, scale row pitch
//   xa:     shared address of this thread's activations for stage-local group 0
// U: groups per loop iteration (2, or 4 where the register budget allows: four independent MMA chains in flight).
template <int F, int U, bool PX>
__device__ __forceinline__ void consume_stage(uint32_t ca, uint32_t cp, uint32_t sc, uint32_t sp, int G0, int G1,
                                              uint32_t xa, int t, float (&acc)[4]) {
    int G = G0;
    if (G & 1) {   // odd start: single group, its scale from the aligned pair
        if (G < G1) {
            const uint32_t p0 = lds32(sc + 2 * (G - 1)), p1 = lds32(sc + 8 * sp + 2 * (G - 1));
            qmv_group<F, PX>(ca, cp, G, t, xa + 64 * G, half_hi_f32(p0), half_hi_f32(p1), acc);
        }
        ++G;
    }
    if constexpr (U == 4) {
#pragma unroll 1
        for (; G + 3 < G1; G += 4) {
            const uint32_t p0 = lds32(sc + 2 * G), p1 = lds32(sc + 8 * sp + 2 * G);
            const uint32_t q0 = lds32(sc + 2 * G + 4), q1 = lds32(sc + 8 * sp + 2 * G + 4);
            qmv_group<F, PX>(ca, cp, G, t, xa + 64 * G, half_lo_f32(p0), half_lo_f32(p1), acc);
            qmv_group<F, PX>(ca, cp, G + 1, t, xa + 64 * (G + 1), half_hi_f32(p0), half_hi_f32(p1), acc);
            qmv_group<F, PX>(ca, cp, G + 2, t, xa + 64 * (G + 2), half_lo_f32(q0), half_lo_f32(q1), acc);
            qmv_group<F, PX>(ca, cp, G + 3, t, xa + 64 * (G + 3), half_hi_f32(q0), half_hi_f32(q1), acc);
        }
    }
#pragma unroll 1
    for (; G + 1 < G1; G += 2) {
        const uint32_t p0 = lds32(sc + 2 * G), p1 = lds32(sc + 8 * sp + 2 * G);
        qmv_group<F, PX>(ca, cp, G, t, xa + 64 * G, half_lo_f32(p0), half_lo_f32(p1), acc);
        qmv_group<F, PX>(ca, cp, G + 1, t, xa + 64 * (G + 1), half_hi_f32(p0), half_hi_f32(p1), acc);
    }
    if (G < G1) {
        const uint32_t p0 = lds32(sc + 2 * G), p1 = lds32(sc + 8 * sp + 2 * G);
        qmv_group<F, PX>(ca, cp, G, t, xa + 64 * G, half_lo_f32(p0), half_lo_f32(p1), acc);
    }
}

// Two fp32 activations (bit patterns) -> one f16x2 register (lo in the low half), round to nearest even: the
// reference's fp32 -> fp16 conversion of the activations.
__device__ __forceinline__ uint32_t cvt_h2(uint32_t lo, uint32_t hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(__uint_as_float(hi)), "f"(__uint_as_float(lo)));
    return d;
}

template <typename OutT> __device__ __forceinline__ OutT to_out(float v);
template <> __device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float to_out<float>(float v) { return v; }

// ---- MoE routing tables (built by each CTA, deterministically: every CTA builds the same) ------------------------
//
// A "segment" is one expert with up to 8 of its (token, slot) pairs: the tokens of one MMA column group. Segment order
// and the order of slots inside an expert change no result -- each output row is one tile's sum, and the MMA's columns
// are independent, so a slot's value does not depend on the column it lands in -- but every CTA of the grid must build
// the same segments, since each takes its own range of (segment, row tile) pairs.
struct MoeTables {
    int* slots;    // [nslots]     slot ids grouped by segment
    int* seg;      // [nslots]     (local expert << 16) | first position in `slots`, per segment
    int* segc;     // [nslots]     slots of the segment (1-8)
    int* nseg;     // [2]          segments; (CTA-wide routing) the largest load of one expert
    int* cnt;      // [E_local]    (more than 32 slots) slots per local expert
    int* off;      // [E_local]    (more than 32 slots) first position of each expert in `slots`
    int* segoff;   // [E_local]    (CTA-wide routing) first segment of each expert
    int* tmp;      // [nslots]     (CTA-wide routing) (local expert << 16) | atomic ticket, or -1
    int* list;     // [nslots]     (CTA-wide routing) slot ids by ticket inside each expert's range
};
// the arrays above, in this order
__host__ __device__ constexpr int moe_table_words(int E_local, int nslots) { return 5 * nslots + 3 * E_local + 2; }

__device__ __forceinline__ MoeTables moe_tables(uint8_t* base, int E_local, int nslots) {
    MoeTables t;
    int* p = reinterpret_cast<int*>(base);
    t.slots = p; p += nslots;
    t.seg = p; p += nslots;
    t.segc = p; p += nslots;
    t.nseg = p; p += 2;
    t.cnt = p; p += E_local;
    t.off = p; p += E_local;
    t.segoff = p; p += E_local;
    t.tmp = p; p += nslots;
    t.list = p;
    return t;
}

// At most 32 slots, one warp (one slot per lane): grouping by __match_any_sync, experts in order of first appearance
// from a ballot of the group leaders, one packed warp scan of (slots, segments) over the leaders -- registers only,
// then the table stores.
__device__ __forceinline__ void moe_route_small(const QmvArgs& a, MoeTables tb, int lane, int nslots) {
    const unsigned all = 0xffffffffu, below = (1u << lane) - 1u;
    int e = lane < nslots ? __ldg(a.idx + lane) - a.e0 : -1;
    if (e < 0 || e >= a.E_local) e = -1;
    const unsigned same = __match_any_sync(all, e);
    const int leader = __ffs(same) - 1;
    const bool lead = e >= 0 && lane == leader;
    const int c = __popc(same), segs = (c + QMV_MAXTOK - 1) / QMV_MAXTOK;
    const int mine = lead ? (c | (segs << 16)) : 0;   // slots in the low half (<= 32), segments in the high half
    int v = mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(all, v, d);
        if (lane >= d) v += u;
    }
    const int excl = v - mine, tot = __shfl_sync(all, v, 31);
    const int gexcl = __shfl_sync(all, excl, leader);
    if (e >= 0) tb.slots[(gexcl & 0xFFFF) + __popc(same & below)] = lane;
    if (lead) {
        const int first = excl & 0xFFFF, s0 = excl >> 16;
        for (int k = 0; k < segs; ++k) {
            tb.seg[s0 + k] = (e << 16) | (first + k * QMV_MAXTOK);
            tb.segc[s0 + k] = min(QMV_MAXTOK, c - k * QMV_MAXTOK);
        }
    }
    if (lane == 0) *tb.nseg = tot >> 16;
    __syncwarp();
}

// 33..MOE_WARP_MAX slots, one warp, in chunks of 32 (slot 32 r + lane). Per chunk, __match_any_sync groups the
// chunk's slots by expert, and a running count per expert (cnt, updated by each group's leader) gives every slot its
// place among its expert's slots in index order and marks the expert's first slot. Then one scan over the chunks of
// (slots, segments) at the experts' first slots orders the experts by first appearance, as moe_route_small does;
// each first slot publishes its expert's offsets (off) and segments, and every slot stores itself. Nine warp
// syncs and no CTA barrier: with 64 slots of 128 experts the CTA-wide routing took ~1.8 us after the dependency on
// B200 (in-kernel clock64 stamps), most of it in its five CTA barriers.
constexpr int MOE_WARP_MAX = 128;

__device__ __forceinline__ void moe_route_warp(const QmvArgs& a, MoeTables tb, int lane, int nslots) {
    constexpr int RM = MOE_WARP_MAX / 32;
    const unsigned all = 0xffffffffu, below = (1u << lane) - 1u;
    const int R = (nslots + 31) >> 5;   // chunks (2..RM)
    int e[RM], rk[RM];
    unsigned own = 0;                   // bit r: slot 32 r + lane is its expert's first slot
#pragma unroll
    for (int r = 0; r < RM; ++r) {      // all loads first
        const int i = 32 * r + lane;
        int v = i < nslots ? __ldg(a.idx + i) - a.e0 : -1;
        if (v < 0 || v >= a.E_local) v = -1;
        e[r] = v;
        rk[r] = 0;
    }
#pragma unroll
    for (int r = 0; r < RM; ++r)
        if (e[r] >= 0) tb.cnt[e[r]] = 0;
    __syncwarp();
#pragma unroll
    for (int r = 0; r < RM; ++r) {
        if (r < R) {   // (uniform over the warp)
            const unsigned same = __match_any_sync(all, e[r]);
            const int before = e[r] >= 0 ? tb.cnt[e[r]] : 0;   // slots of this expert in earlier chunks
            rk[r] = before + __popc(same & below);
            __syncwarp();
            if (e[r] >= 0 && lane == __ffs(same) - 1) {
                if (before == 0) own |= 1u << r;
                tb.cnt[e[r]] = before + __popc(same);
            }
            __syncwarp();
        }
    }
    int carry = 0;   // (slots | segments << 16) of the experts first seen in earlier chunks
#pragma unroll
    for (int r = 0; r < RM; ++r) {
        if (r < R) {
            const bool o = (own >> r) & 1u;
            const int c = o ? tb.cnt[e[r]] : 0, segs = (c + QMV_MAXTOK - 1) / QMV_MAXTOK;
            const int mine = c | (segs << 16);
            int v = mine;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int u = __shfl_up_sync(all, v, d);
                if (lane >= d) v += u;
            }
            const int excl = carry + v - mine;
            if (o) {
                const int first = excl & 0xFFFF, s0 = excl >> 16;
                tb.off[e[r]] = first;
                for (int k = 0; k < segs; ++k) {
                    tb.seg[s0 + k] = (e[r] << 16) | (first + k * QMV_MAXTOK);
                    tb.segc[s0 + k] = min(QMV_MAXTOK, c - k * QMV_MAXTOK);
                }
            }
            carry += __shfl_sync(all, v, 31);
        }
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < RM; ++r)
        if (e[r] >= 0) tb.slots[tb.off[e[r]] + rk[r]] = 32 * r + lane;
    if (lane == 0) *tb.nseg = carry >> 16;
    __syncwarp();
}

// Any number of slots, by every thread of the CTA (`barrier` synchronises them): counts per local expert by shared
// atomics, exclusive scans of the counts and of the segments over the experts (one warp), then the slots in index
// order inside each expert. The atomics' order differs between CTAs while all CTAs must see the same segments, so a
// slot's place is its count of smaller slot ids of its expert, not its atomic ticket. Up to MOE_SCAN_MAX slots per
// expert each slot lists itself in its expert's range by the ticket and counts the smaller ids listed there (a few
// steps for spread routing); past that -- one expert taking most slots -- one warp walks the list from the end in
// 32-slot chunks, counting each expert down from its load. Both give the same tables. Five barriers; the index list
// is read once, one load per thread.
constexpr int MOE_SCAN_MAX = 64;

template <typename Barrier>
__device__ __forceinline__ void moe_route_cta(const QmvArgs& a, MoeTables tb, int nslots, Barrier barrier) {
    const int tid = threadIdx.x, nth = blockDim.x, warp = tid >> 5, lane = tid & 31;
    const unsigned all = 0xffffffffu, below = (1u << lane) - 1u;
    for (int e = tid; e < a.E_local; e += nth) tb.cnt[e] = 0;
    barrier();
    for (int i = tid; i < nslots; i += nth) {
        const int e = __ldg(a.idx + i) - a.e0;
        tb.tmp[i] = (e < 0 || e >= a.E_local) ? -1 : (e << 16) | atomicAdd(&tb.cnt[e], 1);
    }
    barrier();
    if (warp == 0) {
        int run_off = 0, run_seg = 0, cmax = 0;
        for (int b = 0; b < a.E_local; b += 32) {
            const int e = b + lane;
            const int c = e < a.E_local ? tb.cnt[e] : 0;
            const int s = (c + QMV_MAXTOK - 1) / QMV_MAXTOK;
            int ic = c, is = s;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int vc = __shfl_up_sync(all, ic, d);
                const int vs = __shfl_up_sync(all, is, d);
                if (lane >= d) { ic += vc; is += vs; }
            }
            if (e < a.E_local) {
                tb.off[e] = run_off + ic - c;
                tb.segoff[e] = run_seg + is - s;
            }
            run_off += __shfl_sync(all, ic, 31);
            run_seg += __shfl_sync(all, is, 31);
            cmax = max(cmax, c);
        }
        cmax = __reduce_max_sync(all, cmax);
        if (lane == 0) {
            tb.nseg[0] = run_seg;
            tb.nseg[1] = cmax;
        }
    }
    barrier();
    const bool scan = tb.nseg[1] <= MOE_SCAN_MAX;
    if (scan) {
        for (int i = tid; i < nslots; i += nth) {
            const int v = tb.tmp[i];
            if (v >= 0) tb.list[tb.off[v >> 16] + (v & 0xFFFF)] = i;
        }
    }
    for (int e = tid; e < a.E_local; e += nth) {
        const int c = tb.cnt[e], first = tb.off[e], s0 = tb.segoff[e];
        for (int k = 0; k * QMV_MAXTOK < c; ++k) {
            tb.seg[s0 + k] = (e << 16) | (first + k * QMV_MAXTOK);
            tb.segc[s0 + k] = min(QMV_MAXTOK, c - k * QMV_MAXTOK);
        }
    }
    barrier();
    if (scan) {
        for (int i = tid; i < nslots; i += nth) {
            const int v = tb.tmp[i];
            if (v < 0) continue;
            const int first = tb.off[v >> 16], c = tb.cnt[v >> 16];
            int r = 0;
            for (int j = 0; j < c; ++j) r += tb.list[first + j] < i;
            tb.slots[first + r] = i;
        }
    } else if (warp == 0) {
        for (int i0 = (nslots - 1) & ~31; i0 >= 0; i0 -= 32) {   // (cnt becomes a countdown cursor)
            const int i = i0 + lane;
            const int e = i < nslots ? tb.tmp[i] >> 16 : -1;   // (-1 >> 16 == -1)
            const unsigned same = __match_any_sync(all, e);
            const int leader = __ffs(same) - 1;
            int base = 0;
            if (e >= 0 && lane == leader) {
                base = tb.cnt[e] - __popc(same);
                tb.cnt[e] = base;
            }
            base = __shfl_sync(all, base, leader);
            if (e >= 0) tb.slots[tb.off[e] + base + __popc(same & below)] = i;
        }
    }
    barrier();
}

// ---- expert-parallel MoE with peer stores: the push of a CTA's outputs ---------------------------------------------
//
// Called by every consumer thread after its tile loop (also after a failed wait). The CTA's outputs are then complete
// in this rank's y: segment sg's slots over the CTA's tiles [w0, w1) of that segment, one contiguous run of n per
// slot. After a barrier every consumer thread pushes them to the peers (p2p_push); after a second barrier thread 0's
// system-scope fence in p2p_finish releases the stores of every consumer thread (the producer warp stores nothing).
// Kept out of line, so that the tile loop's register allocation does not carry it.
template <typename OutT>
__device__ __noinline__ void qmv_moe_push(const QmvArgs& a, MoeTables tb, int w0, int w1, bool ok,
                                          volatile int* cta_failed) {
    if (threadIdx.x == 0) *cta_failed = 0;   // (set to 1 below by any consumer thread that gave up or skipped)
    named_sync(1, QMV_NW * 32);
    bool rd = ok;
    if ((threadIdx.x & 31) == 0 && rd) rd = p2p_wait_ready(a.pp, p2p_epoch(a.pp));
    rd = __shfl_sync(0xffffffffu, rd ? 1 : 0, 0) != 0;
    if (rd && w1 > w0) {
        const size_t rowp = (size_t)a.N * sizeof(OutT);
        for (int sg = fdiv(w0, a.dv_tiles); sg <= fdiv(w1 - 1, a.dv_tiles); ++sg) {
            const int ta = max(w0, sg * a.tilesN) - sg * a.tilesN;
            const int tb_ = min(w1, (sg + 1) * a.tilesN) - sg * a.tilesN;
            const int n0 = ta * QMV_ROWS, n1 = min(a.N, tb_ * QMV_ROWS);
            if (n1 <= n0) continue;
            const int first = tb.seg[sg] & 0xFFFF, cnt = tb.segc[sg];
            const size_t off0 = (size_t)n0 * sizeof(OutT);
            p2p_push(a.pp, cnt, (n1 - n0) * (int)sizeof(OutT), rowp | off0,
                     [&](int r) { return (size_t)tb.slots[first + r] * rowp + off0; }, threadIdx.x, QMV_NW * 32);
        }
    }
    if (!rd) *cta_failed = 1;
    named_sync(1, QMV_NW * 32);
    if (threadIdx.x == 0) p2p_finish(a.pp, *cta_failed == 0);
}

// ---- the kernel ---------------------------------------------------------------------------------------------------
//
// The consumer warps form WG groups of QMV_NW / WG warps. Group j takes every WG-th tile of the CTA's range (tiles
// are independent), so WG tiles are in flight at once and each tile's partial sums are reduced over QMV_NW / WG warps
// only. The plan sets WG (up to 4); for MoE the host caps it at the most tiles a CTA can get from the call's slot
// count (at one token a CTA holds one or two 16-row tiles, and a tile's latency is each warp's chain of dependent
// MMAs over its share of K, so one tile is best split over all 16 warps). The host keeps nstage >= WG * nchunks: a group then never waits on a ring slot more than one phase ahead of that
// slot's last completed phase, which is all an mbarrier parity wait can tell apart.
//
// Barrier block layout (uint64 slots from bar_off): full[nstage], empty[nstage], xfull[2], xempty[2],
// redfull[2 * QMV_MAXWG], redfree[2 * QMV_MAXWG], gfull[2], gfree[2], and one word of CTA state (the MoE peer-store
// failure flag). The reduction region holds 2 * QMV_NW * 32
// float4 (plus 2 x 32 float4 of gate hand-over slots for QMV_GLU).
constexpr int QMV_MAXWG = 4;
__host__ __device__ constexpr int qmv_nbars(int nstage) { return 2 * nstage + 4 + 4 * QMV_MAXWG + 4 + 1; }

// MINB: CTAs per SM the register budget is sized for. 2 (56 registers a thread) lets the next call's CTA share the SM
// under PDL (its weight prefetch); calls planned with one CTA per SM -- most dense fp16-in calls, and MoE calls, which
// cannot start before their dependency anyway (the index list decides the weights) -- use MINB = 1: no spills, and
// registers for four MMA chains per loop iteration (measured on B200: 8 experts of 512x2048, 8 tokens 13.7 us against
// 14.7; dense 12288x2560 Q4 1 token 8.0 us against 9.1).
// XF32: the activations arrive as fp32 (the reference's fp32-in decode entry). The consumer warps stage every dense
// and gate/up call's activations themselves after the dependency wait; these they round to fp16 on the way (round to
// nearest even, the reference's conversion): no conversion launch, no extra shared memory, and the MMA path is the
// fp16 one.
// XB: a dense fp16-in call whose activations come in by the producer's bulk copy (qmv_xstage_max).
// WR: a MoE call of 33..MOE_WARP_MAX slots, routed by one warp in 32-slot chunks (moe_route_warp). The host picks
// these instances by the slot count, so the others -- one-token calls among them -- keep their code without the
// chunked router (inlined into every MoE instance it cost ~0.04 us at one token on B200).
template <int F, int MODE, typename OutT, bool XF32 = false, int MINB = 2, bool XB = false, bool WR = false>
__global__ void __launch_bounds__(32 * (QMV_NW + 1), MINB)
qmv_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap ts, const __grid_constant__ QmvArgs a) {
    static_assert(!XF32 || MODE == QMV_DENSE || MODE == QMV_GLU, "fp32 activations: dense and gate/up calls");
    static_assert(!XB || (MODE == QMV_DENSE && !XF32), "bulk-copied activations: dense fp16-in calls");
    static_assert(MINB == 2 || (MODE != QMV_GLU && !XF32), "one-CTA register budget: dense fp16-in and MoE calls");
    static_assert(!WR || MODE == QMV_MOE, "chunked one-warp routing: MoE calls without peer stores");
    constexpr bool GLU = MODE == QMV_GLU;
    constexpr bool MOE = MODE == QMV_MOE || MODE == QMV_MOE_P2P;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* sm = smem_raw + pad;   // pointer arithmetic on the shared array keeps the shared address space
    uint8_t* ring = sm + a.ring_off;
    uint8_t* xbuf = sm + a.x_off;
    float4* red = reinterpret_cast<float4*>(sm + a.red_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + a.bar_off);
    uint64_t* full = bars;
    uint64_t* empty = bars + a.nstage;
    uint64_t* xfull = bars + 2 * a.nstage;
    uint64_t* xempty = xfull + 2;
    uint64_t* redfull = xfull + 4;
    uint64_t* redfree = redfull + 2 * QMV_MAXWG;
    uint64_t* gfull = redfree + 2 * QMV_MAXWG;   // QMV_GLU: gate sums handed over in slot 0 / 1
    uint64_t* gfree = gfull + 2;                 // QMV_GLU: the up reducer has taken them
    volatile int* cta_state = reinterpret_cast<volatile int*>(gfree + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KG = a.K / 32;

    pdl_trigger();   // the next call may start its weight prefetch now (it still waits for us before touching x, y)

    // barrier initialisation for wg warp groups (one thread; the CTA's barrier follows)
    auto init_bars = [&](int wg) {
        const int wpg = QMV_NW / wg;
        for (int i = 0; i < a.nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], wpg);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], QMV_NW);
        }
        for (int i = 0; i < 2 * wg; ++i) {
            mbar_init(&redfull[i], wpg);
            mbar_init(&redfree[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&gfull[i], 1);
            mbar_init(&gfree[i], 1);
        }
        fence_mbar_init();
    };
    // the CTA's tiles [w0, w1) of nseg segments x tilesN tiles; gate/up tiles are split in whole pairs
    auto cta_range = [&](int nseg, int& w0, int& w1) {
        const int total = nseg * a.tilesN;
        const unsigned units = GLU ? total / 2 : total, ustep = GLU ? 2 : 1, b = blockIdx.x, n = gridDim.x;
        if ((unsigned long long)units * n < 0x80000000ull) {
            w0 = (int)ustep * fdiv((int)(b * units), a.dv_grid);
            w1 = (int)ustep * fdiv((int)((b + 1) * units), a.dv_grid);
        } else {
            w0 = (int)(ustep * (unsigned)(((unsigned long long)b * units) / n));
            w1 = (int)(ustep * (unsigned)(((unsigned long long)(b + 1) * units) / n));
        }
    };
    MoeTables tb{};
    if constexpr (MOE) {
        // the producer warp: barriers, then -- after the dependency, since the previous grid may have written the
        // index list and the activations -- the resident token rows. Up to 32 slots (up to MOE_WARP_MAX in the WR
        // instances) it also builds the routing tables alone and goes on to the weight stream while the consumers
        // wait for them; more slots are routed by the whole CTA.
        const int nslots = a.T * a.topk;
        constexpr int WMAX = WR ? MOE_WARP_MAX : 32;   // the most slots one warp routes
        tb = moe_tables(sm + a.moe_off, a.E_local, nslots);
        if (warp == QMV_NW) {
            if (lane == 0) {
                prefetch_tmap(&tq);   // (the descriptors' fetch overlaps the dependency wait and the routing)
                prefetch_tmap(&ts);
                init_bars(a.wg);
            }
            pdl_wait();
            if (lane == 0 && a.xres) {
                mbar_arrive_expect_tx(&xfull[0], (uint32_t)(a.T * a.K * 2));
                for (int j = 0; j < a.T; ++j)
                    bulk_load(xbuf + j * a.xpitch, a.x + (size_t)j * a.K, (uint32_t)(a.K * 2), &xfull[0]);
            }
            if (nslots <= 32) moe_route_small(a, tb, lane, nslots);
            else if constexpr (WMAX > 32) { if (nslots <= WMAX) moe_route_warp(a, tb, lane, nslots); }
        } else if (nslots > WMAX) {
            pdl_wait();
        }
        if (nslots <= WMAX) {
            // one warp routed (moe_route_small, moe_route_warp): the producer goes on to the weight stream at once
            if (warp == QMV_NW) named_arrive(2, 32 * (QMV_NW + 1));
            else named_sync(2, 32 * (QMV_NW + 1));
        } else {
            moe_route_cta(a, tb, nslots, [] { __syncthreads(); });
        }
    } else {
        if (threadIdx.x == 0) init_bars(a.wg);
        __syncthreads();
    }

    int nseg = 1;
    if constexpr (MOE) nseg = *tb.nseg;
    int w0, w1;
    cta_range(nseg, w0, w1);
    const int ntl = w1 - w0;   // tiles of this CTA
    const int WG = a.wg;                    // 1, 2 or 4
    const int wpg_log = 5 - __ffs(WG);      // WPG = 16 / WG = 1 << wpg_log
    const int WPG = 1 << wpg_log;
    const bool xres = MOE && a.xres != 0;

    // segment accessors: expert (weight row base), token count, and the slot (dense: token) of column j
    auto seg_expert = [&](int sg) -> int {
        if constexpr (MOE) return tb.seg[sg] >> 16; else return 0;
    };
    auto seg_first = [&](int sg) -> int {
        if constexpr (MOE) return tb.seg[sg] & 0xFFFF; else return 0;
    };
    auto seg_count = [&](int sg) -> int {
        if constexpr (MOE) return tb.segc[sg];
        else return a.T;
    };
    auto seg_slot = [&](int sg, int j) -> int {
        if constexpr (MOE) return tb.slots[seg_first(sg) + j]; else return j;
    };

    // dense and gate/up calls: the consumers load the activations themselves (see their staging), unless XB
    constexpr bool xdirect = !MOE && !XB;

    constexpr int BITS = FmtTraits<F>::BITS;
    const int ksb = a.KS * BITS / 8;                                          // code bytes per row per stage
    const uint32_t stage_tx = (uint32_t)(QMV_ROWS * (a.cpitch + a.spitch));   // both boxes, pads included

    if (warp == QMV_NW) {
        // ===================== producer (one thread) =====================
        if (lane == 0) {
            if constexpr (!MOE) {   // (MoE: prefetched in the prologue, before the dependency wait)
                prefetch_tmap(&tq);
                prefetch_tmap(&ts);
            }
            const int total_it = ntl * a.nchunks;
            const int pre = min(total_it, a.nstage);
            // iteration cursor: chunk c of tile `tile` of segment `sg`; ring slot stg in round rnd
            int c = 0, sg = fdiv(w0, a.dv_tiles), tile = w0 - sg * a.tilesN, stg = 0, rnd = 0, issued = 0;
            auto issue_w = [&]() {
                uint8_t* st = ring + stg * a.stage_bytes;
                uint64_t* fb = &full[stg];
                const int row = GLU ? ((tile & 1) ? a.N : 0) + (tile >> 1) * QMV_ROWS    // gate / up tile pair
                                    : seg_expert(sg) * a.N + tile * QMV_ROWS;
                mbar_arrive_expect_tx(fb, stage_tx);
                tma_load_2d(st, &tq, c * ksb / 8, row, fb);                              // 8-byte elements
                tma_load_2d(st + QMV_ROWS * a.cpitch, &ts, c * (a.KS / 32), row, fb);  // fp16 elements
                ++issued;
                if (++c == a.nchunks) {
                    c = 0;
                    if (++tile == a.tilesN) { tile = 0; ++sg; }
                }
                if (++stg == a.nstage) { stg = 0; ++rnd; }
            };
            int xsegs = xres ? 1 : 0;   // activation copies issued (resident rows: the one of the prologue)
            bool ok = true;
            auto issue_x = [&](int xs) {   // activations of the next segment this CTA meets, double-buffered
                if (xres) return;          // (resident rows: already on their way)
                const int xb = xsegs & 1;
                if (xsegs >= 2) ok = wait_parity(&xempty[xb], ((xsegs >> 1) - 1) & 1);
                if (!ok) return;
                const int cnt = seg_count(xs);
                uint8_t* dst = xbuf + xb * a.xrows * a.xpitch;
                mbar_arrive_expect_tx(&xfull[xb], (uint32_t)(cnt * a.K * 2));
                for (int j = 0; j < cnt; ++j) {
                    int tok = seg_slot(xs, j);
                    if constexpr (MOE) tok /= a.topk;
                    bulk_load(dst + j * a.xpitch, a.x + (size_t)tok * a.K, (uint32_t)(a.K * 2), &xfull[xb]);
                }
                ++xsegs;
            };
            if constexpr (xdirect) {
                // the activations into L2 while the previous grid runs (see bulk_prefetch_l2), each 128-byte line by
                // one CTA: every CTA prefetching all of them cost more L2 bandwidth than the latency saved. Measured
                // on B200 (50-call graphs, weights cycled over 4x L2): 8192x2048 Q4 1 token 4.40 -> 3.97 us; the
                // configs[1] cases unchanged in sum, larger blocks (the XB kernels) 1.5-2% slower, so not there
                // either
                const uint32_t total = (uint32_t)(a.T * a.K * (XF32 ? 4 : 2));
                const uint32_t piece = ((total + gridDim.x - 1) / gridDim.x + 127u) & ~127u;
                const uint32_t off = blockIdx.x * piece;
                if (off < total)
                    bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(a.x) + off, min(piece, total - off));
            }
            for (int i = 0; i < pre; ++i) issue_w();   // the weights do not depend on the previous grid
            pdl_wait();                                // the activations may
            // activations of the segments the prefetched stages belong to, in order
            int last_seg = -1;
            {
                int xsg = fdiv(w0, a.dv_tiles), xtile = w0 - xsg * a.tilesN;
                for (int it = 0; it < pre && ok; it += a.nchunks) {
                    if (xsg != last_seg) {
                        if (!xdirect) issue_x(xsg);   // (else the consumers load the activations)
                        last_seg = xsg;
                    }
                    if (++xtile == a.tilesN) { xtile = 0; ++xsg; }
                }
            }
            for (int it = pre; it < total_it && ok; ++it) {
                if (c == 0 && sg != last_seg) {   // (dense and gate/up calls have one segment)
                    if (MOE) issue_x(sg);
                    last_seg = sg;
                    if (!ok) break;
                }
                ok = wait_parity(&empty[stg], (rnd - 1) & 1);
                if (!ok) break;
                issue_w();
            }
            // drain: every copy this CTA issued lands before the CTA may exit (bounded as well)
            {
                int dstg = 0, drnd = 0;
                for (int it = 0; it < issued; ++it) {
                    if (it >= issued - a.nstage &&
                        !wait_parity(&full[dstg], drnd & 1, DEV_ERR_DRAIN_TIMEOUT))
                        break;
                    if (++dstg == a.nstage) { dstg = 0; ++drnd; }
                }
            }
            for (int j = max(0, xsegs - 2); j < xsegs; ++j)
                if (!wait_parity(&xfull[j & 1], (j >> 1) & 1, DEV_ERR_DRAIN_TIMEOUT)) break;
        }
        return;
    }

    // ===================== consumers (warps 0..NW-1, WG groups) =====================
#ifndef VKB_QMV_SLEEP
#define VKB_QMV_SLEEP 1
#endif
    constexpr bool SLEEP = VKB_QMV_SLEEP == 2 || (VKB_QMV_SLEEP == 1 && MOE);
    auto cwait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if constexpr (SLEEP) return wait_parity_sleep(bar, parity); else return wait_parity(bar, parity);
    };
    const int grp = warp >> wpg_log, wi = warp & (WPG - 1);
    const int g = lane >> 2, t = lane & 3;
    const int GS = a.KS / 32;
    const int G0 = (wi * GS) >> wpg_log, G1w = ((wi + 1) * GS) >> wpg_log;
    const uint32_t cp = (uint32_t)a.cpitch, sp = (uint32_t)a.spitch;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t xbuf_s = smem_u32(xbuf);
    const uint32_t c_row = g * cp;                                       // row g's codes inside a stage
    const uint32_t s_row = (uint32_t)(QMV_ROWS * a.cpitch) + g * sp;     // row g's scales inside a stage
    OutT* y = reinterpret_cast<OutT*>(a.y);
    // x and y may still be written (or y read) by the previous grid. MoE: the producer's wait, which the consumers
    // are ordered after by the routing barrier, has already established that for the whole grid.
    if constexpr (!MOE) pdl_wait();
    if constexpr (xdirect) {
        // dense and gate/up calls: the consumers stage the token rows themselves, in fragment order (frag_order), so
        // that every group's B registers are one 16-byte load; fp32 activations are rounded to fp16 on the way (round
        // to nearest even, the reference's conversion). Items = (token, 16-byte chunk) pairs over the consumer
        // threads, coalesced; each thread keeps R items' loads in flight (one round for the blocks of each instance:
        // up to 16384 values under the two-CTA budget, 32768 under the one-CTA budget). Then
        // one barrier. (Measured on B200 against the producer's bulk copy with the permutation in every group's load:
        // 8192x2048 Q4 1 token 4.6 -> 4.1-4.4 us.)
        constexpr int R = XF32 ? 4 : (MINB == 1 ? 8 : 4);
        const int nch = a.K / 8, items = a.T * nch;
        int m = 0, c = threadIdx.x;   // item threadIdx.x: token m, chunk c
        while (c >= nch) { c -= nch; ++m; }
        for (int i = threadIdx.x; i < items; i += R * QMV_NW * 32) {
            uint32_t dst[R];
            uint2 lo[R], hi[R];
            float4 f0[XF32 ? R : 1], f1[XF32 ? R : 1];
#pragma unroll
            for (int r = 0; r < R; ++r) {   // the loads
                dst[r] = 0xFFFFFFFFu;
                if (i + r * QMV_NW * 32 < items) {
                    const int e0 = chunk_src<F>(c), e1 = e0 + chunk_hi<F>();
                    dst[r] = xbuf_s + (uint32_t)(m * a.xpitch + 16 * c);
                    if constexpr (XF32) {
                        const float* row = reinterpret_cast<const float*>(a.x) + (size_t)m * a.K;
                        f0[r] = __ldcg(reinterpret_cast<const float4*>(row + e0));
                        f1[r] = __ldcg(reinterpret_cast<const float4*>(row + e1));
                    } else if constexpr (F == FMT_Q2) {
                        const __half* row = a.x + (size_t)m * a.K;
                        lo[r] = __ldcg(reinterpret_cast<const uint2*>(row + e0));
                        hi[r] = __ldcg(reinterpret_cast<const uint2*>(row + e1));
                    } else {   // (e1 = e0 + 4: one 16-byte load)
                        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(a.x + (size_t)m * a.K + e0));
                        lo[r] = make_uint2(v.x, v.y);
                        hi[r] = make_uint2(v.z, v.w);
                    }
                    c += QMV_NW * 32;
                    while (c >= nch) { c -= nch; ++m; }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {   // fragment order and the stores
                if (dst[r] == 0xFFFFFFFFu) continue;
                if constexpr (XF32) {
                    lo[r] = make_uint2(cvt_h2(__float_as_uint(f0[r].x), __float_as_uint(f0[r].y)),
                                       cvt_h2(__float_as_uint(f0[r].z), __float_as_uint(f0[r].w)));
                    hi[r] = make_uint2(cvt_h2(__float_as_uint(f1[r].x), __float_as_uint(f1[r].y)),
                                       cvt_h2(__float_as_uint(f1[r].z), __float_as_uint(f1[r].w)));
                }
                sts128(dst[r], frag_order<F>(lo[r], hi[r]));
            }
        }
        named_sync(1, QMV_NW * 32);
    }
    if constexpr (MODE == QMV_MOE_P2P) {   // peer stores: this rank's copy may be written from now on
        if (warp == 0 && lane == 0) p2p_post_ready(a.pp, p2p_epoch(a.pp));
    }
    if constexpr (MOE) {
        if (a.zero_foreign) {   // another rank computes these slots; the combine adds this rank's zeros to them
            const int nslots = a.T * a.topk;
            for (int i = blockIdx.x; i < nslots; i += gridDim.x) {
                const int e = __ldg(a.idx + i) - a.e0;
                if (e >= 0 && e < a.E_local) continue;
                for (int n = threadIdx.x; n < a.N; n += QMV_NW * 32) y[(size_t)i * a.N + n] = to_out<OutT>(0.f);
            }
        }
    }

    // Activation segments of this CTA, in order: j = sg - first_seg. Every warp enters (waits xfull) and leaves (arrives
    // xempty) every segment exactly once and in order -- also the ones it has no tile in -- so that an arrival is
    // never counted towards an earlier use of the same double buffer.
    const int first_seg = fdiv(w0, a.dv_tiles);
    const int last_seg = ntl > 0 ? fdiv(w1 - 1, a.dv_tiles) : first_seg - 1;
    int jn = 0;            // next segment to enter
    bool held = false;     // holding segment jn - 1
    int cnt = 0;
    uint32_t xrow = 0;
    bool ok = true;
    auto leave = [&]() {
        if (held) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&xempty[(jn - 1) & 1]);
            held = false;
        }
    };
    auto enter_upto = [&](int j_target) -> bool {   // hold segment j_target, passing through the ones before it
        while (jn <= j_target) {
            leave();
            if (!cwait(&xfull[jn & 1], (jn >> 1) & 1)) return false;
            held = true;
            ++jn;
        }
        return true;
    };
    // this group's tiles: tl = grp, grp + WG, ...; their first stage iteration is tl * nchunks
    int sg = fdiv(w0 + grp, a.dv_tiles), tile = w0 + grp - sg * a.tilesN;
    int stg = 0, rnd = 0;
    {
        const int it0 = grp * a.nchunks;   // the first iteration of this group (no division in the loop)
        stg = it0;
        while (stg >= a.nstage) { stg -= a.nstage; ++rnd; }
    }
    int ntile = 0;   // tiles this group has done (reduction buffer parity / reducer rotation)
    for (int tl = grp; tl < ntl && ok; tl += WG, ++ntile) {
        if (sg - first_seg != jn - 1 || !held) {
            if (xdirect) {   // staged by the consumers above, before their barrier
                held = true;
                jn = 1;
            } else if (xres) {   // resident token rows: wait for them once
                if (!held && !cwait(&xfull[0], 0)) { ok = false; break; }
                held = true;
                jn = sg - first_seg + 1;
            } else if (!enter_upto(sg - first_seg)) {
                ok = false;
                break;
            }
            const int xb = xres ? 0 : (jn - 1) & 1;
            cnt = seg_count(sg);
            const int col = g < cnt ? g : 0;
            int xr = col;   // staged row of this thread's column
            if constexpr (MOE) if (xres) xr = fdiv(seg_slot(sg, col), a.dv_topk);
            xrow = xbuf_s + (uint32_t)((xb * a.xrows + xr) * a.xpitch) + x_lane_off<F, xdirect>(t);
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int kc = 0;
        for (int c = 0; c < a.nchunks; ++c, kc += GS) {
            if (!cwait(&full[stg], rnd & 1)) { ok = false; break; }
            const uint32_t st = ring_s + (uint32_t)(stg * a.stage_bytes);
            const int G1 = min(G1w, KG - kc);
            // four groups per iteration with the one-CTA register budget and in dense calls (measured on B200 under
            // the 56-register cap: 8192x2048 Q4 1 token 4.59 -> 4.44 us; two groups stay for gate/up, whose two-
            // and four-token calls got 8% slower, and for two-CTA MoE)
            constexpr int U = (MINB == 1 || MODE == QMV_DENSE) ? 4 : 2;
            const uint32_t xa = xrow + (uint32_t)(kc * 64);
            consume_stage<F, U, xdirect>(st + c_row, cp, st + s_row, sp, G0, G1, xa, t, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stg]);
            if (++stg == a.nstage) { stg = 0; ++rnd; }
        }
        if (!ok) break;
        // reduction over the group's warps (double-buffered, bounded mbarrier handshakes); the reducer rotates
        const int tp = ntile & 1, use = ntile >> 1, reducer = ntile & (WPG - 1);
        uint64_t* rfull = &redfull[grp * 2 + tp];
        uint64_t* rfree = &redfree[grp * 2 + tp];
        float4* rb = red + ((grp * 2 + tp) * WPG) * 32;
        if (use > 0 && !cwait(rfree, (use - 1) & 1)) { ok = false; break; }
        rb[wi * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncwarp();
        if (lane == 0) mbar_arrive(rfull);
        if (wi == reducer) {
            if (!cwait(rfull, use & 1)) { ok = false; break; }
            float4 r = rb[lane];
            for (int v = 1; v < WPG; ++v) {
                const float4 q = rb[v * 32 + lane];
                r.x += q.x; r.y += q.y; r.z += q.z; r.w += q.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(rfree);
            const int n0 = (GLU ? (tile >> 1) : tile) * QMV_ROWS + g, n1 = n0 + 8;
            const float vals[4] = {r.x, r.y, r.z, r.w};
            if constexpr (GLU) {
                // tile pair pl of the CTA: the gate half (even local tile) hands its sums over in slot pl & 1, the up
                // half takes them, frees the slot and writes out = silu(gate) * up (the reference's swiglu_split)
                const int pl = tl >> 1, slot = pl & 1, su = pl >> 1;
                float4* xs = red + 2 * QMV_NW * 32 + slot * 32;
                if (!(tl & 1)) {
                    if (su > 0 && !wait_parity(&gfree[slot], (su - 1) & 1)) { ok = false; break; }
                    xs[lane] = r;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&gfull[slot]);
                    if (a.ys) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int col = 2 * t + (q & 1);
                            const int n = (q < 2) ? n0 : n1;
                            if (col < cnt && n < a.N) a.ys[(size_t)col * 2 * a.N + n] = vals[q];
                        }
                    }
                } else {
                    if (!wait_parity(&gfull[slot], su & 1)) { ok = false; break; }
                    const float4 gg = xs[lane];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&gfree[slot]);
                    const float gv[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int col = 2 * t + (q & 1);
                        const int n = (q < 2) ? n0 : n1;
                        if (col < cnt && n < a.N) {
                            if (a.ys) a.ys[(size_t)col * 2 * a.N + a.N + n] = vals[q];
                            y[(size_t)col * a.N + n] = to_out<OutT>(gv[q] / (1.f + __expf(-gv[q])) * vals[q]);
                        }
                    }
                }
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int col = 2 * t + (q & 1);
                    const int n = (q < 2) ? n0 : n1;
                    if (col < cnt && n < a.N) y[(size_t)seg_slot(sg, col) * a.N + n] = to_out<OutT>(vals[q]);
                }
            }
        }
        // next tile of this group: WG tiles further; its first iteration is (WG - 1) * nchunks stages further
        tile += WG;
        while (tile >= a.tilesN) { tile -= a.tilesN; ++sg; }
        stg += (WG - 1) * a.nchunks;
        while (stg >= a.nstage) { stg -= a.nstage; ++rnd; }
    }
    // release the rest of the CTA's segments (also those this group had no tile in)
    if (!xdirect && !xres) {
        if (ok) ok = enter_upto(last_seg - first_seg);
        leave();
    }
    if constexpr (MODE == QMV_MOE_P2P) qmv_moe_push<OutT>(a, tb, w0, w1, ok, cta_state);
}

}  // namespace vkb
