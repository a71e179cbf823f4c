// libvkb.so: the extern "C" entry points of include/vkb.h for the decode GEMV and MoE kernels, with argument
// validation, launch planning (stage width, ring depth, grid), TMA descriptor set-up and the status calls.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "../../include/vkb.h"
#include "qmv.cuh"
#include "qmv_simple.cuh"
#include "tc_gemm.cuh"
#include "vkb_internal.h"

namespace vkb {

VKB_STATUS_ACCESSOR(status_take_qmv)

StatusList status_accessors() {
    static const StatusTake list[] = {status_take_qmv, status_take_comm};
    return {list, list + sizeof(list) / sizeof(list[0])};
}

// ---- per-device facts, computed once ---------------------------------------------------------------------------

const DeviceInfo& device_info(int dev) {
    static DeviceInfo info[kMaxDevices];
    static std::once_flag once[kMaxDevices];
    std::call_once(once[dev], [dev] {
        DeviceInfo d{};
        cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        info[dev] = d;
    });
    return info[dev];
}

int current_device(int* dev) {
    const cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return -(int)e;
    if (*dev < 0 || *dev >= kMaxDevices) return VKB_EINVAL;
    return 0;
}

thread_local int t_pdl = -1;
// PDL is not used on the legacy NULL stream, whose implicit synchronisation with every other stream does not mix
// with programmatic serialisation; any created stream (or the per-thread default stream) gets it.
bool pdl_stream_ok(cudaStream_t st) { return st != nullptr && st != cudaStreamLegacy; }
bool pdl_enabled() {
    if (t_pdl < 0) {
        const char* e = getenv("VKB_PDL");
        t_pdl = (e && e[0] == '0') ? 0 : 1;
    }
    return t_pdl != 0;
}

// ---- TMA descriptors --------------------------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

struct MapKey {
    const void* ptr;
    uint64_t rows, row_bytes;
    uint32_t box0, box1, dtype, swz;
    bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        const uint64_t* w = reinterpret_cast<const uint64_t*>(&k);
        uint64_t h = 1469598103934665603ull;
        for (size_t i = 0; i < sizeof(MapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
        return (size_t)h;
    }
};

// A 2-D row-major tensor of `rows` x `row_bytes` (elements of dtype), boxes of box0 elements x box1 rows. Cached per
// host thread (weights are long-lived; a pointer that is freed and reused for a same-shaped tensor gets the same,
// still valid, descriptor).
int get_tmap_2d(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t row_bytes, CUtensorMapDataType dtype,
                uint32_t elem_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz) {
    thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    MapKey key{};
    key.ptr = ptr; key.rows = rows; key.row_bytes = row_bytes; key.box0 = box0; key.box1 = box1;
    key.dtype = (uint32_t)dtype; key.swz = (uint32_t)swz;
    auto it = cache.find(key);
    if (it != cache.end()) { *out = it->second; return 0; }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return -(int)cudaErrorNotSupported;
    cuuint64_t dims[2] = {row_bytes / elem_bytes, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box0, box1};
    cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    const CUresult r = enc(&m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -(int)cudaErrorInvalidValue;
    if (cache.size() > 65536) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return 0;
}

// Activations x [M][K] fp16 as a 3-D tensor {64 k, M tokens, K/64 k-blocks} (strides 2K and 128 bytes), boxes of
// {64, NT, XK} with 128-byte swizzle: one copy lands XK consecutive K-major UMMA B tiles of NT x 64. Cached per host
// thread like get_tmap_2d.
int get_tmap_x3d(CUtensorMap* out, const void* x, int M, int K, int NT, int XK) {
    struct Key {
        const void* p;
        int M, K, NT, XK;
        bool operator==(const Key& o) const { return p == o.p && M == o.M && K == o.K && NT == o.NT && XK == o.XK; }
    };
    struct Hash {
        size_t operator()(const Key& k) const {
            return std::hash<const void*>()(k.p) ^ ((size_t)k.M * 1000003u) ^ ((size_t)k.K << 20) ^
                   ((size_t)k.NT << 40) ^ ((size_t)k.XK << 52);
        }
    };
    thread_local std::unordered_map<Key, CUtensorMap, Hash> cache;
    const Key key{x, M, K, NT, XK};
    auto it = cache.find(key);
    if (it != cache.end()) { *out = it->second; return 0; }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return -(int)cudaErrorNotSupported;
    cuuint64_t dims[3] = {64, (cuuint64_t)M, (cuuint64_t)(K / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)K * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)NT, (cuuint32_t)XK};
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap m;
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(x), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -(int)cudaErrorInvalidValue;
    if (cache.size() > 65536) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return 0;
}

// ---- decode / MoE planning ---------------------------------------------------------------------------------------

static int fmt_bits(int fmt) { return fmt == VKB_FMT_Q4 ? 4 : fmt == VKB_FMT_Q8 ? 8 : 2; }

struct QmvPlan {
    QmvArgs a;
    int smem;
    int grid;
};

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Stage: 16 rows x KS values, up to 1.5 KB of codes per row (one TMA box each for codes and scales, rows padded so
// the fragment reads are conflict free); ring as deep as fits, preferring a footprint that lets a second CTA (the
// next call, under PDL) share the SM when that still leaves at least 4 stages. The two-CTA footprint pays only while
// the previous call's CTA can share the SM as well: after a one-CTA call its shallow ring streams the weights without
// the head start. Measured on B200 (bench.py, the configs[1] graph of 48 different calls): minimum 3 stages 1385 GB/s,
// 4 stages 1487 GB/s, one CTA always 1622 GB/s; one shape repeated (8192x2048 Q4, 1 token): 4.7 / 4.7 / 5.8 us. 4 keeps the
// repeated-call time and takes part of the chain gain.
// glu: gate/up tile pairs over a [2N][K] table (N output rows, 2 ceil(N / 16) tiles, the gate hand-over slots after
// the reduction region).
static bool plan_qmv(int fmt, int N, int K, int xrows, int moe_slots, int E_local, const DeviceInfo& d, QmvPlan* p,
                     bool glu = false, bool xres = false, bool dense = false) {
    const int bits = fmt_bits(fmt), unit = QMV_KS_UNIT;
    static const int ks_force = getenv("VKB_QMV_KSMAX") ? atoi(getenv("VKB_QMV_KSMAX")) : 0;   // tuning override
    const int ks_max = ks_force >= unit ? ks_force : 12288 / bits;   // 1.5 KB of codes per row per stage (the
                                                                      // 8-byte box row limit is 2 KB)
    const int nchunks = (K + ks_max - 1) / ks_max;
    const int KS = round_up((K + nchunks - 1) / nchunks, unit);
    const int cpitch = KS * bits / 8 + (fmt == VKB_FMT_Q8 ? 32 : 16);
    const int spitch = KS / 16 + ((KS / 256) % 2 == 0 ? 16 : 32);   // pitch / 4 = 4 x odd: conflict-free rows
    const int stage_bytes = round_up(QMV_ROWS * (cpitch + spitch), 128);
    const int xpitch = round_up(K * 2, 128) + 64;
    const int xbufs = moe_slots > 0 && !xres ? 2 : 1;   // MoE over more than 8 tokens: per-segment rows, double-buffered
    const int xbytes = round_up(xbufs * xrows * xpitch, 16);
    const int redbytes = 2 * QMV_NW * 32 * 16 + (glu ? 2 * 32 * 16 : 0);
    const int moebytes = moe_slots > 0 ? round_up(4 * moe_table_words(E_local, moe_slots), 16) : 0;
    const int slack = 1024;
    auto fixed_for = [&](int nstage) { return 8 * qmv_nbars(nstage) + xbytes + redbytes + moebytes + slack; };
    const int pair_budget = d.smem_per_sm / 2 - 1024;   // two CTAs per SM
    const int solo_budget = d.smem_optin;
    static const int pair_min = getenv("VKB_QMV_PAIRMIN") ? atoi(getenv("VKB_QMV_PAIRMIN")) : 4;   // tuning override
    // dense fp16-in calls (`dense`): the two-CTA footprint only for one-stage tiles of K <= 2048 with more tiles than
    // SMs, the short calls whose next call's weight prefetch (under PDL, in the second CTA) is worth a shallow ring;
    // every other dense call takes one CTA per SM with the deepest ring and the kernel's 96-register variant
    // (measured on B200, configs[1] tables, 50 same-shape calls per graph: 12288x2560 Q4 1 token 8.0 us against 9.1,
    // 2048x6144 4.6 against 4.8, 6144x2048 Q4 4.4 against 4.0 -- the exception).
    const bool pair_first = !dense || (K <= 2048 && nchunks == 1 && (N + QMV_ROWS - 1) / QMV_ROWS > d.sm_count);
    int nstage = 0, budget = pair_budget;
    for (int pass = pair_first ? 0 : 1; pass < 2; ++pass) {
        budget = pass == 0 ? pair_budget : solo_budget;
        nstage = 16;
        while (nstage >= 2 && nstage * stage_bytes + fixed_for(nstage) > budget) --nstage;
        if (nstage >= pair_min || (pass == 1 && nstage >= 2)) break;
    }
    if (nstage < 2) return false;
    QmvArgs& a = p->a;
    a.N = N; a.K = K; a.KS = KS; a.nchunks = nchunks; a.nstage = nstage; a.stage_bytes = stage_bytes;
    a.cpitch = cpitch; a.spitch = spitch;
    a.xpitch = xpitch; a.xrows = xrows; a.xres = xres ? 1 : 0;
    a.tilesN = (glu ? 2 : 1) * ((N + QMV_ROWS - 1) / QMV_ROWS);
    a.dv_tiles = make_fastdiv((uint32_t)a.tilesN);
    a.dv_topk = make_fastdiv(1);
    a.ring_off = 0;
    a.x_off = nstage * stage_bytes;
    a.red_off = a.x_off + xbytes;
    a.bar_off = a.red_off + redbytes;
    a.moe_off = a.bar_off + 8 * qmv_nbars(nstage);
    // warp groups: as many tiles in flight as the ring allows (nstage >= wg * nchunks); MoE too (every warp passes
    // through every activation segment of its CTA in order, also those it has no tile in)
    const int nch_tile = nchunks;   // stages per tile
    a.wg = 1;
    for (int wg = QMV_MAXWG; wg > 1; wg /= 2)
        if (nstage >= wg * nch_tile) { a.wg = wg; break; }
    // dense calls with at most one or two row tiles per CTA: groups beyond the CTA's tiles would idle, so long rows
    // go to fewer, larger groups (measured on B200: K = 6144 over 128 tiles, 2-bit: 4.9 us with one group, 6.5 with
    // four)
    if (moe_slots == 0 && K >= 2048) {
        const int tiles = a.tilesN;
        if (tiles <= d.sm_count && K >= 4096) a.wg = 1;
        else if (tiles <= d.sm_count || (tiles <= 2 * d.sm_count && K >= 4096)) a.wg = a.wg < 2 ? a.wg : 2;
    }
    static const int wg_force = getenv("VKB_QMV_WG") ? atoi(getenv("VKB_QMV_WG")) : 0;   // tuning override
    if (wg_force == 1 || ((wg_force == 2 || wg_force == 4) && nstage >= wg_force * nch_tile)) a.wg = wg_force;
    p->smem = a.moe_off + moebytes + slack;
    return true;
}

template <int F, int MODE, typename OutT, bool XF32 = false, int MINB = 2, bool XB = false, bool WR = false>
static int launch_qmv(const QmvPlan& p, const CUtensorMap& tq, const CUtensorMap& ts, int grid, cudaStream_t st,
                      int dev) {
    auto kern = qmv_kernel<F, MODE, OutT, XF32, MINB, XB, WR>;
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr_err[kMaxDevices];
    std::call_once(once[dev], [&] {
        attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             device_info(dev).smem_optin);
    });
    if (attr_err[dev] != cudaSuccess) return -(int)attr_err[dev];
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * (QMV_NW + 1));
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() && pdl_stream_ok(st) ? 1 : 0;
    QmvArgs a = p.a;
    a.dv_grid = make_fastdiv((uint32_t)grid);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tq, ts, a);
    return e == cudaSuccess ? 0 : -(int)e;
}

template <int F, typename OutT>
static int launch_simple(const void* q, const void* s, const void* x, void* y, const int32_t* idx, int N, int K,
                         int M, int topk, int E_local, int e0, int zero_foreign, int slots, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() && pdl_stream_ok(st) ? 1 : 0;
    cudaError_t e;
    if (idx == nullptr) {
        cfg.gridDim = dim3((unsigned)((N + 7) / 8), 1);
        e = cudaLaunchKernelEx(&cfg, qmv_simple_kernel<F, OutT>, q, (const __half*)s, (const __half*)x, (OutT*)y, idx,
                               N, K, M, topk, E_local, e0, zero_foreign);
    } else {
        // the slot list of one expert in dynamic shared memory (slots x 4 bytes; the entry point caps slots at 32767)
        static std::once_flag once[kMaxDevices];
        static cudaError_t attr_err[kMaxDevices];
        int dev = 0;
        if (int r = current_device(&dev)) return r;
        std::call_once(once[dev], [&] {
            attr_err[dev] = cudaFuncSetAttribute(qmv_simple_moe_kernel<F, OutT>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * 32767 + 16);
        });
        if (attr_err[dev] != cudaSuccess) return -(int)attr_err[dev];
        cfg.gridDim = dim3((unsigned)((N + QMV_SIMPLE_MOE_ROWS - 1) / QMV_SIMPLE_MOE_ROWS),
                           (unsigned)(E_local + (zero_foreign ? 1 : 0)));
        cfg.dynamicSmemBytes = (size_t)slots * 4;
        e = cudaLaunchKernelEx(&cfg, qmv_simple_moe_kernel<F, OutT>, q, (const __half*)s, (const __half*)x, (OutT*)y,
                               idx, N, K, M, topk, E_local, e0, zero_foreign);
    }
    return e == cudaSuccess ? 0 : -(int)e;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Common body of the dense and MoE entry points.
template <int F>
static int qmv_entry(const void* q, const void* s, const void* x, void* y, bool f32, const int32_t* idx, int N, int K,
                     int M, int topk, int E_local, int e0, int zero_foreign, cudaStream_t st, const P2PArgs* p2p) {
    const bool moe = idx != nullptr;
    if (p2p && (!moe || zero_foreign)) return VKB_EINVAL;
    if (!q || !s || !x || !y) return VKB_EINVAL;
    if (N < 1 || K < 32 || M < 1) return VKB_EINVAL;
    if (K % 32 != 0) return VKB_EUNSUPPORTED;
    if (!moe && M > QMV_MAXTOK) return VKB_EUNSUPPORTED;
    if (moe && (topk < 1 || E_local < 1 || E_local > 32767 || (long long)M * topk > 32767)) return VKB_EUNSUPPORTED;
    if (F == FMT_Q2 && K % 64 != 0) return VKB_EUNSUPPORTED;
    const long long rows = moe ? (long long)E_local * N : N;
    if (rows > (1ll << 31) - 1) return VKB_EUNSUPPORTED;
    int dev = 0;
    if (int r = current_device(&dev)) return r;
    const DeviceInfo& d = device_info(dev);
    const int slots = moe ? M * topk : 0;

    const bool fast = K % 256 == 0 && aligned16(q) && aligned16(s) && aligned16(x);
    QmvPlan p{};
    // MoE over at most 8 tokens: every token row stays resident (columns index it by slot / topk); more tokens: the
    // rows of each expert segment (at most 8 slots) are staged in turn
    const bool xres = moe && M <= QMV_MAXTOK;
    const int xrows = moe && !xres ? (slots < QMV_MAXTOK ? slots : QMV_MAXTOK) : M;
    if (fast && plan_qmv(F, N, K, xrows, slots, E_local, d, &p, false, xres, !moe)) {
        constexpr int BITS = FmtTraits<F>::BITS;
        CUtensorMap tq, ts;
        int r = get_tmap_2d(&tq, q, (uint64_t)rows, (uint64_t)K * BITS / 8, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8,
                            (uint32_t)(p.a.cpitch / 8), QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (r) return r;
        r = get_tmap_2d(&ts, s, (uint64_t)rows, (uint64_t)K / 16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                        (uint32_t)(p.a.spitch / 2), QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (r) return r;
        p.a.x = (const __half*)x;
        p.a.y = y;
        p.a.idx = idx;
        p.a.T = M;
        p.a.topk = topk;
        if (moe) p.a.dv_topk = make_fastdiv((uint32_t)topk);
        p.a.E_local = E_local;
        p.a.e0 = e0;
        p.a.zero_foreign = zero_foreign;
        if (p2p) p.a.pp = *p2p;
        int grid;
        if (moe) {
            // The tile count is known only in the kernel; the host bounds it: segments <= n + (slots - n) / 8 with
            // n = min(E_local, slots) (each routed expert has ceil(c / 8) <= 1 + (c - 1) / 8 of them). One CTA per
            // SM, or two when two fit (the two-CTA footprint) and a CTA can get 4 or more tiles: twice the stages
            // in flight per SM (measured on B200, the 2048x512 down set: 1 token 5.3 us against 5.8, 8 tokens 18.1
            // against 23.4, 64 tokens 50 against 65), while calls of one or two tiles per CTA pay for the second
            // CTA's prologue (8 experts of 512x2048 at one token: 4.9 us against 4.4). Peer-store calls keep one per
            // SM (one flag pair per CTA).
            const long long n = E_local < slots ? E_local : slots;
            const long long tiles = (n + (slots - n) / QMV_MAXTOK) * p.a.tilesN;
            static const int per_sm_force = getenv("VKB_MOE_CTAS_PER_SM") ? atoi(getenv("VKB_MOE_CTAS_PER_SM")) : 0;
            const bool fits2 = 2 * (p.smem + 1024) <= d.smem_per_sm && !p2p;   // (1 KB reserved per CTA)
            const bool two = per_sm_force ? (per_sm_force == 2 && fits2) : (fits2 && tiles >= 4ll * d.sm_count);
            grid = d.sm_count * (two ? 2 : 1);   // (VKB_MOE_CTAS_PER_SM: tuning override)
            // warp groups: no more than the tiles a CTA can get, bounded without E_local or the grid (a segment per
            // slot, one CTA per SM): the groups set how a tile's K range is split over warps, so an expert-parallel
            // rank and one GPU holding every expert must pick the same number to produce the same bits
            const long long most = ((long long)slots * p.a.tilesN + d.sm_count - 1) / d.sm_count;
            while (p.a.wg > 1 && p.a.wg > most) p.a.wg /= 2;
        } else {
            grid = p.a.tilesN < d.sm_count ? p.a.tilesN : d.sm_count;
        }
        if (p2p && grid > P2P_MAX_CTAS) return VKB_EUNSUPPORTED;   // one flag pair per CTA
        if (moe) {
            if (p2p)   // one CTA per SM
                return f32 ? launch_qmv<F, QMV_MOE_P2P, float, false, 1>(p, tq, ts, grid, st, dev)
                           : launch_qmv<F, QMV_MOE_P2P, __half, false, 1>(p, tq, ts, grid, st, dev);
            if (slots > 32 && slots <= MOE_WARP_MAX) {   // routed by one warp in 32-slot chunks
                if (grid > d.sm_count)
                    return f32 ? launch_qmv<F, QMV_MOE, float, false, 2, false, true>(p, tq, ts, grid, st, dev)
                               : launch_qmv<F, QMV_MOE, __half, false, 2, false, true>(p, tq, ts, grid, st, dev);
                return f32 ? launch_qmv<F, QMV_MOE, float, false, 1, false, true>(p, tq, ts, grid, st, dev)
                           : launch_qmv<F, QMV_MOE, __half, false, 1, false, true>(p, tq, ts, grid, st, dev);
            }
            if (grid > d.sm_count)
                return f32 ? launch_qmv<F, QMV_MOE, float>(p, tq, ts, grid, st, dev)
                           : launch_qmv<F, QMV_MOE, __half>(p, tq, ts, grid, st, dev);
            return f32 ? launch_qmv<F, QMV_MOE, float, false, 1>(p, tq, ts, grid, st, dev)
                       : launch_qmv<F, QMV_MOE, __half, false, 1>(p, tq, ts, grid, st, dev);
        }
        if (2 * (p.smem + 1024) > d.smem_per_sm) {   // one CTA per SM: the 96-register variant
            if ((long long)M * K > qmv_xstage_max(F))    // activations by bulk copy
                return f32 ? launch_qmv<F, QMV_DENSE, float, false, 1, true>(p, tq, ts, grid, st, dev)
                           : launch_qmv<F, QMV_DENSE, __half, false, 1, true>(p, tq, ts, grid, st, dev);
            return f32 ? launch_qmv<F, QMV_DENSE, float, false, 1>(p, tq, ts, grid, st, dev)
                       : launch_qmv<F, QMV_DENSE, __half, false, 1>(p, tq, ts, grid, st, dev);
        }
        return f32 ? launch_qmv<F, QMV_DENSE, float>(p, tq, ts, grid, st, dev)
                   : launch_qmv<F, QMV_DENSE, __half>(p, tq, ts, grid, st, dev);
    }
    if (p2p) return VKB_EUNSUPPORTED;   // peer stores: the pipelined kernel only
    // general path: 4-byte aligned words for Q4/Q2, 2-byte aligned fp16
    if (F != FMT_Q8 && (reinterpret_cast<uintptr_t>(q) & 3u)) return VKB_EUNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 1u)
        return VKB_EUNSUPPORTED;
    return f32 ? launch_simple<F, float>(q, s, x, y, idx, N, K, M, topk, E_local, e0, zero_foreign, slots, st)
               : launch_simple<F, __half>(q, s, x, y, idx, N, K, M, topk, E_local, e0, zero_foreign, slots, st);
}

// fp32 activations -> fp16, round to nearest even (the reference's conversion step, used when the fp32 staging does
// not fit the decode kernel's shared memory). Ordered after the previous kernel like every call.
__global__ void __launch_bounds__(256) f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ xh, int n) {
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) xh[i] = __float2half_rn(x[i]);
}

static int launch_f32_to_f16(const float* x, void* xh, int n, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(256);
    cfg.gridDim = dim3((unsigned)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024));
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() && pdl_stream_ok(st) ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, f32_to_f16_kernel, x, (__half*)xh, n);
    return e == cudaSuccess ? 0 : -(int)e;
}

// Q4 decode with fp32 activations (x_f32) and/or gate + up + SwiGLU over a stacked [2N][K] table (glu; ys: the
// stacked products [M][2N] fp32, or null). The pipelined kernel reads fp32 activations itself and rounds them into
// its fp16 buffer; shapes it does not take (K % 256 != 0, unaligned buffers) convert into xh (M x K fp16,
// caller-owned) with one small kernel first, as the reference does, and run the general kernel (dense only: the fused
// gate/up needs the pipelined kernel).
static int qmv_q4_ext(const void* q, const void* s, const void* x, bool x_f32, void* xh, float* ys, void* y,
                      bool out_f32, bool glu, int N, int K, int M, cudaStream_t st) {
    if (!q || !s || !x || !y) return VKB_EINVAL;
    if (N < 1 || K < 32 || M < 1) return VKB_EINVAL;
    if (K % 32 != 0 || M > QMV_MAXTOK) return VKB_EUNSUPPORTED;
    const long long rows = glu ? 2ll * N : (long long)N;
    if (rows > (1ll << 31) - 1) return VKB_EUNSUPPORTED;
    if (!glu && !x_f32) return qmv_dispatch(VKB_FMT_Q4, q, s, x, y, out_f32, nullptr, N, K, M, 0, 0, 0, 0, st);
    int dev = 0;
    if (int r = current_device(&dev)) return r;
    const DeviceInfo& d = device_info(dev);
    QmvPlan p{};
    const bool fast = K % 256 == 0 && aligned16(q) && aligned16(s) && aligned16(x) &&
                      plan_qmv(VKB_FMT_Q4, N, K, M, 0, 0, d, &p, glu);
    if (!fast) {
        if (glu) return VKB_EUNSUPPORTED;   // nothing launched
        if (!xh) return VKB_EINVAL;
        if ((reinterpret_cast<uintptr_t>(xh) & 1u) || (reinterpret_cast<uintptr_t>(x) & 3u)) return VKB_EUNSUPPORTED;
        if (int r = launch_f32_to_f16((const float*)x, xh, M * K, st)) return r;
        return qmv_dispatch(VKB_FMT_Q4, q, s, xh, y, out_f32, nullptr, N, K, M, 0, 0, 0, 0, st);
    }
    CUtensorMap tq, ts;
    int r = get_tmap_2d(&tq, q, (uint64_t)rows, (uint64_t)K / 2, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8,
                        (uint32_t)(p.a.cpitch / 8), QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
    r = get_tmap_2d(&ts, s, (uint64_t)rows, (uint64_t)K / 16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                    (uint32_t)(p.a.spitch / 2), QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
    p.a.x = (const __half*)x;
    p.a.y = y;
    p.a.ys = glu ? ys : nullptr;
    p.a.T = M;
    const int units = glu ? p.a.tilesN / 2 : p.a.tilesN;   // gate/up tiles go to CTAs in whole pairs
    const int grid = units < d.sm_count ? units : d.sm_count;
    if (glu) {
        if (x_f32)
            return out_f32 ? launch_qmv<FMT_Q4, QMV_GLU, float, true>(p, tq, ts, grid, st, dev)
                           : launch_qmv<FMT_Q4, QMV_GLU, __half, true>(p, tq, ts, grid, st, dev);
        return out_f32 ? launch_qmv<FMT_Q4, QMV_GLU, float, false>(p, tq, ts, grid, st, dev)
                       : launch_qmv<FMT_Q4, QMV_GLU, __half, false>(p, tq, ts, grid, st, dev);
    }
    return out_f32 ? launch_qmv<FMT_Q4, QMV_DENSE, float, true>(p, tq, ts, grid, st, dev)
                   : launch_qmv<FMT_Q4, QMV_DENSE, __half, true>(p, tq, ts, grid, st, dev);
}

int qmv_dispatch(int fmt, const void* q, const void* s, const void* x, void* y, bool f32, const int32_t* idx, int N,
                 int K, int M, int topk, int E_local, int e0, int zero_foreign, cudaStream_t st, const P2PArgs* p2p) {
    switch (fmt) {
        case VKB_FMT_Q4:
            return qmv_entry<FMT_Q4>(q, s, x, y, f32, idx, N, K, M, topk, E_local, e0, zero_foreign, st, p2p);
        case VKB_FMT_Q8:
            return qmv_entry<FMT_Q8>(q, s, x, y, f32, idx, N, K, M, topk, E_local, e0, zero_foreign, st, p2p);
        case VKB_FMT_Q2:
            return qmv_entry<FMT_Q2>(q, s, x, y, f32, idx, N, K, M, topk, E_local, e0, zero_foreign, st, p2p);
        default: return VKB_EUNSUPPORTED;
    }
}

// ---- prompt GEMM (tcgen05) --------------------------------------------------------------------------------------

struct TcPlan {
    TcArgs a;
    int pk;     // K steps per packed chunk (kernel template argument)
    int cg;     // CTAs per tile: 1, or 2 (a cluster pair on 256-row tiles, tcgen05 cta_group::2)
    int rb;     // 128-row blocks per CTA tile: 1, or 2 (two accumulators sharing every activation stage)
    int smem;
    dim3 grid;
};

// Tile shape: rb row blocks of 128 weight rows x NT tokens (NT <= 256, a multiple of 16 above 128 tokens, else of
// 32; any multiple of 16 when forced); the persistent grid (one CTA per SM) walks ceil(tiles / grid) tiles per CTA.
// A K step costs 4 UMMAs per row block of (32 + 0.41 NT) cycles (measured in the kernel, A in TMEM) or the
// dequantisation floor, and a single-buffered accumulator exposes the epilogue once per extra tile. One block: two accumulators when NT <= 128 (the epilogue overlaps the next tile), A
// slots of 4 K steps (128 TMEM columns). Two blocks (VKB_TC_RB=2 only: it halves the activation stream, but measured
// slower at every shape of the sweep, e.g. 12288x2560 at 512 tokens 34.0 vs 32.7 us, 8192x2048 24.5 vs 16.2 us):
// one accumulator per block, A slots of one K step for both blocks (64 columns) in the rest. Ring depths: X stages of
// up to 32 KB (an even count: two producers), P chunks of 8 K steps when they fit (else 4; 4 with two blocks), both
// deepened while shared memory lasts. With cg = 2 the units are CTA pairs (at most `units_max` co-resident), a tile
// has 256 rows and each CTA's X stages hold half of the tile's tokens.
//
// Split-K (split_max > 1: one-CTA tiles, no peer stores unless the row split asks for its exact count): with few tiles the MMAs of one tile's K range are the
// whole call (2560x6144 at 512 tokens: 40 tiles on 148 SMs), so S CTAs of a cluster share a tile, each taking units
// of TC_KUNIT K steps, at one tile per cluster (tiles x S <= SMs, and <= the clusters of S that fit at once:
// clusters_max[S], or SMs / S when null). Cost: the longest share's K steps, plus the partial exchange (shared
// memory stores of the accumulator, two cluster barriers, distributed shared-memory reads of ntok / S tokens of
// every rank: ~2000 + 12 NT cycles).
constexpr int TC_KUNIT = 8;
static bool plan_tc(int N, int K, int M, int out_bytes, const DeviceInfo& d, TcPlan* p, int cg, int units_max,
                    int wf = 0, bool allow_rb2 = false, int split_max = 1, const int* clusters_max = nullptr,
                    int split_exact = 0) {
    TcArgs& a = p->a;
    const int nk = K / TC_BK;
    int NT = 0, RB = 1, SPL = 1;
    double best = 1e300;
    static const int split_env = getenv("VKB_TC_SPLIT") ? atoi(getenv("VKB_TC_SPLIT")) : 0;   // tuning override
    if (cg != 1 || nk % TC_KUNIT != 0 || split_env == 1) split_max = 1;   // (VKB_TC_SPLIT=1: none)
    int split_force = split_max > 1 ? split_env : 0;
    if (split_exact > 0) {   // exactly this split (a row split matching the whole problem's plan): no overrides
        split_max = split_exact;
        split_force = split_exact;
    }
    const int nt_max = round_up(M, 32) < 256 ? round_up(M, 32) : 256;
    static const int nt_force = getenv("VKB_TC_NT") ? atoi(getenv("VKB_TC_NT")) : 0;   // tuning overrides
    static const int rb_force = getenv("VKB_TC_RB") ? atoi(getenv("VKB_TC_RB")) : 0;
    const int rb = rb_force == 2 && allow_rb2 && cg == 1 && wf == 0 ? 2 : 1;
    for (int pass = 0; pass < 3 && NT == 0; ++pass) {   // pass 1: without the NT override (it does not fit); pass 2:
        if (pass == 2 && split_exact == 0) split_force = 0;   // without the split override either
        // steps of 16 above 128 tokens (512 = 3 x 176 wastes 3 % of the MMAs, 3 x 192 11 %; measured 1 % faster),
        // of 32 below (48-token tiles were slower than 64 at 6144x2048 x 128 tokens: more passes over the weights)
        for (int nt = nt_max; nt >= 32; nt -= ((pass == 0 && nt_force > 0) || nt > 128) && cg == 1 ? 16 : 32) {
            if (pass == 0 && nt_force > 0 && nt != nt_force) continue;
            if (rb == 2 && round_up(round_up(nt, 32) + nt, 64) > 384) continue;   // two accumulators, two A slots
            const long tiles = (long)((N + TC_BM * rb * cg - 1) / (TC_BM * rb * cg)) * ((M + nt - 1) / nt);
            const long grid = tiles < units_max ? tiles : units_max;
            const long per_cta = (tiles + grid - 1) / grid;
            const double umma = 4.0 * rb * (32.0 + 0.41 * nt);
            const double step = umma > 180.0 * rb ? umma : 180.0 * rb;
            const double epi = nt <= 128 && rb == 1 ? 0.0 : 1500.0 + 10.0 * nt * rb;
            const double t = (double)per_cta * nk * step + (double)(per_cta - 1) * epi + 6000.0;
            if (t < best * 0.999 && split_force <= 1) { best = t; NT = nt; RB = rb; SPL = 1; }
            if (rb != 1) continue;
            const int nun = nk / TC_KUNIT;
            for (int sp = 2; sp <= split_max && sp <= 8 && sp <= nun; ++sp) {
                if (split_force > 1 && sp != split_force) continue;
                const long fit = clusters_max ? clusters_max[sp] : d.sm_count / sp;
                if (tiles * sp > d.sm_count || tiles > fit) continue;
                const double ts = (double)((nun + sp - 1) / sp) * TC_KUNIT * step + 6000.0 + 2000.0 + 12.0 * nt;
                if (ts < best * 0.999) { best = ts; NT = nt; RB = 1; SPL = sp; }
            }
        }
    }
    if (NT == 0) return false;
    p->rb = RB;
    a.M = M; a.N = N; a.K = K; a.NT = NT; a.nk = nk;
    a.tiles_n = (N + TC_BM * RB * cg - 1) / (TC_BM * RB * cg);
    a.tiles = a.tiles_n * ((M + NT - 1) / NT);
    if (RB == 1) {
        a.na = 2;
        a.nacc = NT <= 128 ? 2 : 1;   // TMEM: accumulators at columns 0 / 128, A ring of two 128-column slots from 256
        a.a_col0 = 256;
    } else {
        a.nacc = 1;   // TMEM: block accumulators at columns 0 and round_up(NT, 32), A ring of 64-column slots after
        a.a_col0 = round_up(round_up(NT, 32) + NT, 64);
        a.na = (512 - a.a_col0) / 64 < 4 ? (512 - a.a_col0) / 64 : 4;
    }
    a.tmem_cols = 512;
    int xk = 8;
    while (xk > 1 && (xk * (NT / cg) * 128 > 32768 || nk % xk != 0)) xk /= 2;
    (void)out_bytes;
    // Q8 chunks of 8 K steps (74 KB) leave too little room for the activation ring: 4 K steps for Q8 (measured:
    // 12288x2560 M=512 35.3 vs 52.6 us), 8 for Q4 (either is the same there); 256-row chunks: 4
    static const int pk_force = getenv("VKB_TC_PK") ? atoi(getenv("VKB_TC_PK")) : 0;   // tuning override
    const int pk_order[2] = {wf == 1 || RB == 2 ? 4 : 8, wf == 1 || RB == 2 ? 8 : 4};
    for (int pk : pk_order) {
        if (nk % pk != 0 || ((pk_force == 4 || pk_force == 8) && pk != pk_force && RB == 1)) continue;
        if (RB == 2 && pk != 4) continue;
        const int pchunk = RB * tc_pchunk(pk, wf);
        int nx = 4, np = 2;   // four X stages first: the activations are the fast-consumed stream
        auto bars_bytes = [&]() { return 8 * (2 * np + 2 * nx + 2 * a.na + 2 * a.nacc) + 16; };
        auto total = [&]() { return nx * xk * (NT / cg) * 128 + np * pchunk + bars_bytes() + 1024; };
        if (total() > d.smem_optin) nx = 2;
        if (total() > d.smem_optin) continue;
        for (bool grew = true; grew;) {
            grew = false;
            if (np < 6) { ++np; if (total() <= d.smem_optin) grew = true; else --np; }
            if (nx < 4 + 2 * cg) { nx += 2; if (total() <= d.smem_optin) grew = true; else nx -= 2; }
        }
        p->pk = pk;
        a.xk = xk;
        a.x_stage = xk * (NT / cg) * 128;
        a.nx = nx;
        a.np = np;
        a.x_off = 0;
        a.p_off = nx * a.x_stage;
        a.bar_off = a.p_off + np * pchunk;
        p->smem = total();
        p->cg = cg;
        p->grid = dim3((unsigned)((a.tiles < units_max ? a.tiles : units_max) * cg));
        a.splits = 1;
        a.kunit = TC_KUNIT;
        // split-K: the partial accumulator (fp32, 128 rows x NT tokens) goes where the rings were
        if (SPL > 1 && TC_BM * NT * 4 <= a.bar_off) {
            a.splits = SPL;
            p->grid = dim3((unsigned)(a.tiles * SPL));
        }
        if (split_exact > 0 && a.splits != split_exact) return false;
        return true;
    }
    return false;
}

// Opt one prompt-GEMM kernel variant into the device's shared memory, once per device.
template <typename OutT, int PK, bool P2P, int CG, int WF = 0, int RB = 1, bool SPLIT = false>
static int tc_attr(int dev, int smem_optin) {
    static std::once_flag once[kMaxDevices];
    static cudaError_t err[kMaxDevices];
    std::call_once(once[dev], [&] {
        err[dev] = cudaFuncSetAttribute(tc_q4_kernel<OutT, PK, P2P, CG, WF, RB, SPLIT>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin);
    });
    return err[dev] == cudaSuccess ? 0 : -(int)err[dev];
}

// Co-resident CTA pairs of the pair kernel at full shared memory (clusters are placed inside GPCs, so this can be
// less than half the SM count), once per device; 0 if the query fails.
template <typename OutT>
static int tc_max_pairs(int dev, int smem) {
    static std::once_flag once[kMaxDevices];
    static int pairs[kMaxDevices];
    std::call_once(once[dev], [&] {
        pairs[dev] = 0;
        if (tc_attr<OutT, 8, false, 2>(dev, smem) != 0) return;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2 * 512);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = (size_t)smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, tc_q4_kernel<OutT, 8, false, 2>, &cfg) == cudaSuccess) pairs[dev] = n;
        else cudaGetLastError();
    });
    return pairs[dev];
}

// Co-resident clusters of S split-K CTAs at full shared memory, for S = 0..8 (0 where the query fails), once per
// device.
static const int* tc_split_clusters(int dev, int smem) {
    static std::once_flag once[kMaxDevices];
    static int n[kMaxDevices][9];
    std::call_once(once[dev], [&] {
        if (tc_attr<__half, 8, false, 1, 0, 1, true>(dev, smem) != 0) return;
        for (int sp = 2; sp <= 8; ++sp) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(sp * 256);
            cfg.blockDim = dim3(TC_THREADS);
            cfg.dynamicSmemBytes = (size_t)smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)sp;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int c = 0;
            if (cudaOccupancyMaxActiveClusters(&c, tc_q4_kernel<__half, 8, false, 1, 0, 1, true>, &cfg) == cudaSuccess)
                n[dev][sp] = c;
            else
                cudaGetLastError();
        }
    });
    return n[dev];
}

template <typename OutT>
static int tc_entry(const void* q, const void* s, const void* x, void* y, int N, int K, int M, cudaStream_t st,
                    const TcOut* out = nullptr, int wf = 0) {
    if (!q || !s || !x || !y) return VKB_EINVAL;
    if (N < 1 || M < 1 || K < 256) return VKB_EINVAL;
    if (wf == 1 && out && out->p2p) return VKB_EUNSUPPORTED;   // peer stores: Q4 weights only
    if (K % 256 != 0) return VKB_EUNSUPPORTED;
    if (!aligned16(q) || !aligned16(s) || !aligned16(x)) return VKB_EUNSUPPORTED;
    int dev = 0;
    if (int r = current_device(&dev)) return r;
    const DeviceInfo& d = device_info(dev);
    if (d.cc_major < 10) return VKB_EUNSUPPORTED;
    // One CTA per tile. The CTA-pair kernel (tcgen05 cta_group::2, 256-row tiles, each SM streaming half of the
    // activations) is correct but measured slower on B200 at every shape of the sweep (12288x2560 M=512: 38.8 vs
    // 34.6 us; 8192x2048 M=64: 13.8 vs 10.6 us): VKB_TC_CG=2 selects it for experiments.
    static const int cg_force = getenv("VKB_TC_CG") ? atoi(getenv("VKB_TC_CG")) : 0;   // tuning override
    int cg = cg_force == 2 && N >= 2 * TC_BM && wf == 0 ? 2 : 1;
    if (out && out->p2p) cg = 1;
    int units_max = d.sm_count;
    if (cg == 2) {
        units_max = tc_max_pairs<OutT>(dev, d.smem_optin);
        if (units_max < 1) cg = 1, units_max = d.sm_count;
    }
    TcPlan p{};
    const bool p2p = out && out->p2p;
    // split-K: the planner's choice, or exactly the caller's count (the row split's); none for other peer-store calls
    const int split_exact = out ? out->split : 0;
    const bool split_ok = cg == 1 && (split_exact > 0 || !p2p);
    const int* clusters = split_ok ? tc_split_clusters(dev, d.smem_optin) : nullptr;
    if (!plan_tc(N, K, M, (int)sizeof(OutT), d, &p, cg, units_max, wf, !p2p, split_ok ? 8 : 1, clusters,
                 split_ok ? split_exact : 0))
        return VKB_EUNSUPPORTED;
    p.a.y = y;
    p.a.ldy = out ? out->ldy : N;
    p.a.ycol0 = out ? out->col0 : 0;
    p.a.p2p = out && out->p2p ? 1 : 0;
    if (p.a.p2p) p.a.pp = *out->p2p;
    if (p.a.p2p && p.grid.x > (unsigned)P2P_MAX_CTAS) return VKB_EUNSUPPORTED;   // one flag pair per CTA
    CUtensorMap tq, ts, tx;
    int r = get_tmap_2d(&tq, q, (uint64_t)N, (uint64_t)(wf == 1 ? K : K / 2), CU_TENSOR_MAP_DATA_TYPE_UINT64, 8,
                        (uint32_t)tc_ppitch(p.pk, wf) / 8, TC_BM * p.rb, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
    r = get_tmap_2d(&ts, s, (uint64_t)N, (uint64_t)K / 16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, TC_SPITCH / 2,
                    TC_BM * p.rb, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
    r = get_tmap_x3d(&tx, x, M, K, p.a.NT / p.cg, p.a.xk);   // a CTA's share of a tile's tokens
    if (r) return r;
    void (*kern)(CUtensorMap, CUtensorMap, CUtensorMap, TcArgs) = nullptr;
    int ra = 0;
    if (p.a.p2p) {
        if constexpr (std::is_same<OutT, __half>::value) {   // peer stores: fp16 outputs, one CTA per tile (share)
            if (p.a.splits > 1) {
                kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, true, 1, 0, 1, true> : tc_q4_kernel<OutT, 4, true, 1, 0, 1, true>;
                ra = p.pk == 8 ? tc_attr<OutT, 8, true, 1, 0, 1, true>(dev, d.smem_optin)
                               : tc_attr<OutT, 4, true, 1, 0, 1, true>(dev, d.smem_optin);
            } else {
                kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, true, 1> : tc_q4_kernel<OutT, 4, true, 1>;
                ra = p.pk == 8 ? tc_attr<OutT, 8, true, 1>(dev, d.smem_optin)
                               : tc_attr<OutT, 4, true, 1>(dev, d.smem_optin);
            }
        } else {
            return VKB_EUNSUPPORTED;
        }
    } else if (p.a.splits > 1 && wf == 1) {   // split-K clusters, Q8 weights
        kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, false, 1, 1, 1, true> : tc_q4_kernel<OutT, 4, false, 1, 1, 1, true>;
        ra = p.pk == 8 ? tc_attr<OutT, 8, false, 1, 1, 1, true>(dev, d.smem_optin)
                       : tc_attr<OutT, 4, false, 1, 1, 1, true>(dev, d.smem_optin);
    } else if (p.a.splits > 1) {   // split-K clusters (Q4, one CTA per tile share)
        kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, false, 1, 0, 1, true> : tc_q4_kernel<OutT, 4, false, 1, 0, 1, true>;
        ra = p.pk == 8 ? tc_attr<OutT, 8, false, 1, 0, 1, true>(dev, d.smem_optin)
                       : tc_attr<OutT, 4, false, 1, 0, 1, true>(dev, d.smem_optin);
    } else if (p.rb == 2) {   // 256-row tiles in one CTA (Q4, chunks of 4 K steps)
        kern = tc_q4_kernel<OutT, 4, false, 1, 0, 2>;
        ra = tc_attr<OutT, 4, false, 1, 0, 2>(dev, d.smem_optin);
    } else if (wf == 1) {   // Q8 weights
        kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, false, 1, 1> : tc_q4_kernel<OutT, 4, false, 1, 1>;
        ra = p.pk == 8 ? tc_attr<OutT, 8, false, 1, 1>(dev, d.smem_optin)
                       : tc_attr<OutT, 4, false, 1, 1>(dev, d.smem_optin);
    } else if (p.cg == 2) {
        kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, false, 2> : tc_q4_kernel<OutT, 4, false, 2>;
        ra = p.pk == 8 ? tc_attr<OutT, 8, false, 2>(dev, d.smem_optin) : tc_attr<OutT, 4, false, 2>(dev, d.smem_optin);
    } else {
        kern = p.pk == 8 ? tc_q4_kernel<OutT, 8, false, 1> : tc_q4_kernel<OutT, 4, false, 1>;
        ra = p.pk == 8 ? tc_attr<OutT, 8, false, 1>(dev, d.smem_optin) : tc_attr<OutT, 4, false, 1>(dev, d.smem_optin);
    }
    if (ra) return ra;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = p.grid;
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl_enabled() && pdl_stream_ok(st)) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (p.cg == 2 || p.a.splits > 1) {   // clusters along x: blocks kc .. kc + k - 1 form cluster c
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = p.cg == 2 ? 2u : (unsigned)p.a.splits;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tq, ts, tx, p.a);
    return e == cudaSuccess ? 0 : -(int)e;
}

int tc_split_for(int N, int K, int M, bool f32, int wf) {
    int dev = 0;
    if (current_device(&dev) != 0) return 1;
    const DeviceInfo& d = device_info(dev);
    if (d.cc_major < 10 || N < 1 || M < 1 || K < 256 || K % 256 != 0 || wf != 0) return 1;
    static const int cg_force = getenv("VKB_TC_CG") ? atoi(getenv("VKB_TC_CG")) : 0;   // (tc_entry's override)
    if (cg_force == 2 && N >= 2 * TC_BM) return 1;
    TcPlan p{};
    const int* clusters = tc_split_clusters(dev, d.smem_optin);
    if (!plan_tc(N, K, M, f32 ? 4 : 2, d, &p, 1, d.sm_count, wf, true, 8, clusters)) return 1;
    return p.a.splits;
}

int tc_dispatch(const void* q, const void* s, const void* x, void* y, bool f32, int N, int K, int M, cudaStream_t st,
                const TcOut* out, int wf) {
    return f32 ? tc_entry<float>(q, s, x, y, N, K, M, st, out, wf) : tc_entry<__half>(q, s, x, y, N, K, M, st, out, wf);
}

}  // namespace vkb

using namespace vkb;

extern "C" {

int vkb_gemv(int fmt, const void* q, const void* s, const void* x, void* y, int out_f32, int N, int K, int M,
             vkb_stream_t stream) {
    return qmv_dispatch(fmt, q, s, x, y, out_f32 != 0, nullptr, N, K, M, 0, 0, 0, 0, (cudaStream_t)stream);
}
int vkb_gemv_q4(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream) {
    return vkb_gemv(VKB_FMT_Q4, q, s, x, y, 0, N, K, M, stream);
}
int vkb_gemv_q8(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream) {
    return vkb_gemv(VKB_FMT_Q8, q, s, x, y, 0, N, K, M, stream);
}
int vkb_gemv_q2(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream) {
    return vkb_gemv(VKB_FMT_Q2, q, s, x, y, 0, N, K, M, stream);
}
int vkb_gemv_q4_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M, vkb_stream_t stream) {
    return vkb_gemv(VKB_FMT_Q4, q, s, x, y, 1, N, K, M, stream);
}
int vkb_gemv_q8_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M, vkb_stream_t stream) {
    return vkb_gemv(VKB_FMT_Q8, q, s, x, y, 1, N, K, M, stream);
}
int vkb_gemv_q2_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M, vkb_stream_t stream) {
    return vkb_gemv(VKB_FMT_Q2, q, s, x, y, 1, N, K, M, stream);
}

int vkb_moe(int fmt, const void* qpool, const void* spool, const int32_t* idx, int T, int topk, const void* x,
            void* y, int out_f32, int E_local, int e0, int N, int K, vkb_stream_t stream) {
    if (!idx) return VKB_EINVAL;
    return qmv_dispatch(fmt, qpool, spool, x, y, out_f32 != 0, idx, N, K, T, topk, E_local, e0, 0,
                        (cudaStream_t)stream);
}
int vkb_moe_q4(const void* qpool, const void* spool, const int32_t* idx, int T, int topk, const void* x, void* y,
               int E_local, int e0, int N, int K, vkb_stream_t stream) {
    return vkb_moe(VKB_FMT_Q4, qpool, spool, idx, T, topk, x, y, 0, E_local, e0, N, K, stream);
}

int vkb_gemv_q4_f32in(const void* q, const void* s, const float* x, void* xh, float* y, int N, int K, int M,
                      vkb_stream_t stream) {
    return qmv_q4_ext(q, s, x, true, xh, nullptr, y, true, false, N, K, M, (cudaStream_t)stream);
}

int vkb_gate_up_glu_q4_f32in(const void* q, const void* s, const float* x, void* xh, float* ystack, float* out, int N,
                             int K, int M, vkb_stream_t stream) {
    return qmv_q4_ext(q, s, x, true, xh, ystack, out, true, true, N, K, M, (cudaStream_t)stream);
}

int vkb_gate_up_glu_q4(const void* q, const void* s, const void* x, float* ystack, void* out, int out_f32, int N, int K,
                       int M, vkb_stream_t stream) {
    return qmv_q4_ext(q, s, x, false, nullptr, ystack, out, out_f32 != 0, true, N, K, M, (cudaStream_t)stream);
}

int vkb_gemm_q4_tc(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream) {
    return tc_entry<__half>(q, s, x, y, N, K, M, (cudaStream_t)stream);
}
int vkb_gemm_q4_tc_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M,
                       vkb_stream_t stream) {
    return tc_entry<float>(q, s, x, y, N, K, M, (cudaStream_t)stream);
}
int vkb_gemm_q8_tc(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream) {
    return tc_entry<__half>(q, s, x, y, N, K, M, (cudaStream_t)stream, nullptr, 1);
}
int vkb_gemm_q8_tc_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M,
                       vkb_stream_t stream) {
    return tc_entry<float>(q, s, x, y, N, K, M, (cudaStream_t)stream, nullptr, 1);
}
int vkb_gemm_tc(int fmt, const void* q, const void* s, const void* x, void* y, int out_f32, int N, int K, int M,
                vkb_stream_t stream) {
    if (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8) return VKB_EUNSUPPORTED;
    return tc_dispatch(q, s, x, y, out_f32 != 0, N, K, M, (cudaStream_t)stream, nullptr, fmt == VKB_FMT_Q8 ? 1 : 0);
}

int vkb_graph_begin(vkb_stream_t stream) {
    const cudaError_t e = cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal);
    return e == cudaSuccess ? 0 : -(int)e;
}

int vkb_graph_end(vkb_stream_t stream, void** graph_exec) {
    if (!graph_exec) return VKB_EINVAL;
    *graph_exec = nullptr;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture((cudaStream_t)stream, &g);
    if (e != cudaSuccess) return -(int)e;
    cudaGraphExec_t ge = nullptr;
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return -(int)e;
    *graph_exec = ge;
    return 0;
}

int vkb_graph_launch(void* graph_exec, vkb_stream_t stream) {
    if (!graph_exec) return VKB_EINVAL;
    const cudaError_t e = cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream);
    return e == cudaSuccess ? 0 : -(int)e;
}

int vkb_graph_destroy(void* graph_exec) {
    if (!graph_exec) return 0;
    const cudaError_t e = cudaGraphExecDestroy((cudaGraphExec_t)graph_exec);
    return e == cudaSuccess ? 0 : -(int)e;
}

const char* vkb_strerror(int code) {
    switch (code) {
        case VKB_OK: return "ok";
        case VKB_EUNSUPPORTED: return "unsupported shape, token count or format (nothing launched)";
        case VKB_EINVAL: return "invalid argument (nothing launched)";
        case VKB_ENOCOMM: return "no communicator for a multi-GPU call";
        case VKB_EDEVICE: return "a kernel reported a device-side timeout";
        default: break;
    }
    if (code <= -VKB_NCCL_BASE) return "NCCL error";
    if (code < 0) return cudaGetErrorString((cudaError_t)(-code));
    return "unknown vkb status";
}

int vkb_device_status(unsigned int* bits) {
    if (!bits) return VKB_EINVAL;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return -(int)e;
    unsigned v = 0;
    for (auto take : status_accessors())
        if (int r = take(&v)) return r;
    *bits = v;
    return 0;
}

int vkb_set_pdl(int enable) {
    const int old = pdl_enabled() ? 1 : 0;
    t_pdl = enable ? 1 : 0;
    return old;
}

int vkb_version(void) { return 100; }

int vkb_plan_describe(int kind, int fmt, int N, int K, int M, int sm_count, int smem_optin, int smem_per_sm,
                      int* info) {
    if (!info || N < 1 || K < 1 || M < 1 || sm_count < 1 || smem_optin < 1 || smem_per_sm < 1) return VKB_EINVAL;
    for (int i = 0; i < VKB_PLAN_INFO_LEN; ++i) info[i] = 0;
    const DeviceInfo d{sm_count, smem_optin, smem_per_sm, 10};
    if (kind == 0 || kind == 2) {   // decode GEMV / gate + up over [2N][K] (the pipelined kernel's shapes only)
        if (fmt < VKB_FMT_Q4 || fmt > VKB_FMT_Q2 || (kind == 2 && fmt != VKB_FMT_Q4)) return VKB_EINVAL;
        if (M > QMV_MAXTOK) return VKB_EUNSUPPORTED;
        if (K % 256 != 0) return VKB_EUNSUPPORTED;
        QmvPlan p{};
        if (!plan_qmv(fmt, N, K, M, 0, 0, d, &p, kind == 2, false, kind == 0)) return VKB_EUNSUPPORTED;
        const QmvArgs& a = p.a;
        const int v[] = {p.smem, a.nstage, a.nchunks, a.KS, a.wg, a.stage_bytes,
                         a.tilesN < sm_count ? a.tilesN : sm_count, a.cpitch, a.spitch, a.tilesN};
        for (int i = 0; i < (int)(sizeof(v) / sizeof(v[0])); ++i) info[i] = v[i];
        return 0;
    }
    if (kind == 1 || kind == 3) {   // prompt GEMM: one CTA per tile / with split-K where the planner picks it
        if (fmt != VKB_FMT_Q4 && fmt != VKB_FMT_Q8) return VKB_EINVAL;
        if (K < 256 || K % 256 != 0) return VKB_EUNSUPPORTED;
        TcPlan p{};
        const int wf = fmt == VKB_FMT_Q8 ? 1 : 0;
        if (!plan_tc(N, K, M, 2, d, &p, 1, sm_count, wf, true, kind == 3 ? 8 : 1)) return VKB_EUNSUPPORTED;
        const TcArgs& a = p.a;
        const int v[] = {p.smem, a.NT, p.rb, a.nacc, a.na, a.a_col0, a.tmem_cols, a.nx, a.xk, a.np, p.pk,
                         (int)p.grid.x, a.tiles, a.x_stage, a.tiles_n, kind == 3 ? a.splits : p.cg};
        for (int i = 0; i < (int)(sizeof(v) / sizeof(v[0])); ++i) info[i] = v[i];
        return 0;
    }
    return VKB_EINVAL;
}

}  // extern "C"
