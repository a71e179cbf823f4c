// libvkb.so, multi-GPU: the communicator (one NCCL rank per GPU, one process per GPU) and the two sharded paths.
//
//   MoE, expert parallel: rank r holds experts [e0, e0 + E_local) and runs the one-launch MoE kernel over the full
//   index list, writing its own slots and zeros into every other slot; one in-place ncclAllReduce(sum) combines the
//   ranks. Each slot has exactly one non-zero contributor, so the sum is exact and equal to the one-GPU result.
//
//   Prompt GEMM, row split: rank r holds weight rows [r N/G, (r+1) N/G). The tcgen05 kernel writes its [M][N/G] slice
//   into block r of a [G][M][N/G] workspace, an in-place ncclAllGather fills the other blocks, and a permute kernel
//   writes y [M][N] (y[m][g N/G + n] = work[g][m][n]).
//
// Every rank takes the same collective steps in the same order: argument checks depend only on values that are equal
// on all ranks (shapes, counts), and once they pass, the collective runs even if the local launch failed, so that no
// rank is left waiting; the call then returns the first error.
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>

#include <vector>

#include "../../include/vkb.h"
#include "p2p.cuh"
#include "ptx.cuh"
#include "vkb_internal.h"

// A symmetric buffer: the same size on every rank, this rank's allocation plus every peer's mapped by CUDA IPC.
struct SymBuf {
    void* base;
    size_t data_bytes;
    void* peer[vkb::P2P_MAX_RANKS];
};

struct vkb_comm {
    ncclComm_t nc;
    int rank, size, dev;
    std::vector<SymBuf> sym;
    SymBuf flags;   // the peer-store protocol's flags block (p2p.cuh), one per communicator: made by the first alloc
};

namespace vkb {

VKB_STATUS_ACCESSOR(status_take_comm)

static int nccl_rc(ncclResult_t r) { return r == ncclSuccess ? 0 : -(VKB_NCCL_BASE + (int)r); }

// y[m][g * nl + n] = work[g][m][n], 16 bytes per thread step when rows allow it.
template <typename T>
__global__ void __launch_bounds__(256) gather_permute_kernel(const T* __restrict__ work, T* __restrict__ y, int M, int nl,
                                                             int G, int vec) {
    pdl_wait();
    constexpr int V = 16 / sizeof(T);
    const long long total = (long long)G * M * nl;
    const long long step = (long long)gridDim.x * blockDim.x * (vec ? V : 1);
    for (long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * (vec ? V : 1); i < total; i += step) {
        const long long g = i / ((long long)M * nl), rem = i - g * M * nl;
        const long long m = rem / nl, n = rem - m * nl;
        T* dst = y + m * (long long)G * nl + g * nl + n;
        if (vec)
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(work + i);
        else
            *dst = work[i];
    }
}

template <typename T>
static int launch_permute(const void* work, void* y, int M, int nl, int G, cudaStream_t st) {
    const long long total = (long long)G * M * nl;
    // 16-byte copies need 16-byte aligned buffers and rows that are whole vectors
    const int vec = (nl % (16 / (int)sizeof(T))) == 0 && (reinterpret_cast<uintptr_t>(work) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
    const long long per = vec ? 16 / (long long)sizeof(T) : 1;
    long long blocks = (total / per + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() && pdl_stream_ok(st) ? 1 : 0;
    const cudaError_t e =
        cudaLaunchKernelEx(&cfg, gather_permute_kernel<T>, (const T*)work, (T*)y, M, nl, G, vec);
    return e == cudaSuccess ? 0 : -(int)e;
}

// The all-gather of a row-split call, joined without computing anything (a rank-local failure after the checks every
// rank shares): buf (M * N elements, any contents) sends this rank's block and receives the peers', so that no peer is
// left waiting in the collective. Returns the collective's own status.
static int rowsplit_join(vkb_comm_t* c, void* buf, bool f32, int N, int M, cudaStream_t st) {
    const size_t chunk = (size_t)M * (N / c->size);
    uint8_t* mine = static_cast<uint8_t*>(buf) + (size_t)c->rank * chunk * (f32 ? 4 : 2);
    return nccl_rc(ncclAllGather(mine, buf, chunk, f32 ? ncclFloat : ncclHalf, c->nc, st));
}

static int rowsplit(vkb_comm_t* c, const void* q, const void* s, const void* x, void* y, void* work, bool f32, int N,
                    int K, int M, cudaStream_t st) {
    if (!c) return VKB_ENOCOMM;
    // shape checks (equal on every rank): a failure here returns before any rank reaches the collective
    if (N < 1 || M < 1 || K < 256) return VKB_EINVAL;
    if (N % c->size != 0 || K % 256 != 0) return VKB_EUNSUPPORTED;
    if (!q || !s || !x || !y || !work) {   // this rank only: join the collective with whichever buffer it has
        if (work || y) rowsplit_join(c, work ? work : y, f32, N, M, st);
        return VKB_EINVAL;                 // (with neither, the peers' all-gather waits: a caller error)
    }
    const int nl = N / c->size;
    const size_t esz = f32 ? 4 : 2;
    const size_t chunk = (size_t)M * nl;                    // elements per rank
    uint8_t* mine = static_cast<uint8_t*>(work) + (size_t)c->rank * chunk * esz;
    // a local refusal past this point (e.g. an unaligned pointer on one rank) still joins the collective. The local
    // product takes the split-K count of the whole problem's one-GPU plan, so y is the one-GPU result bit for bit.
    const TcOut out{nl, 0, nullptr, tc_split_for(N, K, M, f32)};
    int rc = tc_dispatch(q, s, x, mine, f32, nl, K, M, st, &out);
    const int rc_nccl = nccl_rc(ncclAllGather(mine, work, chunk, f32 ? ncclFloat : ncclHalf, c->nc, st));
    if (rc == 0) rc = rc_nccl;
    const int rc_p = f32 ? launch_permute<float>(work, y, M, nl, c->size, st)
                         : launch_permute<__half>(work, y, M, nl, c->size, st);
    return rc != 0 ? rc : rc_p;
}

static int moe_ep(vkb_comm_t* c, int fmt, const void* qpool, const void* spool, const int32_t* idx, int T, int topk,
                  const void* x, void* y, bool f32, int E_local, int e0, int N, int K, cudaStream_t st) {
    if (!c) return VKB_ENOCOMM;
    if (!idx || !y) return VKB_EINVAL;
    // the kernel's checks are shape checks (equal on every rank; unaligned buffers take the general kernel, not a
    // refusal), so a refusal here happens on every rank before any reaches the collective
    int rc = qmv_dispatch(fmt, qpool, spool, x, y, f32, idx, N, K, T, topk, E_local, e0, 1, st);
    if (rc > 0) return rc;
    const size_t count = (size_t)T * topk * N;
    const int rc_nccl = nccl_rc(ncclAllReduce(y, y, count, f32 ? ncclFloat : ncclHalf, ncclSum, c->nc, st));
    return rc != 0 ? rc : rc_nccl;
}

// Workspace of the allocation-free row-split entry point: a file-scope device array (no cudaMalloc anywhere on that
// path), for callers that cannot allocate: a launcher with a fixed signature that has no workspace argument, or a
// process whose device memory is all reserved by its own pool. Every GPU that loads the library holds the 16 MiB
// until the process exits. Its size bounds M * N * 2 bytes. Every byte is written before it is read (block r by this
// rank's kernel, the others by the all-gather), so nothing has to be cleared between calls; calls that overlap in
// time (two streams, two host threads, or two communicators in one process on the same device) share it and race.
// In host code the name g_rowsplit_scratch is a host-side stand-in, not a device address: only the address that
// rowsplit_scratch() looks up may be passed to a kernel.
constexpr size_t kRowsplitScratchBytes = (size_t)16 << 20;
static __device__ __align__(256) uint8_t g_rowsplit_scratch[kRowsplitScratchBytes];

// Device address of the array on device `dev`, looked up once per device (the symbol is per device context) by the
// first call on that device, with `dev` current (the caller's current device); the entry point's first call on a
// device should therefore come before any stream capture.
static int rowsplit_scratch(int dev, void** out) {
    static std::once_flag once[kMaxDevices];
    static void* addr[kMaxDevices];
    static cudaError_t err[kMaxDevices];
    std::call_once(once[dev], [dev] { err[dev] = cudaGetSymbolAddress(&addr[dev], g_rowsplit_scratch); });
    if (err[dev] != cudaSuccess) return -(int)err[dev];
    *out = addr[dev];
    return 0;
}

static SymBuf* find_sym(vkb_comm_t* c, const void* p, size_t need) {
    for (auto& b : c->sym)
        if (b.base == p && b.data_bytes >= need) return &b;
    return nullptr;
}

// The kernels' view of a symmetric buffer (every rank's copy; null: none) and of the communicator's flags block.
static P2PArgs p2p_args(const vkb_comm_t* c, const SymBuf* b) {
    P2PArgs pp{};
    for (int r = 0; r < c->size; ++r) {
        pp.peer_base[r] = b ? b->peer[r] : nullptr;
        pp.peer_flags[r] = static_cast<uint32_t*>(c->flags.peer[r]);
    }
    pp.rank = c->rank;
    pp.size = c->size;
    return pp;
}

// One fused call on a rank that refused it on the host after the checks every rank shares (a pointer that is not a
// symmetric buffer, an unaligned operand, a failed launch): the epoch protocol's part of the call (p2p_abstain), so
// that the peers' kernels finish at once with DEV_ERR_PEER_FAILED instead of waiting out their bounded waits, and the
// ranks' call numbering stays aligned. Nothing is written but flags.
__global__ void __launch_bounds__(256) p2p_abstain_kernel(P2PArgs pp) {
    pdl_wait();
    p2p_abstain(pp);
}

static void abstain(const vkb_comm_t* c, cudaStream_t st) {
    if (!c->flags.base) return;   // no symmetric buffer yet on this communicator: no peer can be in a fused call
    p2p_abstain_kernel<<<1, 256, 0, st>>>(p2p_args(c, nullptr));
    cudaGetLastError();   // a failed launch here leaves the peers to their bounded waits; the caller has its error
}

static int sym_free_one(vkb_comm_t* c, SymBuf& b) {
    int rc = 0;
    for (int r = 0; r < c->size; ++r)
        if (r != c->rank && b.peer[r]) {
            const cudaError_t e = cudaIpcCloseMemHandle(b.peer[r]);
            if (e != cudaSuccess && rc == 0) rc = -(int)e;
        }
    const cudaError_t e = cudaFree(b.base);
    if (e != cudaSuccess && rc == 0) rc = -(int)e;
    return rc;
}

// Collective: `bytes` (rounded up to 256) of zeroed device memory on every rank, every rank's allocation mapped into
// every peer by CUDA IPC (handles exchanged over the communicator). Every rank that reaches the exchange with valid
// arguments joins it, also after a local failure, and the call then returns that failure.
static int sym_alloc(vkb_comm_t* comm, size_t bytes, SymBuf* out) {
    SymBuf b{};
    b.data_bytes = (bytes + 255) / 256 * 256;
    cudaError_t e = cudaMalloc(&b.base, b.data_bytes);
    if (e != cudaSuccess) b.base = nullptr;
    if (e == cudaSuccess) e = cudaMemset(b.base, 0, b.data_bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, b.base);
    void* dh = nullptr;
    if (cudaMalloc(&dh, sizeof(h) * comm->size) != cudaSuccess) dh = nullptr;
    int rc = e == cudaSuccess ? 0 : -(int)e;
    if (rc == 0 && !dh) rc = -(int)cudaErrorMemoryAllocation;
    std::vector<cudaIpcMemHandle_t> all(comm->size);
    if (rc == 0) {
        e = cudaMemcpy(static_cast<uint8_t*>(dh) + comm->rank * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice);
        rc = e == cudaSuccess ? 0 : -(int)e;
    }
    if (dh) {   // the collective runs on every rank that got its exchange buffer
        const int rn = nccl_rc(ncclAllGather(static_cast<uint8_t*>(dh) + comm->rank * sizeof(h), dh, sizeof(h),
                                             ncclUint8, comm->nc, nullptr));
        if (!rc) rc = rn;
        e = cudaStreamSynchronize(nullptr);
        if (!rc && e != cudaSuccess) rc = -(int)e;
        if (!rc) {
            e = cudaMemcpy(all.data(), dh, sizeof(h) * comm->size, cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) rc = -(int)e;
        }
        cudaFree(dh);
    }
    for (int r = 0; r < comm->size && rc == 0; ++r) {
        if (r == comm->rank) { b.peer[r] = b.base; continue; }
        e = cudaIpcOpenMemHandle(&b.peer[r], all[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) rc = -(int)e;
    }
    if (rc) {
        for (int r = 0; r < comm->size; ++r)
            if (r != comm->rank && b.peer[r]) cudaIpcCloseMemHandle(b.peer[r]);
        if (b.base) cudaFree(b.base);
        return rc;
    }
    *out = b;
    return 0;
}

}  // namespace vkb

using namespace vkb;

extern "C" {

int vkb_comm_unique_id(void* id) {
    if (!id) return VKB_EINVAL;
    ncclUniqueId u;
    const int rc = nccl_rc(ncclGetUniqueId(&u));
    if (rc) return rc;
    static_assert(sizeof(ncclUniqueId) == VKB_UNIQUE_ID_BYTES, "NCCL unique id size");
    memcpy(id, &u, sizeof(u));
    return 0;
}

int vkb_comm_init(vkb_comm_t** comm, int rank, int nranks, const void* id) {
    if (!comm || !id) return VKB_EINVAL;
    *comm = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks) return VKB_EINVAL;
    int dev = 0;
    if (int r = current_device(&dev)) return r;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t nc = nullptr;
    const int rc = nccl_rc(ncclCommInitRank(&nc, nranks, u, rank));
    if (rc) return rc;
    vkb_comm* c = new (std::nothrow) vkb_comm{nc, rank, nranks, dev, {}, {}};
    if (!c) {
        ncclCommDestroy(nc);
        return VKB_EINVAL;
    }
    // Warm-up collectives of the kinds and sizes the entry points issue: NCCL sets up connection buffers on a
    // communicator's first use of an algorithm, so this happens here (set-up) rather than inside a later call.
    const size_t per = (size_t)4 << 20;   // bytes per rank
    void* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, per * nranks);
    int wrc = e == cudaSuccess ? 0 : -(int)e;
    if (wrc == 0) {
        const size_t n = per / 2;
        wrc = nccl_rc(ncclAllGather(static_cast<uint8_t*>(tmp) + (size_t)rank * per, tmp, n, ncclHalf, nc, nullptr));
        if (wrc == 0) wrc = nccl_rc(ncclAllReduce(tmp, tmp, n, ncclHalf, ncclSum, nc, nullptr));
        e = cudaStreamSynchronize(nullptr);
        if (wrc == 0 && e != cudaSuccess) wrc = -(int)e;
        cudaFree(tmp);
    }
    if (wrc != 0) {
        ncclCommDestroy(nc);
        delete c;
        return wrc;
    }
    *comm = c;
    return 0;
}

int vkb_comm_destroy(vkb_comm_t* comm) {
    if (!comm) return 0;
    int rc = 0;
    for (auto& b : comm->sym) {
        const int r = sym_free_one(comm, b);
        if (r && !rc) rc = r;
    }
    if (comm->flags.base) {
        const int r = sym_free_one(comm, comm->flags);
        if (r && !rc) rc = r;
    }
    const int r = nccl_rc(ncclCommDestroy(comm->nc));
    delete comm;
    return rc ? rc : r;
}

int vkb_comm_alloc(vkb_comm_t* comm, size_t bytes, void** ptr) {
    if (!comm || !ptr || bytes == 0) return VKB_EINVAL;
    *ptr = nullptr;
    if (comm->size > P2P_MAX_RANKS) return VKB_EUNSUPPORTED;
    if (!comm->flags.base) {   // the communicator's flags block comes with its first symmetric buffer (collective)
        if (int rc = sym_alloc(comm, P2P_FLAG_BYTES, &comm->flags)) return rc;
    }
    SymBuf b{};
    if (int rc = sym_alloc(comm, bytes, &b)) return rc;
    comm->sym.push_back(b);
    *ptr = b.base;
    return 0;
}

int vkb_comm_free(vkb_comm_t* comm, void* ptr) {
    if (!comm || !ptr) return VKB_EINVAL;
    for (size_t i = 0; i < comm->sym.size(); ++i)
        if (comm->sym[i].base == ptr) {
            // nobody may still store into this rank's copy: every rank has finished with the buffer before the
            // mappings go away
            cudaError_t e = cudaDeviceSynchronize();
            int rc = e == cudaSuccess ? 0 : -(int)e;
            void* tmp = nullptr;
            if (cudaMalloc(&tmp, 4) == cudaSuccess) {
                const int rn = nccl_rc(ncclAllReduce(tmp, tmp, 1, ncclInt32, ncclSum, comm->nc, nullptr));
                if (!rc) rc = rn;
                e = cudaStreamSynchronize(nullptr);
                if (!rc && e != cudaSuccess) rc = -(int)e;
                cudaFree(tmp);
            }
            const int rf = sym_free_one(comm, comm->sym[i]);
            comm->sym.erase(comm->sym.begin() + (long)i);
            return rc ? rc : rf;
        }
    return VKB_EINVAL;
}

int vkb_comm_rank(const vkb_comm_t* comm) { return comm ? comm->rank : -1; }
int vkb_comm_size(const vkb_comm_t* comm) { return comm ? comm->size : -1; }

int vkb_moe_ep(vkb_comm_t* comm, int fmt, const void* qpool, const void* spool, const int32_t* idx, int T, int topk,
               const void* x, void* y, int out_f32, int E_local, int e0, int N, int K, vkb_stream_t stream) {
    return moe_ep(comm, fmt, qpool, spool, idx, T, topk, x, y, out_f32 != 0, E_local, e0, N, K, (cudaStream_t)stream);
}

int vkb_moe_q4_ep(vkb_comm_t* comm, const void* qpool, const void* spool, const int32_t* idx, int T, int topk,
                  const void* x, void* y, int E_local, int e0, int N, int K, vkb_stream_t stream) {
    return moe_ep(comm, VKB_FMT_Q4, qpool, spool, idx, T, topk, x, y, false, E_local, e0, N, K, (cudaStream_t)stream);
}

int vkb_moe_ep_p2p(vkb_comm_t* comm, int fmt, const void* qpool, const void* spool, const int32_t* idx, int T,
                   int topk, const void* x, void* y_sym, int out_f32, int E_local, int e0, int N, int K,
                   vkb_stream_t stream) {
    if (!comm) return VKB_ENOCOMM;
    if (T < 1 || topk < 1 || N < 1) return VKB_EINVAL;               // equal on every rank
    if (comm->size > P2P_MAX_RANKS) return VKB_EUNSUPPORTED;
    const cudaStream_t st = (cudaStream_t)stream;
    // past this point a refusal is this rank's alone: it still takes its part in the call's epoch protocol
    SymBuf* b = idx ? find_sym(comm, y_sym, (size_t)T * topk * N * (out_f32 ? 4 : 2)) : nullptr;
    int rc = VKB_EINVAL;   // y must come from vkb_comm_alloc and hold T*topk x N outputs
    if (b) {
        const P2PArgs pp = p2p_args(comm, b);
        rc = qmv_dispatch(fmt, qpool, spool, x, y_sym, out_f32 != 0, idx, N, K, T, topk, E_local, e0, 0, st, &pp);
    }
    if (rc != 0) abstain(comm, st);
    return rc;
}

size_t vkb_gemm_rowsplit_work_bytes(int M, int N, int out_f32) {
    if (M < 1 || N < 1) return 0;
    return (size_t)M * N * (out_f32 ? 4 : 2);
}

int vkb_gemm_q4_tc_rowsplit(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, void* y,
                            void* work, int N, int K, int M, vkb_stream_t stream) {
    return rowsplit(comm, q_local, s_local, x, y, work, false, N, K, M, (cudaStream_t)stream);
}

int vkb_gemm_q4_tc_rowsplit_noalloc(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, void* y,
                                    int N, int K, int M, vkb_stream_t stream) {
    if (!comm) return VKB_ENOCOMM;
    if (N < 1 || M < 1 || K < 256) return VKB_EINVAL;                                  // equal on every rank
    if ((size_t)M * (size_t)N * 2 > kRowsplitScratchBytes) return VKB_EUNSUPPORTED;   // equal on every rank
    if (N % comm->size != 0 || K % 256 != 0) return VKB_EUNSUPPORTED;                 // equal on every rank
    int dev = 0;
    void* work = nullptr;
    int r = current_device(&dev);
    if (r == 0) r = rowsplit_scratch(dev, &work);
    if (r != 0) {   // this rank only: join the peers' all-gather through y, then report the lookup failure
        if (y) rowsplit_join(comm, y, false, N, M, (cudaStream_t)stream);
        return r;
    }
    return rowsplit(comm, q_local, s_local, x, y, work, false, N, K, M, (cudaStream_t)stream);
}

int vkb_gemm_q4_tc_rowsplit_p2p(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, void* y_sym,
                                int N, int K, int M, vkb_stream_t stream) {
    if (!comm) return VKB_ENOCOMM;
    if (N < 1 || M < 1 || K < 256) return VKB_EINVAL;                                        // equal on every rank
    if (N % comm->size != 0 || K % 256 != 0 || comm->size > P2P_MAX_RANKS) return VKB_EUNSUPPORTED;
    const cudaStream_t st = (cudaStream_t)stream;
    // past this point a refusal is this rank's alone: it still takes its part in the call's epoch protocol
    SymBuf* b = (q_local && s_local && x) ? find_sym(comm, y_sym, (size_t)M * N * 2) : nullptr;
    int rc = VKB_EINVAL;   // y must come from vkb_comm_alloc and hold M x N fp16
    if (b) {
        const P2PArgs pp = p2p_args(comm, b);
        const int nl = N / comm->size;
        const TcOut out{N, comm->rank * nl, &pp, tc_split_for(N, K, M, false)};   // (the one-GPU split: same bits)
        rc = tc_dispatch(q_local, s_local, x, y_sym, false, nl, K, M, st, &out);
    }
    if (rc != 0) abstain(comm, st);
    return rc;
}

int vkb_comm_epoch(const vkb_comm_t* comm, unsigned int* epoch) {
    if (!comm || !epoch) return VKB_EINVAL;
    *epoch = 0;
    if (!comm->flags.base) return 0;
    uint32_t v = 0;
    const cudaError_t e = cudaMemcpy(&v, static_cast<const uint32_t*>(comm->flags.base) + P2P_EPOCH, sizeof(v),
                                     cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return -(int)e;
    *epoch = v;
    return 0;
}

int vkb_gemm_q4_tc_rowsplit_f32(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, float* y,
                                void* work, int N, int K, int M, vkb_stream_t stream) {
    return rowsplit(comm, q_local, s_local, x, y, work, true, N, K, M, (cudaStream_t)stream);
}

}  // extern "C"
