// Internal helpers shared by the translation units of libvkb.so (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vkb {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    int sm_count;
    int smem_optin;    // max dynamic shared memory per block (opt-in)
    int smem_per_sm;   // shared memory per SM
    int cc_major;
};

// Facts about device `dev`, queried once per process.
const DeviceInfo& device_info(int dev);
// The current device, or an error code (see vkb.h).
int current_device(int* dev);
// Whether launches on this host thread use programmatic dependent launch.
bool pdl_enabled();
// Encode (or fetch from this thread's cache) a 2-D tiled TMA descriptor over a row-major tensor.
int get_tmap_2d(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t row_bytes, CUtensorMapDataType dtype,
                uint32_t elem_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz);

// The decode / MoE entry (formats VKB_FMT_*; idx == nullptr: dense) and the prompt GEMM entry, shared with the
// multi-GPU entry points. Same return codes as the C ABI.
struct P2PArgs;
int qmv_dispatch(int fmt, const void* q, const void* s, const void* x, void* y, bool f32, const int32_t* idx, int N,
                 int K, int M, int topk, int E_local, int e0, int zero_foreign, cudaStream_t st,
                 const P2PArgs* p2p = nullptr);
// Where the prompt GEMM writes: y rows of ldy elements starting at column col0, and with p2p also into every peer's
// copy of a symmetric buffer (epoch protocol of p2p.cuh).
struct TcOut {
    int ldy, col0;
    const P2PArgs* p2p;
    int split = 0;   // split-K CTAs per tile: 0 the planner's choice (none with peer stores), n >= 1 exactly n
};
// The split-K count the one-GPU prompt GEMM of the whole problem takes on the current device (1: none): a row split
// whose ranks use it sums every output in the one-GPU order.
int tc_split_for(int N, int K, int M, bool f32, int wf = 0);
// wf: weight format of the prompt GEMM (0 = Q4, 1 = Q8).
int tc_dispatch(const void* q, const void* s, const void* x, void* y, bool f32, int N, int K, int M, cudaStream_t st,
                const TcOut* out = nullptr, int wf = 0);
bool pdl_stream_ok(cudaStream_t st);

// Host accessors of the per-translation-unit device status words (read and clear, OR into *bits).
using StatusTake = int (*)(unsigned*);
int status_take_qmv(unsigned* bits);
int status_take_comm(unsigned* bits);
struct StatusList {
    const StatusTake* b;
    const StatusTake* e;
    const StatusTake* begin() const { return b; }
    const StatusTake* end() const { return e; }
};
StatusList status_accessors();

}  // namespace vkb
