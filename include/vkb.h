/*
 * vkb.h -- C ABI of libvkb.so, the B200 (sm_100a) quantised matrix-multiply hot path of volta-kernel-bakeoff.
 *
 * Every entry point replaces one "contender launcher" of the reference harness, whose convention is
 *     bool launch(int M, const uint32_t* q, const half* s, const half* x, float* y, int N, int K)
 * (reference src/bakeoff.cu:263-280, src/stage2.cuh:221-224, src/stage4_tc.cuh:197-200): the caller owns every device
 * buffer, the call is asynchronous on the given stream, and an unsupported shape launches nothing and writes nothing.
 *
 * Conventions of this library:
 *   - return 0: launched. return > 0: VKB_E* below, nothing launched, nothing written. return < 0: -(cudaError_t) of
 *     a CUDA runtime error, or -(VKB_NCCL_BASE + ncclResult_t) of an NCCL error. Nothing exits, traps or asserts.
 *   - stream: a cudaStream_t (NULL = the legacy default stream).
 *   - Weight formats (byte-identical to the reference, src/bakeoff.cu:5-8, :210-219, :486-490; src/stage2.cuh:235-244;
 *     src/stage3_lut.cuh:4, :90-97), one fp16 scale per 32 consecutive values of a row, scales [N][K/32]:
 *       Q4  uint32 [N][K/8]   word w of a row holds codes 8w..8w+7, code i in nibble i, stored as code + 8 (-8..7)
 *       Q8  int8   [N][K]     one two's-complement code per value (-127..127)
 *       Q2  uint32 [N][K/16]  word w holds codes 16w..16w+15, code i in bits 2i..2i+1, stored as code + 2 (-2..1)
 *     value = code * scale. Activations x are fp16 [M][K] row-major; outputs y are fp16 [M][N] row-major (the _f32
 *     variants write fp32, exactly the reference launchers' float* y).
 *   - K must be a multiple of 32. The fast path (TMA-staged, tensor cores) needs K % 256 == 0 and 16-byte aligned
 *     q, s and x; other shapes run a plain CUDA-core kernel with the same results.
 *   - Thread-safe: per-device one-time set-up is guarded; tensor-map caches are per host thread.
 *   - Launches use programmatic dependent launch (PDL) unless vkb_set_pdl(0): the weight stream of call i+1 overlaps
 *     the tail of call i; activations and outputs are still ordered after the previous kernel on the stream. The
 *     weights and scales are read BEFORE the preceding kernel in the stream has finished, so that kernel must not
 *     write them (weights are normally static; after a kernel that repacks them, call vkb_set_pdl(0) for the next
 *     call or put any other kernel in between). MoE calls read nothing before the preceding kernel has finished: their
 *     index list (which a router kernel may have just written) decides which weights they read.
 */
#ifndef VKB_H
#define VKB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* vkb_stream_t; /* == cudaStream_t */

enum {
    VKB_OK = 0,
    VKB_EUNSUPPORTED = 1, /* shape, token count or format not supported: nothing launched */
    VKB_EINVAL = 2,       /* null pointer or out-of-range argument: nothing launched */
    VKB_ENOCOMM = 3,      /* multi-GPU call without a communicator */
    VKB_EDEVICE = 4,      /* a kernel reported a device-side timeout (see vkb_device_status) */
};
#define VKB_NCCL_BASE 1000

enum { VKB_FMT_Q4 = 0, VKB_FMT_Q8 = 1, VKB_FMT_Q2 = 2 };

/* ---- decode GEMV: y[M][N] = x[M][K] . W[N][K]^T, 1 <= M <= 8 ------------------------------------------------------
 * Replace fused_q4_v2w<M> / fused_q4_v3 (reference src/stage2.cuh:61-92, :217-224; src/stage5_gap8.cuh:57-137,
 * :203-205), fused_q8<M> (src/bakeoff.cu:115-155, :272-280) and q2w_alu_v3 (src/stage3_lut.cuh:155-185; the
 * reference has 1 token only). fp16 output. */
int vkb_gemv_q4(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream);
int vkb_gemv_q8(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream);
int vkb_gemv_q2(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream);
/* The same with fp32 output, the reference launchers' own float* y (src/bakeoff.cu:263-280). */
int vkb_gemv_q4_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M, vkb_stream_t stream);
int vkb_gemv_q8_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M, vkb_stream_t stream);
int vkb_gemv_q2_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M, vkb_stream_t stream);
/* Format chosen at run time (fmt = VKB_FMT_*), out_f32 selects the fp32 output. */
int vkb_gemv(int fmt, const void* q, const void* s, const void* x, void* y, int out_f32, int N, int K, int M,
             vkb_stream_t stream);

/* ---- decode with fp32 activations, and gate + up + SwiGLU ---------------------------------------------------------
 * Replace fused_q4_v3_fp32in and gate_up_glu_fp32in (reference src/stage5_gap8.cuh:207-245), Q4 only like them.
 *
 * vkb_gemv_q4_f32in: x fp32 [M][K] is rounded to fp16 (round to nearest even) and multiplied as vkb_gemv_q4_f32
 * would on the rounded x (up to the order of fp32 sums). The pipelined decode kernel (K % 256 == 0, 16-byte aligned
 * q, s, x) reads and rounds the fp32 activations itself: one launch. Other shapes first convert x into xh (M * K fp16,
 * caller-owned scratch, the reference's xh) with one small kernel; xh may be null when the pipelined kernel runs.
 *
 * vkb_gate_up_glu_q4_f32in: q, s hold the stacked [2N][K] table (rows 0..N-1 gate, N..2N-1 up). ystack [M][2N] fp32
 * receives the stacked product (may be null); out [M][N] fp32 = silu(gate) * up, silu(g) = g / (1 + exp(-g)).
 * One kernel: gate tile j and up tile j go to adjacent warp groups of one CTA; the SwiGLU is applied where the two
 * sums meet. It needs K % 256 == 0 and 16-byte aligned q, s, x: VKB_EUNSUPPORTED otherwise (xh is not used).
 * vkb_gate_up_glu_q4 is the same with fp16 activations and fp16 (out_f32 = 0) or fp32 output.
 *
 * Token counts 1..8 (the reference: 1, 2, 4, 8 only; 3, 5, 6, 7 work here too); M > 8 is VKB_EUNSUPPORTED. */
int vkb_gemv_q4_f32in(const void* q, const void* s, const float* x, void* xh, float* y, int N, int K, int M,
                      vkb_stream_t stream);
int vkb_gate_up_glu_q4_f32in(const void* q, const void* s, const float* x, void* xh, float* ystack, float* out, int N,
                             int K, int M, vkb_stream_t stream);
int vkb_gate_up_glu_q4(const void* q, const void* s, const void* x, float* ystack, void* out, int out_f32, int N, int K,
                       int M, vkb_stream_t stream);

/* ---- GGUF Q4_0 / Q8_0 weights in device memory -> the split layout above ----------------------------------------------
 * blocks: N * K/32 GGUF blocks (Q4_0 18 bytes, Q8_0 34 bytes; 2-byte aligned) in device memory; q (16-byte aligned)
 * and scales receive the packed codes and fp16 scales of the formats above, bit-exactly (the host counterparts and
 * the block layouts: vkb_host.h). One memory-bound kernel on stream. No counterpart in the reference, which states
 * value parity with GGUF (src/bakeoff.cu:5-7) but loads no GGUF data. */
int vkb_gguf_to_vkb_device(int fmt, const void* blocks, int N, int K, void* q, void* scales, vkb_stream_t stream);
/* Dense copy of packed weights: w [N][K] fp16 (out_bf16 = 0) or bf16 = code * scale with one round-to-nearest (the
 * reference's dequant_q4, src/bakeoff.cu:52-68, that feeds its "dq4+cublas" control, :687-690; here for every
 * format). q in the layout of the format's GEMV (4-byte aligned for Q4, 8 for Q8, 2 for Q2), s fp16 [N][K/32], w
 * 16-byte aligned. K % 32 == 0 (Q2: K % 64 == 0). */
int vkb_dequant(int fmt, const void* q, const void* s, void* w, int N, int K, int out_bf16, vkb_stream_t stream);

/* ---- MoE decode, one launch ----------------------------------------------------------------------------------------
 * Replaces moe_fused_q4 + MoePtrs (reference src/bakeoff.cu:157-186, :826-830), where the host picked one pointer set
 * per expert, with a device-side index list:
 *   qpool [E_local][N][K/8] (Q4; Q8/Q2 analogously), spool [E_local][N][K/32] fp16 -- the experts e0..e0+E_local-1
 *   idx   int32 [T][topk] global expert ids (distinct per token in the reference's usage; duplicates are allowed)
 *   x     fp16 [T][K], y fp16 [T][topk][N]: y[t][j] = W_{idx[t][j]} . x[t]
 * Slots whose expert is outside [e0, e0 + E_local) are not written (expert parallelism: each rank fills its own). All
 * slots of one expert share a single pass over that expert's weights (up to 8 tokens per pass). */
int vkb_moe_q4(const void* qpool, const void* spool, const int32_t* idx, int T, int topk, const void* x, void* y,
               int E_local, int e0, int N, int K, vkb_stream_t stream);
int vkb_moe(int fmt, const void* qpool, const void* spool, const int32_t* idx, int T, int topk, const void* x, void* y,
            int out_f32, int E_local, int e0, int N, int K, vkb_stream_t stream);

/* ---- prompt GEMM on tcgen05: y[M][N] = x[M][K] . W[N][K]^T, any M >= 1 -----------------------------------------------
 * Replaces tc_q4 / tc_q4_v2 (reference src/stage2.cuh:94-154, :226-229; src/stage4_tc.cuh:38-200): the weights are
 * dequantised to fp16 exactly as the reference rounds them ((code - 8) * scale, one rounding) and multiplied on the
 * 5th-generation tensor cores with fp32 accumulation. Needs K % 256 == 0 and 16-byte aligned q, s, x; any M
 * and N (no tile-multiple requirement). fp16 output; _f32 writes fp32 (the reference's float* y).
 * Tables with few 128-row tiles (K % 512 == 0) run split-K (the reference's split-K, src/stage4_tc.cuh:130-141):
 * clusters of 2-8 CTAs share a tile's K range and sum their fp32 partials in a fixed order over distributed shared
 * memory, so repeated calls give identical bits (the reference's atomicAdd reduction does not). */
int vkb_gemm_q4_tc(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream);
int vkb_gemm_q4_tc_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M,
                       vkb_stream_t stream);

/* Q8 weights (int8 codes [N][K], scales [N][K/32]) on the same tcgen05 kernel: the tc_q8 the reference planned but
 * never built (its STAGE3.md). Weights are rounded to fp16 as code * scale (one rounding), as in the Q4 kernel (fp16
 * class). Same shapes and alignment rules as vkb_gemm_q4_tc. vkb_gemm_tc takes the format at run time (Q4 or Q8). */
int vkb_gemm_q8_tc(const void* q, const void* s, const void* x, void* y, int N, int K, int M, vkb_stream_t stream);
int vkb_gemm_q8_tc_f32(const void* q, const void* s, const void* x, float* y, int N, int K, int M,
                       vkb_stream_t stream);
int vkb_gemm_tc(int fmt, const void* q, const void* s, const void* x, void* y, int out_f32, int N, int K, int M,
                vkb_stream_t stream);

/* ---- multi-GPU: one process (and one rank) per GPU ---------------------------------------------------------------------
 * No counterpart in the reference, which runs on one GPU: these shard the MoE (by experts) and the prompt GEMM (by
 * weight rows) over the GPUs of one node. A communicator wraps one NCCL rank on the device that is current at vkb_comm_init. Collective entry points must be
 * called by every rank, in the same order, with equal shapes and counts; they return an error instead of leaving a
 * peer waiting when a local launch fails after the argument checks. */
typedef struct vkb_comm vkb_comm_t;
#define VKB_UNIQUE_ID_BYTES 128
/* Rank 0 creates the id; the caller distributes the 128 bytes to every rank (any host channel). */
int vkb_comm_unique_id(void* id);
/* Collective over the ranks: creates the NCCL communicator and runs warm-up collectives (4 MiB per rank, a temporary
 * device buffer), so that NCCL's lazily created connection buffers exist before the first vkb call. */
int vkb_comm_init(vkb_comm_t** comm, int rank, int nranks, const void* id);
int vkb_comm_destroy(vkb_comm_t* comm);
int vkb_comm_rank(const vkb_comm_t* comm);
int vkb_comm_size(const vkb_comm_t* comm);
/* MoE, expert parallel: this rank holds experts [e0, e0 + E_local) (qpool / spool as in vkb_moe_q4); idx and x are
 * the full batch on every rank. After the call every rank's y [T][topk][N] holds every slot, bit-identical to one GPU
 * (each rank writes its slots and zeros elsewhere; an in-place ncclAllReduce sums the ranks). */
int vkb_moe_q4_ep(vkb_comm_t* comm, const void* qpool, const void* spool, const int32_t* idx, int T, int topk,
                  const void* x, void* y, int E_local, int e0, int N, int K, vkb_stream_t stream);
int vkb_moe_ep(vkb_comm_t* comm, int fmt, const void* qpool, const void* spool, const int32_t* idx, int T, int topk,
               const void* x, void* y, int out_f32, int E_local, int e0, int N, int K, vkb_stream_t stream);
/* Prompt GEMM, row split: this rank holds weight rows [r N/G, (r+1) N/G) (q_local, s_local in the vkb_gemm_q4_tc
 * layout, N/G rows); x [M][K] on every rank. After the call every rank's y [M][N] is the full product. work: device
 * memory of vkb_gemm_rowsplit_work_bytes(M, N, out_f32) bytes (caller-owned). N must be divisible by the rank count.
 * y is the one-GPU vkb_gemm_q4_tc result bit for bit (each rank's part uses the whole problem's split-K count). */
size_t vkb_gemm_rowsplit_work_bytes(int M, int N, int out_f32);
int vkb_gemm_q4_tc_rowsplit(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, void* y,
                            void* work, int N, int K, int M, vkb_stream_t stream);
int vkb_gemm_q4_tc_rowsplit_f32(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, float* y,
                                void* work, int N, int K, int M, vkb_stream_t stream);
/* vkb_gemm_q4_tc_rowsplit (fp16 y) with no workspace argument and no allocation, for callers that cannot allocate
 * device memory: a launcher with the reference harness's fixed contender signature, which has no workspace argument
 * (allocating inside it would put cudaMalloc / cudaFree, and cudaFree's device-wide synchronisation, into every
 * timed call), and a serving process whose device memory belongs to a pool reserved at start-up, where a cudaMalloc
 * either fails or takes memory the pool has promised elsewhere. The workspace is a static device array of the
 * library: 16 MiB on every GPU that loads libvkb.so, held until the process exits. The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress, with that device current; its error is returned): make
 * that first call before any stream capture. No counterpart in the reference. M * N * 2 must
 * not exceed VKB_ROWSPLIT_NOALLOC_MAX_BYTES (VKB_EUNSUPPORTED otherwise, nothing launched). Calls that overlap in time
 * on one device (other streams, host threads or communicators) share the array and race: serialise them. If the
 * array's lookup fails on one rank, that rank still joins the all-gather (through y) and returns the lookup error.
 * In every row-split entry point a null pointer on one rank is refused before the collective only when that rank has
 * neither y nor a workspace to join it with; with either, it joins and returns VKB_EINVAL. */
#define VKB_ROWSPLIT_NOALLOC_MAX_BYTES (16u << 20)
int vkb_gemm_q4_tc_rowsplit_noalloc(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, void* y,
                                    int N, int K, int M, vkb_stream_t stream);

/* ---- multi-GPU, fused: the exchange inside the kernel (peer stores over NVLink, no NCCL call) --------------------
 * Symmetric device buffers: collective, the same `bytes` on every rank; each rank's buffer is mapped into every peer
 * (CUDA IPC, exchanged over the communicator). The first allocation also makes the communicator's flags block (8448
 * bytes, mapped the same way). Freed by vkb_comm_free (collective) or vkb_comm_destroy. At most 8 ranks.
 * The fused calls below write every rank's copy of a symmetric y. Every rank makes the same fused calls on the
 * communicator in the same order; each call is numbered by an epoch kept in the flags block (device memory, so the
 * calls may be captured in a CUDA graph and replayed): a rank's copy is written only after that rank started the
 * call, and each rank's kernel ends only when every rank's part has arrived or is known to be missing.
 * A call refused on one rank only, after the checks every rank shares (a pointer that is not a symmetric buffer, an
 * unaligned operand, a failed launch there), returns its error code on that rank and still takes part in the call's
 * numbering with a small kernel; the other ranks' kernels then end at once with bit 8 (a peer's part is missing) in
 * vkb_device_status, and the next call is exact again. A rank whose own waits give up marks its part missing the same
 * way. vkb_comm_epoch: the number of the last fused call completed on this rank (0 before the first; read from device
 * memory: synchronise the streams of the fused calls first). */
int vkb_comm_alloc(vkb_comm_t* comm, size_t bytes, void** ptr);
int vkb_comm_free(vkb_comm_t* comm, void* ptr);
int vkb_comm_epoch(const vkb_comm_t* comm, unsigned int* epoch);
/* Row split with the all-gather fused into the GEMM: the tcgen05 epilogue stores this rank's columns of y straight
 * into every rank's copy of y_sym (>= M x N fp16). Same operands and result as vkb_gemm_q4_tc_rowsplit (the one-GPU
 * result bit for bit; with split-K each CTA pushes its finished token slice). */
int vkb_gemm_q4_tc_rowsplit_p2p(vkb_comm_t* comm, const void* q_local, const void* s_local, const void* x, void* y_sym,
                                int N, int K, int M, vkb_stream_t stream);
/* Expert-parallel MoE with the combine fused into the GEMV: each rank's kernel stores the slots of its own experts
 * straight into every rank's copy of y_sym (>= T*topk x N outputs); no zero slots, no all-reduce. Same operands and
 * result as vkb_moe_ep for every slot whose expert some rank holds (slots of an expert that no rank holds are not
 * written). Needs the pipelined kernel's shapes and alignment (K % 256 == 0, 16-byte aligned pools and x):
 * VKB_EUNSUPPORTED otherwise. */
int vkb_moe_ep_p2p(vkb_comm_t* comm, int fmt, const void* qpool, const void* spool, const int32_t* idx, int T,
                   int topk, const void* x, void* y_sym, int out_f32, int E_local, int e0, int N, int K,
                   vkb_stream_t stream);

/* ---- CUDA graphs of vkb calls ---------------------------------------------------------------------------------------
 * Capture a sequence of calls on a stream into one executable graph (a decode step: many short GEMVs) and replay it
 * with one launch; programmatic dependent launch edges between the captured kernels are kept. No counterpart in the
 * reference. begin: start capturing `stream` (thread-local mode); end: stop, instantiate, return the executable graph
 * handle; launch: replay on any stream; destroy: release. Return codes as above. */
int vkb_graph_begin(vkb_stream_t stream);
int vkb_graph_end(vkb_stream_t stream, void** graph_exec);
int vkb_graph_launch(void* graph_exec, vkb_stream_t stream);
int vkb_graph_destroy(void* graph_exec);

/* ---- status --------------------------------------------------------------------------------------------------------- */
/* Human-readable text of a return code. */
const char* vkb_strerror(int code);
/* Synchronises the current device, returns (and clears) the device-side status bits that kernels raise when a bounded
 * wait gives up (1 = pipeline wait timeout, 2 = drain timeout, 4 = peer timeout) or a peer rank reports its part of a
 * fused multi-GPU call missing (8). 0 = healthy. */
int vkb_device_status(unsigned int* bits);
/* Enable (1) or disable (0) programmatic dependent launch for later calls on this host thread; returns the old value. */
int vkb_set_pdl(int enable);
/* Library version, e.g. 100 for 0.1.0. */
int vkb_version(void);

/* ---- plan inspection -------------------------------------------------------------------------------------------------
 * The launch plan the library would use for a shape on a device with `sm_count` SMs and the given shared-memory
 * limits (bytes: per block with opt-in, per SM). Host only: no CUDA call, no device needed (tuning overrides in the
 * environment apply). Fills info[0 .. VKB_PLAN_INFO_LEN - 1]; returns 0, VKB_EUNSUPPORTED when the pipelined kernel
 * does not take the shape, or VKB_EINVAL. No counterpart in the reference, whose launchers fix their tiles at
 * compile time (src/stage2.cuh:217-229).
 *   kind 0, decode GEMV (fmt Q4 / Q8 / Q2, M = 1-8 tokens) and kind 2, gate + up over the stacked [2N][K] Q4 table:
 *     info = {smem, ring stages, stages per row tile, K values per stage, warp groups, stage bytes, grid, code pitch,
 *             scale pitch, row tiles}
 *   kind 1, prompt GEMM (fmt Q4 / Q8, any M), one CTA per tile:
 *     info = {smem, tokens per tile NT, 128-row blocks per tile, TMEM accumulators, A slots, first A column, TMEM
 *             columns, X stages, K steps per X stage, P chunks, K steps per P chunk, grid, tiles, X stage bytes,
 *             row tiles, CTAs per tile}
 *   kind 3, prompt GEMM as the entry points plan it, split-K included (Q4 tables with few row tiles: a cluster of
 *     CTAs shares each tile's K range; the cluster-occupancy limit is taken as sm_count / CTAs per cluster):
 *     the info of kind 1 with the last field = CTAs sharing a tile's K range (1: no split) */
#define VKB_PLAN_INFO_LEN 16
int vkb_plan_describe(int kind, int fmt, int N, int K, int M, int sm_count, int smem_optin, int smem_per_sm,
                      int* info);

#ifdef __cplusplus
}
#endif

#endif /* VKB_H */
