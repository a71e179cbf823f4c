"""Multi-GPU side of the binding: one process (one NCCL rank) per GPU.

  * partition helpers -- the contiguous expert ranges of expert parallelism and the weight-row ranges of the row-split
    prompt GEMM, shared by the library's callers, the tests and bench.py;
  * Comm -- a libvkb communicator (vkb_comm_init) whose NCCL unique id travels over an existing torch.distributed
    process group (gloo or nccl), with the expert-parallel MoE and row-split prompt GEMM calls on torch tensors.

The combine steps live in libvkb.so (vkb_moe_ep: in-place all-reduce of zero-filled slots; vkb_gemm_q4_tc_rowsplit:
in-place all-gather of [M][N/G] blocks plus a permute kernel). combine_* below restate them on the host for the CPU
tests of the decomposition.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import check, lib, _ptr, _stream, FMT_Q4

UNIQUE_ID_BYTES = 128


def expert_range(E: int, G: int, r: int) -> tuple[int, int]:
    """(e0, E_local) of rank r when E experts are split into G contiguous ranges (the first E % G ranks hold one
    more)."""
    if not (0 <= r < G) or E < G:
        raise ValueError(f"cannot split {E} experts over {G} ranks")
    base, extra = divmod(E, G)
    e0 = r * base + min(r, extra)
    return e0, base + (1 if r < extra else 0)


def row_range(N: int, G: int, r: int) -> tuple[int, int]:
    """(n0, N_local) of rank r in the row-split prompt GEMM (N must be divisible by G)."""
    if N % G != 0 or not (0 <= r < G):
        raise ValueError(f"{N} rows do not split over {G} ranks")
    nl = N // G
    return r * nl, nl


def combine_moe_slots(per_rank: list[np.ndarray]) -> np.ndarray:
    """Host statement of the expert-parallel combine: every rank's [T][k][N] slots (own experts' values, zeros
    elsewhere) summed -- exact, since each slot has one non-zero contributor."""
    out = np.zeros_like(per_rank[0])
    for y in per_rank:
        out = out + y
    return out


def combine_rowsplit(blocks: list[np.ndarray]) -> np.ndarray:
    """Host statement of the row-split combine: the gathered [G][M][N/G] blocks permuted into y [M][N]
    (y[m][g N/G + n] = work[g][m][n])."""
    work = np.stack(blocks)                       # [G][M][nl]
    G, M, nl = work.shape
    return work.transpose(1, 0, 2).reshape(M, G * nl)


class Comm:
    """A libvkb communicator on the current CUDA device."""

    def __init__(self, rank: int, size: int, unique_id: bytes):
        self.rank, self.size = rank, size
        self._h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), UNIQUE_ID_BYTES)
        check(lib().vkb_comm_init(ctypes.byref(self._h), rank, size, buf), "vkb_comm_init")

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
        check(lib().vkb_comm_unique_id(buf), "vkb_comm_unique_id")
        return buf.raw

    @classmethod
    def from_torch(cls, group=None) -> "Comm":
        """Every rank of an initialised torch.distributed group calls this; rank 0's unique id is broadcast."""
        import torch.distributed as dist
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(rank, size, obj[0])

    def close(self) -> None:
        if self._h:
            check(lib().vkb_comm_destroy(self._h), "vkb_comm_destroy")
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def moe_ep(self, qpool, spool, idx, x, E_local: int, e0: int, y=None, fmt: int = FMT_Q4, out_f32: bool = False,
               stream=None):
        """Expert-parallel MoE: this rank's experts [e0, e0 + E_local) in qpool / spool; idx [T][k] and x [T][K] the
        whole batch. Returns y [T][k][N] with every slot, on every rank."""
        import torch
        N = spool.shape[1]
        T, topk = idx.shape
        K = x.shape[1]
        if y is None:
            y = torch.empty((T, topk, N), dtype=torch.float32 if out_f32 else torch.float16, device=x.device)
        rc = lib().vkb_moe_ep(self._h, fmt, _ptr(qpool), _ptr(spool), _ptr(idx), T, topk, _ptr(x), _ptr(y),
                              int(out_f32), E_local, e0, N, K, _stream(stream))
        check(rc, "vkb_moe_ep")
        return y

    def moe_ep_p2p(self, qpool, spool, idx, x, E_local: int, e0: int, y_sym: "SymTensor", fmt: int = FMT_Q4,
                   stream=None):
        """Expert-parallel MoE with the combine fused into the kernel (peer stores over NVLink): y_sym (from alloc,
        [T][k][N], fp16 or fp32) holds every slot on every rank after the call."""
        import torch
        N = spool.shape[1]
        T, topk = idx.shape
        K = x.shape[1]
        rc = lib().vkb_moe_ep_p2p(self._h, fmt, _ptr(qpool), _ptr(spool), _ptr(idx), T, topk, _ptr(x), y_sym.ptr,
                                  int(y_sym.dtype == torch.float32), E_local, e0, N, K, _stream(stream))
        check(rc, "vkb_moe_ep_p2p")
        return y_sym

    def epoch(self) -> int:
        """The number of the last fused (peer-store) call completed on this rank (vkb_comm_epoch; synchronise first)."""
        e = ctypes.c_uint(0)
        check(lib().vkb_comm_epoch(self._h, ctypes.byref(e)), "vkb_comm_epoch")
        return e.value

    def alloc(self, shape, dtype):
        """A symmetric tensor (collective: same shape on every rank): this rank's buffer, mapped into every peer, for
        the fused peer-store calls. Freed with free()."""
        import torch
        nbytes = int(np.prod(shape)) * torch.tensor([], dtype=dtype).element_size()
        p = ctypes.c_void_p()
        check(lib().vkb_comm_alloc(self._h, nbytes, ctypes.byref(p)), "vkb_comm_alloc")
        return SymTensor(self, p, shape, dtype)

    def gemm_rowsplit_p2p(self, q_local, s_local, x, N: int, y_sym: "SymTensor", stream=None):
        """Row-split prompt GEMM with the all-gather fused into the epilogue (peer stores over NVLink): y_sym (from
        alloc, [M][N] fp16) holds the full product on every rank after the call."""
        M, K = x.shape
        check(lib().vkb_gemm_q4_tc_rowsplit_p2p(self._h, _ptr(q_local), _ptr(s_local), _ptr(x), y_sym.ptr, N, K, M,
                                                 _stream(stream)), "vkb_gemm_q4_tc_rowsplit_p2p")
        return y_sym

    def gemm_rowsplit(self, q_local, s_local, x, N: int, y=None, work=None, out_f32: bool = False, stream=None):
        """Row-split prompt GEMM: q_local / s_local hold this rank's N/G weight rows. Returns y [M][N] on every
        rank."""
        import torch
        M, K = x.shape
        dt = torch.float32 if out_f32 else torch.float16
        if y is None:
            y = torch.empty((M, N), dtype=dt, device=x.device)
        if work is None:
            nbytes = lib().vkb_gemm_rowsplit_work_bytes(M, N, int(out_f32))
            work = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        fn = lib().vkb_gemm_q4_tc_rowsplit_f32 if out_f32 else lib().vkb_gemm_q4_tc_rowsplit
        check(fn(self._h, _ptr(q_local), _ptr(s_local), _ptr(x), _ptr(y), _ptr(work), N, K, M, _stream(stream)),
              "vkb_gemm_q4_tc_rowsplit")
        return y


class SymTensor:
    """A symmetric device buffer of a communicator, viewed as a torch tensor (tensor())."""

    def __init__(self, comm: Comm, ptr: ctypes.c_void_p, shape, dtype):
        self.comm, self.ptr, self.shape, self.dtype = comm, ptr, tuple(shape), dtype

    def tensor(self):
        """A torch view of the buffer (no copy; valid until free())."""
        import torch
        n = int(np.prod(self.shape))
        esz = torch.tensor([], dtype=self.dtype).element_size()
        iface = {"shape": (n * esz,), "typestr": "|u1", "data": (self.ptr.value, False), "version": 3}
        holder = type("_CudaArray", (), {"__cuda_array_interface__": iface})()
        return torch.as_tensor(holder, device="cuda").view(self.dtype).view(self.shape)

    def free(self):
        if self.ptr:
            check(lib().vkb_comm_free(self.comm._h, self.ptr), "vkb_comm_free")
            self.ptr = ctypes.c_void_p()
