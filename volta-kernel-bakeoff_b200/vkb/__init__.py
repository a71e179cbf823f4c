"""Python binding of libvkb.so (include/vkb.h, include/vkb_host.h) over ctypes.

Two layers:
  * the raw C ABI (lib(), plain integers and pointers, return codes) -- what an FFI user of the library sees;
  * torch-tensor helpers (gemv(), moe(), quantize_pack(), ...) that validate devices, dtypes and shapes, pass the
    current CUDA stream, and raise VkbError on a non-zero return code.

There is no CPU fallback: every compute call goes to the CUDA kernels in libvkb.so, and importing a compute helper
without the built library raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG, "lib", "libvkb.so")

FMT_Q4, FMT_Q8, FMT_Q2 = 0, 1, 2
FMT_NAMES = {"q4": FMT_Q4, "q8": FMT_Q8, "q2": FMT_Q2}
BITS = {FMT_Q4: 4, FMT_Q8: 8, FMT_Q2: 2}
OK, EUNSUPPORTED, EINVAL, ENOCOMM, EDEVICE = 0, 1, 2, 3, 4

_lib = None


class VkbError(RuntimeError):
    def __init__(self, code: int, where: str = ""):
        self.code = code
        super().__init__(f"{where}: vkb error {code}: {strerror(code)}")


def lib() -> ctypes.CDLL:
    """Load libvkb.so (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with python volta-kernel-bakeoff_b200/build.py")
    # libvkb.so needs libnccl.so.2. When torch is installed, load it first: its bundled (newer) NCCL then serves both;
    # loaded the other way round, the system NCCL would be bound first and torch's import would miss symbols.
    try:
        import torch  # noqa: F401
    except ImportError:
        pass
    L = ctypes.CDLL(LIB_PATH)
    vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    for name in ("vkb_gemv_q4", "vkb_gemv_q8", "vkb_gemv_q2", "vkb_gemv_q4_f32", "vkb_gemv_q8_f32", "vkb_gemv_q2_f32"):
        f = getattr(L, name)
        f.argtypes = [vp, vp, vp, vp, i, i, i, vp]
        f.restype = i
    L.vkb_gemv.argtypes = [i, vp, vp, vp, vp, i, i, i, i, vp]
    L.vkb_gemv.restype = i
    L.vkb_moe_q4.argtypes = [vp, vp, vp, i, i, vp, vp, i, i, i, i, vp]
    L.vkb_moe_q4.restype = i
    L.vkb_moe.argtypes = [i, vp, vp, vp, i, i, vp, vp, i, i, i, i, i, vp]
    L.vkb_moe.restype = i
    L.vkb_strerror.argtypes = [i]
    L.vkb_strerror.restype = ctypes.c_char_p
    L.vkb_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    L.vkb_device_status.restype = i
    L.vkb_set_pdl.argtypes = [i]
    L.vkb_set_pdl.restype = i
    L.vkb_version.argtypes = []
    L.vkb_version.restype = i
    L.vkb_quantize.argtypes = [i, vp, i, i, vp, vp]
    L.vkb_quantize.restype = i
    L.vkb_pack.argtypes = [i, vp, i, i, i, vp]
    L.vkb_pack.restype = i
    L.vkb_packed_bytes.argtypes = [i, i, i]
    L.vkb_packed_bytes.restype = sz
    L.vkb_synth_normal.argtypes = [ctypes.c_uint32, sz, ctypes.c_float, vp]
    L.vkb_synth_normal.restype = i
    L.vkb_f32_to_f16.argtypes = [vp, sz, vp]
    L.vkb_f32_to_f16.restype = i
    L.vkb_synth_topk.argtypes = [ctypes.c_uint32, i, i, i, vp]
    L.vkb_synth_topk.restype = i
    _register_optional(L)
    _lib = L
    return L


def _register_optional(L) -> None:
    """Entry points added by later parts of the library (bound when present)."""
    vp, i = ctypes.c_void_p, ctypes.c_int
    opt = {
        "vkb_gemm_q4_tc": ([vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gemm_q4_tc_f32": ([vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_comm_unique_id": ([vp], i),
        "vkb_comm_init": ([ctypes.POINTER(vp), i, i, vp], i),
        "vkb_comm_destroy": ([vp], i),
        "vkb_comm_rank": ([vp], i),
        "vkb_comm_size": ([vp], i),
        "vkb_moe_q4_ep": ([vp, vp, vp, vp, i, i, vp, vp, i, i, i, i, vp], i),
        "vkb_moe_ep": ([vp, i, vp, vp, vp, i, i, vp, vp, i, i, i, i, i, vp], i),
        "vkb_gemm_rowsplit_work_bytes": ([i, i, i], ctypes.c_size_t),
        "vkb_gemm_q4_tc_rowsplit": ([vp, vp, vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gemm_q4_tc_rowsplit_f32": ([vp, vp, vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gemm_q4_tc_rowsplit_noalloc": ([vp, vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_comm_alloc": ([vp, ctypes.c_size_t, ctypes.POINTER(vp)], i),
        "vkb_comm_free": ([vp, vp], i),
        "vkb_comm_epoch": ([vp, ctypes.POINTER(ctypes.c_uint)], i),
        "vkb_gemm_q4_tc_rowsplit_p2p": ([vp, vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_moe_ep_p2p": ([vp, i, vp, vp, vp, i, i, vp, vp, i, i, i, i, i, vp], i),
        "vkb_gemv_q4_f32in": ([vp, vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gemm_tc": ([i, vp, vp, vp, vp, i, i, i, i, vp], i),
        "vkb_gemm_q8_tc": ([vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gemm_q8_tc_f32": ([vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gguf_to_vkb_device": ([i, vp, i, i, vp, vp, vp], i),
        "vkb_dequant": ([i, vp, vp, vp, i, i, i, vp], i),
        "vkb_gguf_bytes": ([i, i, i], ctypes.c_size_t),
        "vkb_gguf_to_vkb": ([i, vp, i, i, vp, vp], i),
        "vkb_vkb_to_gguf": ([i, vp, vp, i, i, vp], i),
        "vkb_gate_up_glu_q4_f32in": ([vp, vp, vp, vp, vp, vp, i, i, i, vp], i),
        "vkb_gate_up_glu_q4": ([vp, vp, vp, vp, vp, i, i, i, i, vp], i),
        "vkb_graph_begin": ([vp], i),
        "vkb_graph_end": ([vp, ctypes.POINTER(vp)], i),
        "vkb_graph_launch": ([vp, vp], i),
        "vkb_graph_destroy": ([vp], i),
        "vkb_plan_describe": ([i, i, i, i, i, i, i, i, vp], i),
    }
    for name, (args, res) in opt.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res


# B200: 148 SMs, 227 KB of shared memory per block (opt-in), 228 KB per SM
B200_LIMITS = {"sm_count": 148, "smem_optin": 232448, "smem_per_sm": 233472}
PLAN_GEMV, PLAN_TC, PLAN_GLU, PLAN_TC_SPLIT = 0, 1, 2, 3
_PLAN_FIELDS = {
    PLAN_GEMV: ("smem", "nstage", "nchunks", "KS", "wg", "stage_bytes", "grid", "cpitch", "spitch", "tiles"),
    PLAN_GLU: ("smem", "nstage", "nchunks", "KS", "wg", "stage_bytes", "grid", "cpitch", "spitch", "tiles"),
    PLAN_TC: ("smem", "NT", "rb", "nacc", "na", "a_col0", "tmem_cols", "nx", "xk", "np", "pk", "grid", "tiles",
              "x_stage", "tiles_n", "cg"),
    PLAN_TC_SPLIT: ("smem", "NT", "rb", "nacc", "na", "a_col0", "tmem_cols", "nx", "xk", "np", "pk", "grid", "tiles",
                    "x_stage", "tiles_n", "splits"),
}


def plan(kind: int, fmt: int, N: int, K: int, M: int, sm_count: int = 148, smem_optin: int = 232448,
         smem_per_sm: int = 233472) -> dict | None:
    """The launch plan the library would use (vkb_plan_describe; host only, no device needed): a dict of named
    fields, or None when the pipelined kernel does not take the shape."""
    info = (ctypes.c_int * 16)()
    rc = lib().vkb_plan_describe(kind, fmt, N, K, M, sm_count, smem_optin, smem_per_sm, ctypes.cast(info,
                                                                                                     ctypes.c_void_p))
    if rc == EUNSUPPORTED:
        return None
    check(rc, "vkb_plan_describe")
    return dict(zip(_PLAN_FIELDS[kind], info))


def strerror(code: int) -> str:
    try:
        return lib().vkb_strerror(code).decode()
    except ImportError:
        return "libvkb.so not loaded"


def check(rc: int, where: str = "vkb") -> None:
    if rc != 0:
        raise VkbError(rc, where)


def device_status() -> int:
    bits = ctypes.c_uint(0)
    check(lib().vkb_device_status(ctypes.byref(bits)), "vkb_device_status")
    return bits.value


def set_pdl(enable: bool) -> bool:
    return bool(lib().vkb_set_pdl(1 if enable else 0))


# ---- host-side formats (numpy) ----------------------------------------------------------------------------------

def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def synth_normal(seed: int, shape, std: float) -> np.ndarray:
    out = np.empty(int(np.prod(shape)), np.float32)
    check(lib().vkb_synth_normal(seed, out.size, std, _p(out)), "vkb_synth_normal")
    return out.reshape(shape)


def to_f16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, np.uint16)
    check(lib().vkb_f32_to_f16(_p(a), a.size, _p(out)), "vkb_f32_to_f16")
    return out


def quantize(fmt: int, w: np.ndarray):
    """fp32 [N][K] -> (codes int8 [N][K], scales uint16 fp16 bits [N][K/32])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    codes = np.empty((N, K), np.int8)
    scales = np.empty((N, K // 32), np.uint16)
    check(lib().vkb_quantize(fmt, _p(w), N, K, _p(codes), _p(scales)), "vkb_quantize")
    return codes, scales


def pack(fmt: int, codes: np.ndarray, sabotage: bool = False) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    N, K = codes.shape
    if fmt == FMT_Q8:
        out = np.empty((N, K), np.int8)
    else:
        out = np.empty((N, K * BITS[fmt] // 32), np.uint32)
    check(lib().vkb_pack(fmt, _p(codes), N, K, int(sabotage), _p(out)), "vkb_pack")
    return out


def synth_topk(seed: int, T: int, E: int, k: int) -> np.ndarray:
    idx = np.empty((T, k), np.int32)
    check(lib().vkb_synth_topk(seed, T, E, k, _p(idx)), "vkb_synth_topk")
    return idx


# ---- torch helpers ----------------------------------------------------------------------------------------------

def _torch():
    import torch
    return torch


def _stream(stream=None) -> ctypes.c_void_p:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _optr(t) -> ctypes.c_void_p | None:
    """_ptr, or a null pointer for None (optional outputs)."""
    return None if t is None else _ptr(t)


def gemv(fmt: int, q, s, x, y=None, out_f32: bool = False, stream=None):
    """y[M][N] = x[M][K] . W[N][K]^T for M <= 8. q: packed codes (uint8/int8/int32 storage), s: fp16 [N][K/32],
    x: fp16 [M][K] on the same CUDA device. Returns y (fp16, or fp32 with out_f32)."""
    torch = _torch()
    M, K = x.shape
    N = s.shape[0]
    if y is None:
        y = torch.empty((M, N), dtype=torch.float32 if out_f32 else torch.float16, device=x.device)
    rc = lib().vkb_gemv(fmt, _ptr(q), _ptr(s), _ptr(x), _ptr(y), int(out_f32), N, K, M, _stream(stream))
    check(rc, "vkb_gemv")
    return y


def gemv_q4_f32in(q, s, x, xh=None, y=None, stream=None):
    """Q4 decode with fp32 activations x [M][K] (rounded to fp16, round to nearest even): y fp32 [M][N]. xh: fp16
    scratch of M x K, used when the kernel cannot stage the fp32 activations itself (allocated here if not given)."""
    torch = _torch()
    M, K = x.shape
    N = s.shape[0]
    if y is None:
        y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    if xh is None:
        xh = torch.empty((M, K), dtype=torch.float16, device=x.device)
    check(lib().vkb_gemv_q4_f32in(_ptr(q), _ptr(s), _ptr(x), _ptr(xh), _ptr(y), N, K, M, _stream(stream)),
          "vkb_gemv_q4_f32in")
    return y


def gate_up_glu_q4(q, s, x, ystack=None, out=None, out_f32: bool = True, want_stack: bool = True, xh=None,
                   stream=None):
    """Gate + up + SwiGLU: q, s the stacked [2N][K] Q4 table (gate rows, then up rows), x [M][K] fp32 (the
    reference's fp32-in entry) or fp16. Returns (out [M][N] = silu(gate) * up, ystack [M][2N] fp32 or None)."""
    torch = _torch()
    M, K = x.shape
    N = s.shape[0] // 2
    if want_stack and ystack is None:
        ystack = torch.empty((M, 2 * N), dtype=torch.float32, device=x.device)
    if x.dtype == torch.float32:
        if out is None:
            out = torch.empty((M, N), dtype=torch.float32, device=x.device)
        if xh is None:
            xh = torch.empty((M, K), dtype=torch.float16, device=x.device)
        rc = lib().vkb_gate_up_glu_q4_f32in(_ptr(q), _ptr(s), _ptr(x), _ptr(xh), _optr(ystack), _ptr(out), N, K, M,
                                            _stream(stream))
        check(rc, "vkb_gate_up_glu_q4_f32in")
    else:
        if out is None:
            out = torch.empty((M, N), dtype=torch.float32 if out_f32 else torch.float16, device=x.device)
        rc = lib().vkb_gate_up_glu_q4(_ptr(q), _ptr(s), _ptr(x), _optr(ystack), _ptr(out),
                                      int(out.dtype == torch.float32), N, K, M, _stream(stream))
        check(rc, "vkb_gate_up_glu_q4")
    return out, ystack


def gguf_to_vkb(fmt: int, blocks: np.ndarray, N: int, K: int) -> tuple[np.ndarray, np.ndarray]:
    """Host: GGUF Q4_0 / Q8_0 blocks (uint8, N * K/32 blocks) -> (packed codes uint8, fp16 scale bits uint16 [N][K/32])."""
    q = np.zeros(lib().vkb_packed_bytes(fmt, N, K), dtype=np.uint8)
    s = np.zeros((N, K // 32), dtype=np.uint16)
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    check(lib().vkb_gguf_to_vkb(fmt, b.ctypes.data, N, K, q.ctypes.data, s.ctypes.data), "vkb_gguf_to_vkb")
    return q, s


def vkb_to_gguf(fmt: int, q: np.ndarray, s: np.ndarray, N: int, K: int) -> np.ndarray:
    """Host: packed codes + fp16 scale bits -> GGUF Q4_0 / Q8_0 blocks (uint8)."""
    out = np.zeros(lib().vkb_gguf_bytes(fmt, N, K), dtype=np.uint8)
    qc, sc = np.ascontiguousarray(q), np.ascontiguousarray(s, dtype=np.uint16)
    check(lib().vkb_vkb_to_gguf(fmt, qc.ctypes.data, sc.ctypes.data, N, K, out.ctypes.data), "vkb_vkb_to_gguf")
    return out


def gguf_to_vkb_device(fmt: int, blocks, N: int, K: int, stream=None):
    """Device: GGUF blocks (a uint8 CUDA tensor) -> (packed codes, fp16 scales) CUDA tensors, one kernel."""
    torch = _torch()
    q = torch.empty(lib().vkb_packed_bytes(fmt, N, K), dtype=torch.uint8, device=blocks.device)
    s = torch.empty((N, K // 32), dtype=torch.float16, device=blocks.device)
    check(lib().vkb_gguf_to_vkb_device(fmt, _ptr(blocks), N, K, _ptr(q), _ptr(s), _stream(stream)),
          "vkb_gguf_to_vkb_device")
    return q, s


def dequant(fmt: int, q, s, N: int, K: int, bf16: bool = False, w=None, stream=None):
    """Device: packed weights -> a dense fp16 (or bf16) [N][K] tensor, code * scale rounded once (vkb_dequant)."""
    torch = _torch()
    if w is None:
        w = torch.empty((N, K), dtype=torch.bfloat16 if bf16 else torch.float16, device=q.device)
    check(lib().vkb_dequant(fmt, _ptr(q), _ptr(s), _ptr(w), N, K, int(bf16), _stream(stream)), "vkb_dequant")
    return w


def moe(fmt: int, qpool, spool, idx, x, y=None, E_local: int | None = None, e0: int = 0, out_f32: bool = False,
        stream=None):
    """MoE decode: qpool [E_local][N][...], spool [E_local][N][K/32] fp16, idx int32 [T][topk], x fp16 [T][K] ->
    y [T][topk][N] (slots of non-local experts untouched)."""
    torch = _torch()
    E, N = spool.shape[0], spool.shape[1]
    T, topk = idx.shape
    K = x.shape[1]
    if y is None:
        y = torch.zeros((T, topk, N), dtype=torch.float32 if out_f32 else torch.float16, device=x.device)
    rc = lib().vkb_moe(fmt, _ptr(qpool), _ptr(spool), _ptr(idx), T, topk, _ptr(x), _ptr(y), int(out_f32),
                       E if E_local is None else E_local, e0, N, K, _stream(stream))
    check(rc, "vkb_moe")
    return y


def gemm_tc(q, s, x, y=None, out_f32: bool = False, stream=None, fmt: int = FMT_Q4):
    """Prompt GEMM on tcgen05: y[M][N] = x[M][K] . W[N][K]^T for any M. q: packed Q4 codes (or int8 Q8 codes with
    fmt=FMT_Q8), s: fp16 [N][K/32], x: fp16 [M][K]. Returns y (fp16, or fp32 with out_f32)."""
    torch = _torch()
    M, K = x.shape
    N = s.shape[0]
    if y is None:
        y = torch.empty((M, N), dtype=torch.float32 if out_f32 else torch.float16, device=x.device)
    if fmt == FMT_Q4:
        fn = lib().vkb_gemm_q4_tc_f32 if out_f32 else lib().vkb_gemm_q4_tc
        check(fn(_ptr(q), _ptr(s), _ptr(x), _ptr(y), N, K, M, _stream(stream)), "vkb_gemm_q4_tc")
    else:
        check(lib().vkb_gemm_tc(fmt, _ptr(q), _ptr(s), _ptr(x), _ptr(y), int(out_f32), N, K, M, _stream(stream)),
              "vkb_gemm_tc")
    return y


class Graph:
    """A CUDA graph of vkb calls captured on a stream through the C ABI (vkb_graph_*): replay() launches them all at
    once. Used like torch.cuda.graph, without torch's per-replay generator bookkeeping."""

    def __init__(self, stream=None):
        self.stream = stream
        self._h = ctypes.c_void_p()

    def __enter__(self):
        check(lib().vkb_graph_begin(_stream(self.stream)), "vkb_graph_begin")
        return self

    def __exit__(self, exc_type, exc, tb):
        h = ctypes.c_void_p()
        rc = lib().vkb_graph_end(_stream(self.stream), ctypes.byref(h))
        if exc_type is None:
            check(rc, "vkb_graph_end")
            self._h = h
        return False

    def replay(self, stream=None):
        check(lib().vkb_graph_launch(self._h, _stream(stream if stream is not None else self.stream)),
              "vkb_graph_launch")

    def __del__(self):
        try:
            if self._h:
                lib().vkb_graph_destroy(self._h)
        except Exception:
            pass


def to_device_packed(packed: np.ndarray, device="cuda"):
    """numpy packed codes -> a torch uint8 tensor with the same bytes (kept 2-D: [rows][bytes per row])."""
    torch = _torch()
    b = np.ascontiguousarray(packed).view(np.uint8).reshape(packed.shape[0], -1)
    return torch.from_numpy(b.copy()).to(device)


def to_device_f16(bits: np.ndarray, device="cuda"):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).to(device).view(torch.float16)
