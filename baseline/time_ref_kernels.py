"""Same-GPU comparison: the reference's own kernels (rebuilt for sm_100a into baseline/_ref/librefkernels.so by
baseline/Makefile) against this library's kernels and cuBLAS bf16, on the same weights, timed the same way.

    python baseline/time_ref_kernels.py [--quick]      (prints one JSON object)

Run by bench.py in a child process: the reference's CK macro exits the process on a CUDA error (src/bakeoff.cu:43-46).

Cases (weights N(0,0.02) seed 0 quantised per 32, activations fp16 N(0,1)):
  decode    configs[0] (Q4 8192x2048) and configs[1] (Q4/Q8/2-bit x 12288x2560, 2560x6144, 6144x2048, 2048x6144) at
            1/2/4/8 tokens: ours (vkb_gemv, fp16 out) against fused_q4_v2w and fused_q4_v3 (Q4), fused_q8 (Q8),
            q2w_alu_v3 (2-bit, 1 token: the only count it has), and cuBLAS bf16 (torch.matmul, bf16 weights);
  moe       configs[2]/[3] at 1 token (the reference's one-launch MoE takes one token per expert, E <= 16): 8 experts of
            512x2048 and 10 of 640x2560, ours (vkb_moe) against moe_fused_q4;
  prompt    configs[4]: Q4 12288x2560 and 8192x2048 at 64 and 512 tokens, ours (vkb_gemm_q4_tc) against tc_q4 and
            tc_q4_v2 (the reference's prompt bar) and cuBLAS bf16.
Timing: every contender's 50 calls captured in one CUDA graph, median of 5 replays (the reference's time_us without
host launch cost); every contender cycles weight copies spanning >= 4x the L2. "agree": max |y_ref - y_ours| /
max |y_ours| on one call, a sanity check that the timed reference kernel computes the same product.
"""
from __future__ import annotations

import ctypes
import json
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "volta-kernel-bakeoff_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)
LIB = os.path.join(HERE, "_ref", "librefkernels.so")

RK_FUSED_Q4_V2W, RK_FUSED_Q8, RK_Q2W_ALU_V3, RK_FUSED_Q4_V3, RK_TC_Q4, RK_TC_Q4_V2 = range(6)
DECODE_TABLES = [(8192, 2048), (12288, 2560), (2560, 6144), (6144, 2048), (2048, 6144)]
FORMATS = [("q4", 0, [("fused_q4_v2w", RK_FUSED_Q4_V2W), ("fused_q4_v3", RK_FUSED_Q4_V3)]),
           ("q8", 1, [("fused_q8", RK_FUSED_Q8)]),
           ("q2", 2, [("q2w_alu_v3", RK_Q2W_ALU_V3)])]
TOKENS = [1, 2, 4, 8]
MOE = [("qwen36_gate_up_128x512x2048_top8", 128, 8, 512, 2048), ("flashnext_gate_up_160x640x2560_top10", 160, 10,
                                                                   640, 2560)]
PROMPT = [(12288, 2560), (8192, 2048)]
PROMPT_TOKENS = [64, 512]


def load():
    if not os.path.exists(LIB):
        return None
    L = ctypes.CDLL(LIB)
    vp, i, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
    L.ref_kernel_run.argtypes = [i, i, vp, vp, vp, vp, i, i]
    L.ref_kernel_run.restype = i
    L.ref_kernel_time_us.argtypes = [i, i, vp, vp, i, vp, vp, i, i]
    L.ref_kernel_time_us.restype = d
    L.ref_moe_run.argtypes = [i, vp, vp, vp, ctypes.c_longlong, vp, i, i]
    L.ref_moe_run.restype = i
    L.ref_moe_time_us.argtypes = [i, vp, vp, i, vp, ctypes.c_longlong, vp, i, i]
    L.ref_moe_time_us.restype = d
    return L


def _ptrs(tensors):
    arr = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
    return arr


def _copies(nbytes: int, L2: int) -> int:
    return max(2, math.ceil(4 * L2 / max(1, nbytes)))


def _graph_us(torch, vkb, stream, run, vkb_graph=True) -> float:
    """Median us per call over 5 replays of a 50-call CUDA graph (run(i) issues call i)."""
    for i in range(20):
        run(i)
    torch.cuda.synchronize()
    g = vkb.Graph(stream) if vkb_graph else torch.cuda.CUDAGraph()
    with (g if vkb_graph else torch.cuda.graph(g, stream=stream)):
        for i in range(50):
            run(20 + i)
    g.replay()
    ts = []
    for _ in range(5):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1000.0 / 50)
    del g
    return sorted(ts)[2]


def _agree(y_ref, y_ours) -> float:
    yo = y_ours.float()
    return float((y_ref.float() - yo).abs().max() / yo.abs().max().clamp_min(1e-30))


def main(quick: bool = False) -> dict:
    import torch
    import vkb
    L = load()
    if L is None:
        return {"unavailable": f"{os.path.relpath(LIB, ROOT)} not built (make -f baseline/Makefile REF=...)"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    L2 = torch.cuda.get_device_properties(dev).L2_cache_size
    out = {"decode": {}, "moe": {}, "prompt": {}}
    tables = DECODE_TABLES[:2] if quick else DECODE_TABLES
    for N, K in tables:
        wb = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        nb = _copies(wb.numel() * 2, L2)
        wl = [wb] + [wb.clone() for _ in range(nb - 1)]
        cub = {}
        for M in TOKENS:
            xb = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            yb = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            cub[M] = _graph_us(torch, vkb, stream, lambda i: torch.matmul(xb, wl[i % nb].t(), out=yb), vkb_graph=False)
        del wl, wb
        for fname, fmt, refs in FORMATS:
            if (N, K) == (8192, 2048) and fmt != 0:
                continue   # configs[0] is Q4 only
            codes, scales = vkb.quantize(fmt, vkb.synth_normal(0, (N, K), 0.02))
            q0 = vkb.to_device_packed(vkb.pack(fmt, codes), dev)
            s0 = vkb.to_device_f16(scales, dev)
            n = _copies(q0.numel() + 2 * s0.numel(), L2)
            ql = [q0] + [q0.clone() for _ in range(n - 1)]
            sl = [s0] + [s0.clone() for _ in range(n - 1)]
            qp, sp = _ptrs(ql), _ptrs(sl)
            for M in TOKENS:
                x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(1 + M, (M, K), 1.0)), dev)
                y = torch.empty((M, N), dtype=torch.float16, device=dev)
                yf = torch.empty((M, N), dtype=torch.float32, device=dev)
                ours = _graph_us(torch, vkb, stream, lambda i: vkb.gemv(fmt, ql[i % n], sl[i % n], x, y=y))
                vkb.gemv(fmt, q0, s0, x, y=yf, out_f32=True)
                torch.cuda.synchronize()
                rec = {"us": round(ours, 3), "cublas_bf16_us": round(cub[M], 3)}
                for rname, kind in refs:
                    yr = torch.zeros((M, N), dtype=torch.float32, device=dev)
                    if L.ref_kernel_run(kind, M, q0.data_ptr(), s0.data_ptr(), x.data_ptr(), yr.data_ptr(), N, K):
                        continue   # the reference kernel has no such token count
                    us = L.ref_kernel_time_us(kind, M, qp, sp, n, x.data_ptr(), yr.data_ptr(), N, K)
                    rec[rname] = {"us": round(us, 3), "speedup": round(us / ours, 2), "agree": _agree(yr, yf)}
                out["decode"][f"{fname}_{N}x{K}_m{M}"] = rec
            del ql, sl
    for name, E, k, N, K in MOE:
        codes, scales = vkb.quantize(0, vkb.synth_normal(7, (E * N, K), 0.02))
        q0 = vkb.to_device_packed(vkb.pack(0, codes), dev).view(E, N, -1)
        s0 = vkb.to_device_f16(scales, dev).view(E, N, K // 32)
        n = _copies(q0.numel() + 2 * s0.numel(), L2)
        ql = [q0] + [q0.clone() for _ in range(n - 1)]
        sl = [s0] + [s0.clone() for _ in range(n - 1)]
        idx_np = vkb.synth_topk(12, 1, E, k)
        sel = [int(e) for e in idx_np[0]]
        idx = torch.from_numpy(idx_np).to(dev)
        x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(13, (1, K), 1.0)), dev)
        y = torch.empty((1, k, N), dtype=torch.float16, device=dev)
        yf = torch.empty((1, k, N), dtype=torch.float32, device=dev)
        ours = _graph_us(torch, vkb, stream, lambda i: vkb.moe(0, ql[i % n], sl[i % n], idx, x, y=y))
        vkb.moe(0, q0, s0, idx, x, y=yf, out_f32=True)
        # the reference's MoePtrs: the host picks each selected expert's pointers (copy c, expert j at c * k + j)
        qe = _ptrs([ql[c][e] for c in range(n) for e in sel])
        se = _ptrs([sl[c][e] for c in range(n) for e in sel])
        yr = torch.zeros((k, N), dtype=torch.float32, device=dev)
        L.ref_moe_run(k, qe, se, x.data_ptr(), 0, yr.data_ptr(), N, K)
        us = L.ref_moe_time_us(k, qe, se, n, x.data_ptr(), 0, yr.data_ptr(), N, K)
        out["moe"][f"{name}_t1"] = {"us": round(ours, 3), "moe_fused_q4": {
            "us": round(us, 3), "speedup": round(us / ours, 2), "agree": _agree(yr, yf.view(k, N))}}
        del ql, sl
    for N, K in PROMPT:
        codes, scales = vkb.quantize(0, vkb.synth_normal(0, (N, K), 0.02))
        q0 = vkb.to_device_packed(vkb.pack(0, codes), dev)
        s0 = vkb.to_device_f16(scales, dev)
        n = _copies(q0.numel() + 2 * s0.numel(), L2)
        ql = [q0] + [q0.clone() for _ in range(n - 1)]
        sl = [s0] + [s0.clone() for _ in range(n - 1)]
        qp, sp = _ptrs(ql), _ptrs(sl)
        wb = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        nb = _copies(wb.numel() * 2, L2)
        wl = [wb] + [wb.clone() for _ in range(nb - 1)]
        for M in PROMPT_TOKENS:
            x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(5, (M, K), 1.0)), dev)
            y = torch.empty((M, N), dtype=torch.float16, device=dev)
            yf = torch.empty((M, N), dtype=torch.float32, device=dev)
            xb = x.to(torch.bfloat16)
            yb = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            ours = _graph_us(torch, vkb, stream, lambda i: vkb.gemm_tc(ql[i % n], sl[i % n], x, y=y))
            cub = _graph_us(torch, vkb, stream, lambda i: torch.matmul(xb, wl[i % nb].t(), out=yb), vkb_graph=False)
            vkb.gemm_tc(q0, s0, x, y=yf, out_f32=True)
            torch.cuda.synchronize()
            fl = 2.0 * M * N * K
            rec = {"us": round(ours, 2), "tflops": round(fl / ours / 1e6, 1), "cublas_bf16_us": round(cub, 2)}
            for rname, kind in (("tc_q4", RK_TC_Q4), ("tc_q4_v2", RK_TC_Q4_V2)):
                yr = torch.zeros((M, N), dtype=torch.float32, device=dev)
                if L.ref_kernel_run(kind, M, q0.data_ptr(), s0.data_ptr(), x.data_ptr(), yr.data_ptr(), N, K):
                    continue
                us = L.ref_kernel_time_us(kind, M, qp, sp, n, x.data_ptr(), yr.data_ptr(), N, K)
                rec[rname] = {"us": round(us, 2), "tflops": round(fl / us / 1e6, 1), "speedup": round(us / ours, 2),
                              "agree": _agree(yr, yf)}
            out["prompt"][f"q4_{N}x{K}_m{M}"] = rec
        del ql, sl, wl
    torch.cuda.synchronize()
    out["how"] = ("reference kernels: src/bakeoff.cu and stage2..5.cuh compiled for sm_100a (baseline/Makefile), "
                  "called through the reference's own launchers; every contender 50 calls per CUDA graph, median of 5 "
                  "replays, weight copies >= 4x L2; speedup = reference us / ours")
    return out


if __name__ == "__main__":
    res = main(quick="--quick" in sys.argv)
    print(json.dumps(res), flush=True)
