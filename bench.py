#!/usr/bin/env python
"""bench.py -- the benchmark driver contract for the B200 quantised matmul hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the dense quantised GEMV sweep -- Q4_0, Q8_0 and 2-bit weights, tables
12288x2560, 2560x6144, 6144x2048 and 2048x6144 (N_out x K_in), 1, 2, 4 and 8 tokens: 48 calls per step, each through
the library's C ABI (vkb_gemv), weights N(0,0.02) seed 0 quantised per 32-value block, activations fp16 N(0,1).
One step = one pass over the 48 (format, table, tokens) cases. Every case reads a different copy of its table and the
copies of each table cycle through >= 4x L2 across steps, so every call reads its weights from HBM (the reference's
fairness rule, src/bakeoff.cu:16-18, :314, with 96 MB raised to 4x B200's L2).

Metric: aggregate decode-GEMV HBM throughput in GB/s = algorithmic bytes (packed codes + fp16 scales + x + y) of the
step / step time, and the reference's own µs per call for each case (time_us: 5 batches of 50 back-to-back calls,
median), including configs[0] (Q4_0 8192x2048, 1 token).

Multi-GPU: the dense GEMV does not shard (replicas only): every rank runs the whole step on its own GPU; value sums the
ranks' bytes over the slowest rank's time (weak scaling).

Extra fields of the same JSON line: "prompt_gemm" (configs[4]: the tcgen05 Q4 prompt GEMM at 64 and 512 tokens against
cuBLAS bf16 on the same GPU), "moe" (configs[2]/[3] one-launch MoE, µs per call), and with N > 1 GPUs "sharded": the
expert-parallel MoE and the row-split prompt GEMM across the ranks (max over ranks).

The reference arm (--impl reference) times the reference's own CPU path, ref_value (src/bakeoff.cu:221-227, compiled
from the reference source into oracle/_ref/ by oracle/Makefile), on all host cores over a bounded sample of each
step's outputs, scaled to the full step.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "volta-kernel-bakeoff_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

SHAPES = [(12288, 2560), (2560, 6144), (6144, 2048), (2048, 6144)]   # configs[1] tables (N_out x K_in)
FORMATS = [("q4", 0, 0.5625), ("q8", 1, 1.0625), ("q2", 2, 0.3125)]  # name, vkb format, bytes per weight
TOKENS = [1, 2, 4, 8]
HEADLINE = ("q4", 0, 8192, 2048, 1)                                   # configs[0]
METRIC = "decode GEMV HBM throughput, configs[1] sweep (Q4_0/Q8_0/2-bit x 4 tables x 1/2/4/8 tokens)"


def case_bytes(bw: float, N: int, K: int, M: int) -> float:
    """Algorithmic bytes of one call: packed codes + scales (bw per weight), x in, y out (fp16)."""
    return N * K * bw + M * K * 2 + M * N * 2


def step_bytes() -> float:
    return sum(case_bytes(bw, N, K, M) for _, _, bw in FORMATS for N, K in SHAPES for M in TOKENS)


# ---- clocks ----------------------------------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples of the SM clock, clock-event reasons, utilisation, temperature and ECC during the timed
    region, judged by vkb.load_judge (the B200 counterpart of the reference's bench/load_flag.py)."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_gpu{gpu_index}.csv")

    def start(self):
        from vkb import load_judge
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={load_judge.SAMPLE_FIELDS}",
                                          "--format=csv,noheader,nounits", "-i", str(self.gpu), "-lms", "20"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        from vkb import load_judge
        if self.proc is None:
            return None
        time.sleep(0.06)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        with open(self.path, encoding="utf-8", errors="replace") as fh:
            v = load_judge.judge(fh.read())
        return {"sm_mhz": v.median_clock, "sm_max_mhz": v.max_clock, "reasons": v.reason_names(),
                "samples": v.busy, "flagged": v.flagged, "judge": load_judge.format_line("timed", v)}


# ---- the reference's CPU path ----------------------------------------------------------------------------------------

def cpu_reference_step(cases, frac: float, threads: int):
    """Times the reference's ref_value (oracle/_ref) over the first frac of every case's output rows, all threads;
    returns (seconds for the full step, scaled; kind; sample description). Falls back to the numpy oracle port when the
    reference library is not built."""
    import numpy as np
    from oracle import refbind
    L = refbind.load()
    t_total = 0.0
    for c in cases:
        rows = max(16, int(c["N"] * frac))
        if L is not None:
            t0 = time.perf_counter()
            refbind.gemv_mt(c["codes"][:rows], c["scales"][:rows], c["x"], 0, rows, threads)
            dt = time.perf_counter() - t0
        else:
            from oracle import oracle as O
            t0 = time.perf_counter()
            O.ref_value(c["codes"][:rows], c["scales"][:rows], c["x"])
            dt = time.perf_counter() - t0
        t_total += dt * c["N"] / rows
    kind = "reference" if L is not None else "port"
    sample = f"first {frac:.3g} of the output rows of each of the {len(cases)} step cases, scaled to the full step"
    return t_total, kind, sample


def cpu_frac_for(cases, threads: int, budget_s: float) -> float:
    """The sampled row fraction that makes one CPU step take about budget_s (from a tiny calibration sample)."""
    f0 = 1.0 / 1024
    t0, _, _ = cpu_reference_step(cases, f0, threads)   # t0 is already scaled to the full step
    return max(1.0 / 4096, min(0.25, budget_s / max(t0, 1e-9)))


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            return int(parts[local_rank])
    return local_rank


def host_cases(for_cpu: bool = True):
    """Host-side weights/activations of the 48 step cases (codes int8, fp16 scales and x as uint16 bits)."""
    import vkb
    cases = []
    for fname, fmt, bw in FORMATS:
        for N, K in SHAPES:
            codes, scales = vkb.quantize(fmt, vkb.synth_normal(0, (N, K), 0.02))
            for M in TOKENS:
                x = vkb.to_f16_bits(vkb.synth_normal(1 + M, (M, K), 1.0))
                cases.append(dict(fname=fname, fmt=fmt, bw=bw, N=N, K=K, M=M, codes=codes, scales=scales, x=x))
    return cases


# ---- extra sections: prompt GEMM, MoE, sharded paths -------------------------------------------------------------

PROMPT_SHAPES = [(12288, 2560), (8192, 2048)]          # configs[4]
PROMPT_TOKENS = [64, 512]
MOE_CASES = [  # configs[2] and configs[3]: (name, experts, top-k, N, K, token counts)
    ("qwen36_gate_up_128x512x2048_top8", 128, 8, 512, 2048, [1, 8, 64]),
    ("qwen36_down_128x2048x512_top8", 128, 8, 2048, 512, [1, 8, 64]),
    ("flashnext_gate_up_160x640x2560_top10", 160, 10, 640, 2560, [1, 8]),
]


def _median_us(torch, stream, run, calls: int = 50, reps: int = 5, graph: bool = True, vkb_graph: bool = True) -> float:
    """The reference's time_us: median over reps of `calls` back-to-back calls (run(i) issues call i), captured in one
    CUDA graph when `graph` (no host launch cost in the number; vkb calls through the library's own graph helpers,
    torch calls through torch.cuda.graph), else launched directly."""
    import vkb
    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    g = None
    if graph:
        g = vkb.Graph(stream) if vkb_graph else torch.cuda.CUDAGraph()
        with (g if vkb_graph else torch.cuda.graph(g, stream=stream)):
            for i in range(calls):
                run(i)
        g.replay()
    ts = []
    for r in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        if g is not None:
            g.replay()
        else:
            for i in range(calls):
                run(r * calls + i)
        b.record(stream)
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1000.0 / calls)
    del g
    return sorted(ts)[len(ts) // 2]


def _max_over_ranks(torch, dist, dev, v: float) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _copies(nbytes: int, L2: int) -> int:
    return max(2, math.ceil(4 * L2 / max(1, nbytes)))


def prompt_section(torch, vkb, dev, stream, L2, peaks):
    """configs[4] on one GPU: the tcgen05 prompt GEMM against cuBLAS bf16 (torch.matmul, bf16 in and out) at the same
    shapes, weights cycled over >= 4x L2 for both; the same shapes with Q8 weights (the Q8 prompt kernel, SURVEY
    8(f)) as q8_* entries."""
    out = {}
    for N, K in PROMPT_SHAPES:
        sets = {}
        for fmt in (0, 1):
            codes, scales = vkb.quantize(fmt, vkb.synth_normal(0, (N, K), 0.02))
            q0 = vkb.to_device_packed(vkb.pack(fmt, codes), dev)
            s0 = vkb.to_device_f16(scales, dev)
            nq = _copies(q0.numel() * q0.element_size() + 2 * s0.numel(), L2)
            sets[fmt] = ([q0] + [q0.clone() for _ in range(nq - 1)], [s0] + [s0.clone() for _ in range(nq - 1)], nq)
        wb = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        nb = _copies(wb.numel() * 2, L2)
        wl = [wb] + [wb.clone() for _ in range(nb - 1)]
        for M in PROMPT_TOKENS:
            x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(5, (M, K), 1.0)), dev)
            xb = x.to(torch.bfloat16)
            y = torch.empty((M, N), dtype=torch.float16, device=dev)
            yb = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            us_b = _median_us(torch, stream, lambda i: torch.matmul(xb, wl[i % nb].t(), out=yb), vkb_graph=False)
            fl = 2.0 * M * N * K
            for fmt, tag in ((0, "q4"), (1, "q8")):
                ql, sl, nq = sets[fmt]
                us = _median_us(torch, stream, lambda i: vkb.gemm_tc(ql[i % nq], sl[i % nq], x, y=y, fmt=fmt))
                out[f"{tag}_{N}x{K}_m{M}"] = {
                    "us": round(us, 2), "tflops": round(fl / us / 1e6, 1), "cublas_bf16_us": round(us_b, 2),
                    "cublas_bf16_tflops": round(fl / us_b / 1e6, 1), "time_vs_cublas_bf16": round(us_b / us, 3),
                    "frac_of_bf16_peak": round(fl / us / 1e6 / float(peaks.get("bf16_tflops", 1590.0)), 3)}
        del sets, wl
    return out


def moe_section(torch, vkb, dev, stream, L2, comm=None, rank=0, world=1):
    import numpy as np
    """configs[2]/[3]: one-launch MoE over a device index list, T tokens x k distinct experts. With a communicator,
    the experts are split over the ranks (vkb_moe_ep: own slots + zeros, in-place all-reduce)."""
    from vkb import dist as D
    out = {}
    for name, E, k, N, K, Ts in MOE_CASES:
        e0, el = D.expert_range(E, world, rank) if comm is not None else (0, E)
        codes, scales = vkb.quantize(0, vkb.synth_normal(7, (el * N, K), 0.02))
        q0 = vkb.to_device_packed(vkb.pack(0, codes), dev).view(el, N, -1)
        s0 = vkb.to_device_f16(scales, dev).view(el, N, K // 32)
        per_expert = N * K * 0.5625
        n = _copies(int(el * per_expert), L2)
        ql, sl = [q0] + [q0.clone() for _ in range(n - 1)], [s0] + [s0.clone() for _ in range(n - 1)]
        for T in Ts:
            idx_np = vkb.synth_topk(11 + T, T, E, k)
            idx = torch.from_numpy(idx_np).to(dev)
            x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(13, (T, K), 1.0)), dev)
            y = torch.empty((T, k, N), dtype=torch.float16, device=dev)
            us_p2p = None
            if comm is None:
                us = _median_us(torch, stream, lambda i: vkb.moe(0, ql[i % n], sl[i % n], idx, x, y=y))
            else:
                us = _median_us(torch, stream, lambda i: comm.moe_ep(ql[i % n], sl[i % n], idx, x, E_local=el,
                                                                      e0=e0, y=y), graph=False)
                ysym = comm.alloc((T, k, N), torch.float16)
                us_p2p = _median_us(torch, stream, lambda i: comm.moe_ep_p2p(ql[i % n], sl[i % n], idx, x, E_local=el,
                                                                              e0=e0, y_sym=ysym))
                torch.cuda.synchronize()
                ysym.free()
            U = len(np.unique(idx_np))
            nbytes = U * per_expert + idx_np.nbytes + T * K * 2 + T * k * N * 2
            out[f"{name}_t{T}"] = {"us": round(us, 2), "distinct_experts": U,
                                   "GBps": round(nbytes / us / 1e3, 1) if comm is None else None}
            if us_p2p is not None:
                out[f"{name}_t{T}"]["us_p2p"] = round(us_p2p, 2)
        del ql, sl
    return out


def glu_section(torch, vkb, dev, stream, L2):
    """SURVEY 8(f) row 1, the reference's like-for-like decode entries: Q4 decode with fp32 activations (rounded to
    fp16 inside the kernel) on configs[0]'s table, and gate + up + SwiGLU (Qwen3-1.7B's MLP, gate and up 6144x2048
    stacked) with fp32 activations, one kernel; weights cycled over >= 4x L2. GB/s: packed weights + activations +
    outputs per call."""
    out = {}
    cases = [("q4_f32in_8192x2048", 8192, 2048, False), ("glu_q4_f32in_2x6144x2048", 6144, 2048, True)]
    for name, N, K, glu in cases:
        rows = 2 * N if glu else N
        codes, scales = vkb.quantize(0, vkb.synth_normal(3, (rows, K), 0.02))
        q0 = vkb.to_device_packed(vkb.pack(0, codes), dev)
        s0 = vkb.to_device_f16(scales, dev)
        wbytes = q0.numel() + 2 * s0.numel()
        n = _copies(wbytes, L2)
        ql, sl = [q0] + [q0.clone() for _ in range(n - 1)], [s0] + [s0.clone() for _ in range(n - 1)]
        for M in (1, 2, 4, 8):
            x = torch.from_numpy(vkb.synth_normal(17 + M, (M, K), 1.0).astype("float32")).to(dev)
            xh = torch.empty((M, K), dtype=torch.float16, device=dev)
            if glu:
                ys = torch.empty((M, 2 * N), dtype=torch.float32, device=dev)
                y = torch.empty((M, N), dtype=torch.float32, device=dev)
                us = _median_us(torch, stream, lambda i: vkb.gate_up_glu_q4(ql[i % n], sl[i % n], x, ystack=ys, out=y,
                                                                              xh=xh))
                nbytes = wbytes + M * K * 4 + M * 2 * N * 4 + M * N * 4
            else:
                y = torch.empty((M, N), dtype=torch.float32, device=dev)
                us = _median_us(torch, stream, lambda i: vkb.gemv_q4_f32in(ql[i % n], sl[i % n], x, xh=xh, y=y))
                nbytes = wbytes + M * K * 4 + M * N * 4
            out[f"{name}_m{M}"] = {"us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1)}
        del ql, sl
    return out


def rowsplit_section(torch, vkb, dev, stream, L2, comm, rank, world):
    """configs[4] with the weight rows split over the ranks (vkb_gemm_q4_tc_rowsplit: local tcgen05 GEMM, in-place
    all-gather, permute)."""
    from vkb import dist as D
    out = {}
    for N, K in PROMPT_SHAPES:
        n0, nl = D.row_range(N, world, rank)
        codes, scales = vkb.quantize(0, vkb.synth_normal(0, (N, K), 0.02)[n0:n0 + nl])
        q0 = vkb.to_device_packed(vkb.pack(0, codes), dev)
        s0 = vkb.to_device_f16(scales, dev)
        nq = _copies(q0.numel() + 2 * s0.numel(), L2)
        ql, sl = [q0] + [q0.clone() for _ in range(nq - 1)], [s0] + [s0.clone() for _ in range(nq - 1)]
        for M in PROMPT_TOKENS:
            x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(5, (M, K), 1.0)), dev)
            y = torch.empty((M, N), dtype=torch.float16, device=dev)
            work = torch.empty(vkb.lib().vkb_gemm_rowsplit_work_bytes(M, N, 0), dtype=torch.uint8, device=dev)
            us = _median_us(torch, stream, lambda i: comm.gemm_rowsplit(ql[i % nq], sl[i % nq], x, N, y=y, work=work),
                            graph=False)
            ysym = comm.alloc((M, N), torch.float16)
            us_p2p = _median_us(torch, stream, lambda i: comm.gemm_rowsplit_p2p(ql[i % nq], sl[i % nq], x, N, ysym))
            torch.cuda.synchronize()
            ysym.free()
            out[f"q4_{N}x{K}_m{M}"] = {"us": us, "us_p2p": us_p2p, "flop": 2.0 * M * N * K,
                                       "allgather_bytes": M * N * 2}
        del ql, sl
    return out


# ---- our arm ---------------------------------------------------------------------------------------------------------

def run_ours(args, rank: int, world: int, local_rank: int, dist):
    import numpy as np
    import torch
    import vkb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    L2 = torch.cuda.get_device_properties(dev).L2_cache_size
    L = vkb.lib()

    # weights: one quantised table per (format, shape), C copies each (>= 4 x L2 of that table)
    cases = host_cases()
    tables = {}
    for c in cases:
        key = (c["fmt"], c["N"], c["K"])
        if key not in tables:
            q0 = vkb.to_device_packed(vkb.pack(c["fmt"], c["codes"]), dev)
            s0 = vkb.to_device_f16(c["scales"], dev)
            tb = q0.numel() + 2 * s0.numel()
            ncopy = max(4, math.ceil(4 * L2 / tb))
            tables[key] = dict(q=[q0] + [q0.clone() for _ in range(ncopy - 1)],
                               s=[s0] + [s0.clone() for _ in range(ncopy - 1)], n=ncopy)
    # every distinct activation block in one device buffer and every output in another (views into them), so that an
    # end-to-end step moves each direction with one copy
    x_keys, x_host_parts = [], []
    for c in cases:
        key = (c["K"], c["M"])
        if key not in x_keys:
            x_keys.append(key)
            x_host_parts.append(np.ascontiguousarray(c["x"]).reshape(-1))
    x_all = vkb.to_device_f16(np.concatenate(x_host_parts), dev)
    xs, off = {}, 0
    for key, part in zip(x_keys, x_host_parts):
        xs[key] = x_all[off:off + part.size].view(key[1], key[0])
        off += part.size
    y_all = torch.empty(sum(c["M"] * c["N"] for c in cases), dtype=torch.float16, device=dev)
    ys, off = [], 0
    for c in cases:
        ys.append(y_all[off:off + c["M"] * c["N"]].view(c["M"], c["N"]))
        off += c["M"] * c["N"]
    max_copies = max(t["n"] for t in tables.values())
    ngraph = max(1, math.ceil(max_copies / len(TOKENS)))

    def launch_step(j: int):
        for ci, c in enumerate(cases):
            tb = tables[(c["fmt"], c["N"], c["K"])]
            m = TOKENS.index(c["M"])
            k = (j * len(TOKENS) + m) % tb["n"]
            vkb.gemv(c["fmt"], tb["q"][k], tb["s"][k], xs[(c["K"], c["M"])], y=ys[ci])

    # correctness guard on this box before timing: the headline table against the oracle
    for i in range(2):
        launch_step(i)
    torch.cuda.synchronize()
    if vkb.device_status() != 0:
        raise RuntimeError("device-side timeout during warm-up")

    graphs = []
    for j in range(ngraph):   # the library's graph helpers (vkb_graph_*): one launch per step, nothing else replayed
        g = vkb.Graph(stream)
        with g:
            launch_step(j)
        graphs.append(g)

    for w in range(args.warmup):
        graphs[w % ngraph].replay()
    torch.cuda.synchronize()

    clk = ClockSampler(gpu_index(local_rank))
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.steps):
        graphs[(args.warmup + k) % ngraph].replay()
    e1.record(stream)
    e1.synchronize()
    clocks = clk.stop()
    if dist is not None:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    sbytes = step_bytes()
    value = sbytes * args.steps * world / (ms_max * 1e-3) / 1e9
    per_gpu = sbytes * args.steps / (ms_max * 1e-3) / 1e9

    # per-case µs/call, the reference's time_us: 5 batches of 50 back-to-back calls, median (graph of 50 calls)
    table = {}
    def time_case(fmt, q_list, s_list, x, y, n):
        g = vkb.Graph(stream)
        with g:
            for i in range(50):
                vkb.gemv(fmt, q_list[i % n], s_list[i % n], x, y=y)
        for _ in range(2):
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
    if rank == 0:
        for c in cases:
            tb = tables[(c["fmt"], c["N"], c["K"])]
            yc = torch.empty((c["M"], c["N"]), dtype=torch.float16, device=dev)
            us = time_case(c["fmt"], tb["q"], tb["s"], xs[(c["K"], c["M"])], yc, tb["n"])
            table[f'{c["fname"]}_{c["N"]}x{c["K"]}_m{c["M"]}'] = {
                "us": round(us, 3), "GBps": round(case_bytes(c["bw"], c["N"], c["K"], c["M"]) / us / 1e3, 1)}
        # Q4_0 8192x2048, 1 token
        fname, fmt, N, K, M = HEADLINE
        codes, scales = vkb.quantize(fmt, vkb.synth_normal(0, (N, K), 0.02))
        q0 = vkb.to_device_packed(vkb.pack(fmt, codes), dev)
        s0 = vkb.to_device_f16(scales, dev)
        n = max(4, math.ceil(4 * L2 / (q0.numel() + 2 * s0.numel())))
        ql, sl = [q0] + [q0.clone() for _ in range(n - 1)], [s0] + [s0.clone() for _ in range(n - 1)]
        xh = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(2, (M, K), 1.0)), dev)
        yh = torch.empty((M, N), dtype=torch.float16, device=dev)
        us = time_case(fmt, ql, sl, xh, yh, n)
        headline = {"case": "configs[0] Q4_0 8192x2048, 1 token", "us_per_call": round(us, 3),
                    "GBps": round(case_bytes(0.5625, N, K, M) / us / 1e3, 1), "copies": n}
        del ql, sl

    # end to end through the public API: per step the host->device copy of every activation block from pinned memory
    # (one copy: they are contiguous), the step's 48 calls as one vkb_graph_launch (the graphs above), and the
    # device->host read of every output (one copy), then a stream sync; host wall clock
    x_all_host = torch.from_numpy(np.concatenate(x_host_parts).view(np.int16)).view(torch.float16).pin_memory()
    y_all_host = torch.empty(y_all.shape, dtype=torch.float16).pin_memory()
    h2d = x_all_host.numel() * 2
    d2h = y_all_host.numel() * 2

    def e2e_step(j):
        with torch.cuda.stream(stream):
            x_all.copy_(x_all_host, non_blocking=True)
            graphs[j % ngraph].replay()
            y_all_host.copy_(y_all, non_blocking=True)
        stream.synchronize()

    e2e_steps = max(3, min(args.steps, 200))
    for j in range(3):
        e2e_step(j)
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for j in range(e2e_steps):
        e2e_step(j)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = sbytes * e2e_steps * world / float(te.item()) / 1e9

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass

    # prompt GEMM and MoE on this GPU (every rank runs them: replicas), then the sharded paths when world > 1
    prompt = prompt_section(torch, vkb, dev, stream, L2, peaks)
    moe1 = moe_section(torch, vkb, dev, stream, L2)
    glu1 = glu_section(torch, vkb, dev, stream, L2)
    sharded = None
    if dist is not None:
        from vkb import dist as D
        comm = D.Comm.from_torch()
        moe_ep = moe_section(torch, vkb, dev, stream, L2, comm, rank, world)
        rows = rowsplit_section(torch, vkb, dev, stream, L2, comm, rank, world)
        for d in (moe_ep, rows):
            for v in d.values():
                for key in ("us", "us_p2p"):
                    if key in v:
                        v[key] = round(_max_over_ranks(torch, dist, dev, v[key]), 2)
                if "flop" in v:   # throughput of the max-over-ranks time
                    fl = v.pop("flop")
                    v["tflops"] = round(fl / v["us"] / 1e6, 1)
                    v["tflops_p2p"] = round(fl / v["us_p2p"] / 1e6, 1)
        torch.cuda.synchronize()
        comm.close()
        sharded = {"gpus": world, "moe_expert_parallel": moe_ep, "prompt_row_split": rows,
                   "timing": "median of 5 x 50 calls, device events, max over ranks; us: NCCL combine, launched directly; "
                             "us_p2p: combine fused into the kernel (peer stores), the 50 calls in one CUDA graph"}

    if rank != 0:
        return None
    peak = float(peaks.get("hbm_gbs", 6650.0))
    traffic = None
    tf = os.path.join(ROOT, "profiles", "qmv_dram_traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get("step_bytes_per_launch")
        except (OSError, ValueError):
            traffic = None

    cpu = None
    if world == 1:
        threads = os.cpu_count() or 1
        frac = cpu_frac_for(cases, threads, budget_s=10.0)
        t_cpu, kind, sample = cpu_reference_step(cases, frac, threads)
        cpu = {"value": round(sbytes / t_cpu / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": sample, "s_per_step": round(t_cpu, 3)}

    return {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 x int{4,8,2} codes -> f32",
        "data": "synthetic: weights N(0,0.02) seed 0 quantised per 32 (Q4_0/Q8_0/2-bit), x fp16 N(0,1)",
        "config": {
            "workload": "configs[1]: dense quantised GEMV sweep, 48 calls per step",
            "tables": [f"{n}x{k}" for n, k in SHAPES], "tokens": TOKENS, "formats": [f[0] for f in FORMATS],
            "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
            "l2": "inputs larger than L2: every call reads a different copy; each table's copies cycle >= 4x L2",
            "launch": "one CUDA graph per step (48 vkb_gemv calls captured with vkb_graph_begin/end, programmatic "
                      "dependent launch between them)",
            "step_bytes": sbytes,
        },
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu / peak, 4), "traffic": traffic,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else "fallback 6650"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "how": "per step: one H2D copy of every activation block from pinned memory, the "
                "48 vkb_gemv calls as one vkb_graph_launch (C ABI), one D2H copy of every output, stream sync; host "
                "wall clock"},
        "gpu_launches": 48 * args.steps,
        "clocks": clocks,
        "cases_us": table,
        "headline": headline,
        "prompt_gemm": prompt,
        "moe": moe1,
        "f32in_and_glu": glu1,
        "sharded": sharded,
    }


# ---- the reference arm -----------------------------------------------------------------------------------------------

def run_reference(args, rank: int, world: int):
    if rank != 0:
        return None
    cases = host_cases()
    threads = os.cpu_count() or 1
    # every step is a bounded sample of the step's outputs: the whole run takes about 90 s of CPU time
    frac = cpu_frac_for(cases, threads, budget_s=90.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_reference_step(cases, frac, threads)
    t = 0.0
    kind = sample = None
    for _ in range(args.steps):
        dt, kind, sample = cpu_reference_step(cases, frac, threads)
        t += dt
    sbytes = step_bytes()
    value = sbytes * args.steps / t / 1e9
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f64 (the reference's ref_value: double sums of fp16 x * int code * fp16 scale)",
        "data": "synthetic: weights N(0,0.02) seed 0 quantised per 32 (Q4_0/Q8_0/2-bit), x fp16 N(0,1)",
        "config": {"workload": "configs[1]: dense quantised GEMV sweep, 48 calls per step",
                   "tables": [f"{n}x{k}" for n, k in SHAPES], "tokens": TOKENS, "formats": [f[0] for f in FORMATS],
                   "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if args.impl == "reference":
        res = run_reference(args, rank, world)
    else:
        if world > 1:
            import torch
            import torch.distributed as tdist
            torch.cuda.set_device(local_rank)
            tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                     device_id=torch.device("cuda", local_rank))
            dist = tdist
        res = run_ours(args, rank, world, local_rank, dist)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
