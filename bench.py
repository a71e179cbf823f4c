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
median), including configs[0] (Q4_0 8192x2048, 1 token), with cuBLAS bf16 on the same GPU beside every case.

Multi-GPU: the dense GEMV does not shard (replicas only): every rank runs the whole step on its own GPU; value sums the
ranks' bytes over the slowest rank's time (weak scaling). The paths that do shard -- the expert-parallel MoE
(configs[2]/[3]) and the row-split prompt GEMM -- are timed beside their one-GPU time in "sharded", each
case with its parity against the one-GPU kernel (bit for bit, NCCL and fused combines); a mismatch makes the run exit
non-zero after the JSON line.

Extra fields of the same JSON line: "prompt_gemm" (configs[4] against cuBLAS bf16), "moe" (configs[2]/[3]),
"f32in_and_glu" (the reference's fp32-in and gate/up entries) and, on one GPU, "reference_kernels": the reference's
own kernels rebuilt for sm_100a (baseline/) timed on the same GPU and weights as ours (baseline/time_ref_kernels.py, in a
child process).

The reference arm (--impl reference) times the reference's own CPU path, ref_value (src/bakeoff.cu:221-227, compiled
from the reference source into oracle/_ref/ by oracle/Makefile), on all host cores over the step's outputs -- all of
them when the run's budget allows, else the same leading rows of every case, reported unscaled. Its inputs are built
without libvkb.so (oracle/_ref's input generator and the numpy quantiser). Our arm's cpu_baseline is the same
procedure.
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
    """Clock samples during the timed region -- SM clock, max clock, power, clock-event reasons, utilization,
    temperature, uncorrected ECC, in nvidia-smi's CSV columns -- judged by vkb.load_judge (the B200 counterpart of the
    reference's bench/load_flag.py). NVML is polled from a thread as fast as it answers while the timed work runs (the
    timed region of a default run is a few milliseconds, shorter than nvidia-smi's sampling period); without NVML it
    falls back to nvidia-smi every 20 ms."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.rows = []
        self.path = None

    def _poll(self, handle, nv):
        # the fast queries (SM clock, clock-event reasons) in the loop; power, utilization, temperature and uncorrected
        # ECC -- slower queries -- once at the start and once at the end of the timed window
        def field(fn, fmt):
            try:
                return fmt(fn())
            except Exception:
                return "[N/A]"

        def slow():
            return (field(lambda: nv.nvmlDeviceGetPowerUsage(handle) / 1000.0, lambda w: f"{w:.1f}"),
                    field(lambda: nv.nvmlDeviceGetUtilizationRates(handle).gpu, str),
                    field(lambda: nv.nvmlDeviceGetTemperature(handle, nv.NVML_TEMPERATURE_GPU), str),
                    field(lambda: nv.nvmlDeviceGetTotalEccErrors(handle, nv.NVML_MEMORY_ERROR_TYPE_UNCORRECTED,
                                                                 nv.NVML_VOLATILE_ECC), str))
        mx = field(lambda: nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM), str)
        sl = slow()
        fast = []
        while not self.stop_flag:
            fast.append((field(lambda: nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM), str),
                         field(lambda: nv.nvmlDeviceGetCurrentClocksEventReasons(handle), lambda b: f"0x{b:016x}")))
            self.polling.set()
        sl_end = slow()
        for i, (clk, why) in enumerate(fast):
            pw, util, temp, ecc = sl if i < len(fast) // 2 else sl_end
            self.rows.append(",".join([str(self.gpu), clk, mx, pw, why, "-", "-", "-", "-", util, temp, ecc]))

    def start(self):
        import threading
        self.stop_flag = False
        self.polling = threading.Event()
        try:
            import pynvml as nv
            nv.nvmlInit()
            handle = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.switch = sys.getswitchinterval()
            sys.setswitchinterval(1e-4)   # let the sampling thread run while the main thread waits on the GPU
            self.thread = threading.Thread(target=self._poll, args=(handle, nv), daemon=True)
            self.thread.start()
            self.polling.wait(timeout=2.0)   # the timed region starts once the sampling loop runs
            return
        except Exception:
            self.thread = None
        import tempfile
        from vkb import load_judge
        try:
            fd, self.path = tempfile.mkstemp(prefix=f"vkb_clocks_gpu{self.gpu}_", suffix=".csv")
            self.f = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={load_judge.SAMPLE_FIELDS}",
                                          "--format=csv,noheader,nounits", "-i", str(self.gpu), "-lms", "20"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        from vkb import load_judge
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
            sys.setswitchinterval(self.switch)
            text, how = "\n".join(self.rows) + "\n", f"NVML polled inside the timed region, {len(self.rows)} samples"
            v = load_judge.judge(text, assume_busy=True)
        elif self.proc is not None:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()
            with open(self.path, encoding="utf-8", errors="replace") as fh:
                v = load_judge.judge(fh.read())
            os.unlink(self.path)
            how = "nvidia-smi every 20 ms"
        else:
            return None
        return {"sm_mhz": v.median_clock, "sm_max_mhz": v.max_clock, "reasons": v.reason_names(),
                "samples": v.busy, "flagged": v.flagged, "how": how, "judge": load_judge.format_line("timed", v)}


# ---- the reference's CPU path ----------------------------------------------------------------------------------------

def cpu_reference(cases, threads: int, frac: float):
    """One step of the reference's CPU path: its ref_value (oracle/_ref, src/bakeoff.cu:221-227) over the leading
    `frac` of every case's output rows (all of them at frac = 1), on `threads` host threads. Returns (seconds,
    algorithmic bytes of the outputs computed). Falls back to the numpy oracle port when the reference library is not
    built."""
    from oracle import refbind
    L = refbind.load()
    t_total, nbytes = 0.0, 0.0
    for c in cases:
        rows = c["N"] if frac >= 1.0 else max(16, int(c["N"] * frac))
        t0 = time.perf_counter()
        if L is not None:
            refbind.gemv_mt(c["codes"][:rows], c["scales"][:rows], c["x"], 0, rows, threads)
        else:
            from oracle import oracle as O
            O.ref_value(c["codes"][:rows], c["scales"][:rows], c["x"])
        t_total += time.perf_counter() - t0
        nbytes += case_bytes(c["bw"], rows, c["K"], c["M"])
    return t_total, nbytes


def cpu_plan(cases, threads: int, steps: int, budget_s: float) -> float:
    """The output-row fraction per step that keeps `steps` CPU steps within about budget_s (1.0 when the full step
    fits), from a timed 1/64 sample."""
    t, _ = cpu_reference(cases, threads, 1.0 / 64)
    full = t * 64
    return 1.0 if full * steps <= budget_s else max(1.0 / 4096, budget_s / steps / full)


def cpu_kind() -> str:
    from oracle import refbind
    return "reference" if refbind.load() is not None else "port"


def cpu_sample_text(frac: float, ncases: int) -> str:
    if frac >= 1.0:
        return f"every output of the {ncases} step cases (the full step, nothing scaled)"
    return (f"the first {frac:.3g} of the output rows of each of the {ncases} step cases per step; value = those "
            f"outputs' algorithmic bytes / their time, unscaled")


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            return int(parts[local_rank])
    return local_rank


def host_cases(source: str = "vkb"):
    """Host-side weights/activations of the 48 step cases (codes int8, fp16 scales and x as uint16 bits). source
    "vkb": the library's host functions (our arm); "oracle": oracle/_ref's input generator and the numpy quantiser (the
    reference arm, which loads no libvkb.so) -- the same bits (tests/test_oracle.py)."""
    import numpy as np
    if source == "vkb":
        import vkb
        normal, quantize, f16 = vkb.synth_normal, vkb.quantize, vkb.to_f16_bits
    else:
        from oracle import oracle as O
        from oracle import refbind
        normal, quantize = refbind.synth_normal, O.quantize
        f16 = lambda a: np.ascontiguousarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)  # noqa: E731
    cases = []
    for fname, fmt, bw in FORMATS:
        for N, K in SHAPES:
            codes, scales = quantize(fmt, normal(0, (N, K), 0.02))
            for M in TOKENS:
                x = f16(normal(1 + M, (M, K), 1.0))
                cases.append(dict(fname=fname, fmt=fmt, bw=bw, N=N, K=K, M=M, codes=codes, scales=scales, x=x))
    return cases


def bench_config():
    """The workload's config, identical in both arms."""
    return {"workload": "configs[1]: dense quantised GEMV sweep, 48 calls per step",
            "tables": [f"{n}x{k}" for n, k in SHAPES], "tokens": TOKENS, "formats": [f[0] for f in FORMATS],
            "step_bytes": step_bytes(),
            "l2": "inputs larger than L2: every call reads a different copy; each table's copies cycle >= 4x L2"}


# ---- extra sections: prompt GEMM, MoE, sharded paths -------------------------------------------------------------

PROMPT_SHAPES = [(12288, 2560), (8192, 2048)]          # configs[4]
PROMPT_TABLES = PROMPT_SHAPES + [(2560, 6144), (2048, 6144)]   # + configs[1]'s tables with few row tiles
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
    shapes, weights cycled over >= 4x L2 for both; the same shapes with Q8 weights (the Q8 prompt kernel the reference
    planned but never built) as q8_* entries; also the small-N / large-K tables, which the planner runs as split-K
    clusters. dq4_cublas_fp16_us: the reference's dq4+cublas control (GPU dequantisation, then an fp16 cuBLAS GEMM)."""
    out = {}
    for N, K in PROMPT_TABLES:
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
            # the reference's dq4+cublas control: the packed Q4 weights dequantised on the GPU (vkb_dequant), then
            # an fp16 GEMM (torch.matmul, cuBLAS)
            ql4, sl4, nq4 = sets[0]
            wtmp = torch.empty((N, K), dtype=torch.float16, device=dev)
            us_dq = _median_us(torch, stream, lambda i: (vkb.dequant(0, ql4[i % nq4], sl4[i % nq4], N, K, w=wtmp),
                                                         torch.matmul(x, wtmp.t(), out=y)), vkb_graph=False)
            del wtmp
            for fmt, tag in ((0, "q4"), (1, "q8")):
                ql, sl, nq = sets[fmt]
                us = _median_us(torch, stream, lambda i: vkb.gemm_tc(ql[i % nq], sl[i % nq], x, y=y, fmt=fmt))
                out[f"{tag}_{N}x{K}_m{M}"] = {
                    "us": round(us, 2), "tflops": round(fl / us / 1e6, 1), "cublas_bf16_us": round(us_b, 2),
                    "cublas_bf16_tflops": round(fl / us_b / 1e6, 1), "time_vs_cublas_bf16": round(us_b / us, 3),
                    "frac_of_bf16_peak": round(fl / us / 1e6 / float(peaks.get("bf16_tflops", 1590.0)), 3)}
                if fmt == 0:
                    out[f"{tag}_{N}x{K}_m{M}"]["dq4_cublas_fp16_us"] = round(us_dq, 2)
        del sets, wl
    return out


def moe_section(torch, vkb, dev, stream, L2):
    """configs[2]/[3] on one GPU: one-launch MoE over a device index list, T tokens x k distinct experts."""
    import numpy as np
    out = {}
    for name, E, k, N, K, Ts in MOE_CASES:
        codes, scales = vkb.quantize(0, vkb.synth_normal(7, (E * N, K), 0.02))
        q0 = vkb.to_device_packed(vkb.pack(0, codes), dev).view(E, N, -1)
        s0 = vkb.to_device_f16(scales, dev).view(E, N, K // 32)
        per_expert = N * K * 0.5625
        n = _copies(int(E * per_expert), L2)
        ql, sl = [q0] + [q0.clone() for _ in range(n - 1)], [s0] + [s0.clone() for _ in range(n - 1)]
        for T in Ts:
            idx_np = vkb.synth_topk(11 + T, T, E, k)
            idx = torch.from_numpy(idx_np).to(dev)
            x = vkb.to_device_f16(vkb.to_f16_bits(vkb.synth_normal(13, (T, K), 1.0)), dev)
            y = torch.empty((T, k, N), dtype=torch.float16, device=dev)
            us = _median_us(torch, stream, lambda i: vkb.moe(0, ql[i % n], sl[i % n], idx, x, y=y))
            U = len(np.unique(idx_np))
            nbytes = U * per_expert + idx_np.nbytes + T * K * 2 + T * k * N * 2
            out[f"{name}_t{T}"] = {"us": round(us, 2), "distinct_experts": U, "GBps": round(nbytes / us / 1e3, 1)}
        del ql, sl
    return out


def glu_section(torch, vkb, dev, stream, L2):
    """The reference's like-for-like decode entries (fused_q4_v3_fp32in, gate_up_glu_fp32in): Q4 decode with fp32 activations (rounded to
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


def _fp64_err(torch, codes, scales, x_bits, y, rows, dev) -> float:
    """The reference's error metric, max |y - ref| / sum |x w| (src/bakeoff.cu:565-583), on the output rows `rows` of
    every token, with ref computed in float64 by torch on the device from the host codes and scales (a sampled
    slice: the -m gpu tests hold the full oracle comparisons)."""
    import numpy as np
    c = torch.from_numpy(np.ascontiguousarray(codes[rows])).to(dev).double()
    sc = torch.from_numpy(np.ascontiguousarray(scales[rows]).view(np.float16).astype(np.float64)).to(dev)
    w = c * sc.repeat_interleave(32, dim=1)
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.float16).astype(np.float64)).to(dev)
    ref = x @ w.t()
    mag = x.abs() @ w.abs().t()
    got = y[:, rows].double()
    return float(((got - ref).abs() / (mag + 1e-12)).max())


def sharded_section(torch, vkb, dev, stream, L2, comm, rank, world):
    """The paths that shard, each case on `world` GPUs beside the same problem on one GPU (every rank times the whole
    problem on its own GPU; all times max over ranks):
      MoE expert parallel (configs[2]/[3]): vkb_moe_ep (own slots + zeros, NCCL all-reduce) and vkb_moe_ep_p2p (the
        combine fused into the kernel, peer stores);
      prompt row split: vkb_gemm_q4_tc_rowsplit (NCCL all-gather + permute) and _p2p (the all-gather fused
        into the tcgen05 epilogue).
    parity: both results equal the one-GPU kernel's bit for bit on every rank (the combines only add zeros or move
    values); err_fp64: the reference's error metric on a sampled slice against a float64 product."""
    import numpy as np
    from vkb import dist as D
    moe, rows = {}, {}
    for name, E, k, N, K, Ts in MOE_CASES:
        codes, scales = vkb.quantize(0, vkb.synth_normal(7, (E * N, K), 0.02))
        qf = vkb.to_device_packed(vkb.pack(0, codes), dev).view(E, N, -1)
        sf = vkb.to_device_f16(scales, dev).view(E, N, K // 32)
        e0, el = D.expert_range(E, world, rank)
        q0, s0 = qf[e0:e0 + el].contiguous(), sf[e0:e0 + el].contiguous()
        n = _copies(int(el * N * K * 0.5625), L2)
        ql, sl = [q0] + [q0.clone() for _ in range(n - 1)], [s0] + [s0.clone() for _ in range(n - 1)]
        nf = _copies(int(E * N * K * 0.5625), L2)
        qfl, sfl = [qf] + [qf.clone() for _ in range(nf - 1)], [sf] + [sf.clone() for _ in range(nf - 1)]
        for T in Ts:
            idx_np = vkb.synth_topk(11 + T, T, E, k)
            idx = torch.from_numpy(idx_np).to(dev)
            x_bits = vkb.to_f16_bits(vkb.synth_normal(13, (T, K), 1.0))
            x = vkb.to_device_f16(x_bits, dev)
            y = torch.empty((T, k, N), dtype=torch.float16, device=dev)
            y1 = torch.empty((T, k, N), dtype=torch.float16, device=dev)
            ysym = comm.alloc((T, k, N), torch.float16)
            # parity first, on weight copy 0
            y_one = vkb.moe(0, qf, sf, idx, x)
            y_nccl = comm.moe_ep(q0, s0, idx, x, E_local=el, e0=e0)
            comm.moe_ep_p2p(q0, s0, idx, x, E_local=el, e0=e0, y_sym=ysym)
            torch.cuda.synchronize()
            same = bool(torch.equal(y_one, y_nccl)) and bool(torch.equal(y_one, ysym.tensor()))
            # fp64 slice: slots of token 0, output rows 0..63 of each slot's expert
            err = 0.0
            for j in range(k):
                e = int(idx_np[0, j])
                err = max(err, _fp64_err(torch, codes[e * N:(e + 1) * N], scales[e * N:(e + 1) * N], x_bits[:1],
                                         y_nccl[0, j:j + 1], np.arange(min(64, N)), dev))
            us1 = _median_us(torch, stream, lambda i: vkb.moe(0, qfl[i % nf], sfl[i % nf], idx, x, y=y1))
            us = _median_us(torch, stream, lambda i: comm.moe_ep(ql[i % n], sl[i % n], idx, x, E_local=el, e0=e0,
                                                                  y=y), graph=False)
            us_p2p = _median_us(torch, stream, lambda i: comm.moe_ep_p2p(ql[i % n], sl[i % n], idx, x, E_local=el,
                                                                          e0=e0, y_sym=ysym))
            torch.cuda.synchronize()
            ysym.free()
            moe[f"{name}_t{T}"] = {"us_1gpu": us1, "us": us, "us_p2p": us_p2p, "parity": same, "err_fp64": err}
        del ql, sl, qfl, sfl
    for N, K in PROMPT_SHAPES:
        codes, scales = vkb.quantize(0, vkb.synth_normal(0, (N, K), 0.02))
        qf = vkb.to_device_packed(vkb.pack(0, codes), dev)
        sf = vkb.to_device_f16(scales, dev)
        n0, nl = D.row_range(N, world, rank)
        q0, s0 = qf[n0:n0 + nl].contiguous(), sf[n0:n0 + nl].contiguous()
        nq = _copies(q0.numel() + 2 * s0.numel(), L2)
        ql, sl = [q0] + [q0.clone() for _ in range(nq - 1)], [s0] + [s0.clone() for _ in range(nq - 1)]
        nf = _copies(qf.numel() + 2 * sf.numel(), L2)
        qfl, sfl = [qf] + [qf.clone() for _ in range(nf - 1)], [sf] + [sf.clone() for _ in range(nf - 1)]
        for M in PROMPT_TOKENS:
            x_bits = vkb.to_f16_bits(vkb.synth_normal(5, (M, K), 1.0))
            x = vkb.to_device_f16(x_bits, dev)
            y = torch.empty((M, N), dtype=torch.float16, device=dev)
            y1 = torch.empty((M, N), dtype=torch.float16, device=dev)
            work = torch.empty(vkb.lib().vkb_gemm_rowsplit_work_bytes(M, N, 0), dtype=torch.uint8, device=dev)
            ysym = comm.alloc((M, N), torch.float16)
            y_one = vkb.gemm_tc(qf, sf, x)
            y_nccl = comm.gemm_rowsplit(q0, s0, x, N, work=work)
            comm.gemm_rowsplit_p2p(q0, s0, x, N, ysym)
            torch.cuda.synchronize()
            same = bool(torch.equal(y_one, y_nccl)) and bool(torch.equal(y_one, ysym.tensor()))
            sample = np.unique(np.linspace(0, N - 1, 97).astype(np.int64))   # rows of every rank's block
            err = _fp64_err(torch, codes, scales, x_bits[:8], y_nccl[:8], sample, dev)
            us1 = _median_us(torch, stream, lambda i: vkb.gemm_tc(qfl[i % nf], sfl[i % nf], x, y=y1))
            us = _median_us(torch, stream, lambda i: comm.gemm_rowsplit(ql[i % nq], sl[i % nq], x, N, y=y, work=work),
                            graph=False)
            us_p2p = _median_us(torch, stream, lambda i: comm.gemm_rowsplit_p2p(ql[i % nq], sl[i % nq], x, N, ysym))
            torch.cuda.synchronize()
            ysym.free()
            rows[f"q4_{N}x{K}_m{M}"] = {"us_1gpu": us1, "us": us, "us_p2p": us_p2p, "parity": same, "err_fp64": err,
                                        "flop": 2.0 * M * N * K, "allgather_bytes": M * N * 2}
        del ql, sl, qfl, sfl
    return moe, rows


def reference_kernels_section(timeout_s: float = 600.0):
    """The reference's own kernels rebuilt for sm_100a, timed on this GPU beside ours and cuBLAS bf16
    (baseline/time_ref_kernels.py) in a child process: the reference's error handling exits its process."""
    script = os.path.join(ROOT, "baseline", "time_ref_kernels.py")
    try:
        r = subprocess.run([sys.executable, script], capture_output=True, text=True, timeout=timeout_s,
                           env=dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0")
                                    .split(",")[0]))
    except subprocess.TimeoutExpired:
        return {"unavailable": f"timed out after {timeout_s:.0f} s"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout).strip()[-300:]}"}
    return json.loads(lines[-1])


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

    def launch_step(j: int, c0: int = 0, c1: int = len(cases)):
        for ci in range(c0, c1):
            c = cases[ci]
            tb = tables[(c["fmt"], c["N"], c["K"])]
            m = TOKENS.index(c["M"])
            k = (j * len(TOKENS) + m) % tb["n"]
            vkb.gemv(c["fmt"], tb["q"][k], tb["s"][k], xs[(c["K"], c["M"])], y=ys[ci])

    # guard before timing: two eager steps, then the library's device-side status (a wait that gave up raises it);
    # parity itself is the -m gpu tests' job
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
    # (one copy: they are contiguous), the step's 48 calls as E2E chunks of consecutive calls, each one
    # vkb_graph_launch, and the device->host read of every output, then a sync; host wall clock. A chunk's outputs are
    # consecutive in y_all: they are read back on a copy stream as soon as the chunk is done, while the next chunk
    # runs, so only the last chunk's read-back is exposed (a serving loop would overlap it the same way)
    x_all_host = torch.from_numpy(np.concatenate(x_host_parts).view(np.int16)).view(torch.float16).pin_memory()
    y_all_host = torch.empty(y_all.shape, dtype=torch.float16).pin_memory()
    h2d = x_all_host.numel() * 2
    d2h = y_all_host.numel() * 2
    nch = max(1, min(args.e2e_chunks, len(cases)))
    bounds = [round(i * len(cases) / nch) for i in range(nch + 1)]
    yoff = [0]
    for c in cases:
        yoff.append(yoff[-1] + c["M"] * c["N"])
    e2e_graphs = []
    for j in range(ngraph):
        row = []
        for c in range(nch):
            g = vkb.Graph(stream)
            with g:
                launch_step(j, bounds[c], bounds[c + 1])
            row.append(g)
        e2e_graphs.append(row)
    copy_stream = torch.cuda.Stream(device=dev)
    done = [torch.cuda.Event() for _ in range(nch)]

    def e2e_step(j):
        with torch.cuda.stream(stream):
            x_all.copy_(x_all_host, non_blocking=True)
            for c in range(nch):
                e2e_graphs[j % ngraph][c].replay()
                done[c].record(stream)
        with torch.cuda.stream(copy_stream):
            for c in range(nch):
                a, b = yoff[bounds[c]], yoff[bounds[c + 1]]
                copy_stream.wait_event(done[c])
                y_all_host[a:b].copy_(y_all[a:b], non_blocking=True)
        copy_stream.synchronize()

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
    sharded, parity_ok = None, True
    if dist is not None:
        from vkb import dist as D
        comm = D.Comm.from_torch()
        moe_ep, rows = sharded_section(torch, vkb, dev, stream, L2, comm, rank, world)
        for d in (moe_ep, rows):
            for v in d.values():
                for key in ("us_1gpu", "us", "us_p2p", "err_fp64"):
                    v[key] = round(_max_over_ranks(torch, dist, dev, v[key]), 3 if key != "err_fp64" else 9)
                v["parity"] = _max_over_ranks(torch, dist, dev, 0.0 if v["parity"] else 1.0) == 0.0   # every rank
                parity_ok &= v["parity"]
                v["speedup_vs_1gpu"] = round(v["us_1gpu"] / v["us"], 3)
                v["speedup_p2p_vs_1gpu"] = round(v["us_1gpu"] / v["us_p2p"], 3)
                if "flop" in v:   # throughput of the max-over-ranks time
                    fl = v.pop("flop")
                    v["tflops"] = round(fl / v["us"] / 1e6, 1)
                    v["tflops_p2p"] = round(fl / v["us_p2p"] / 1e6, 1)
        torch.cuda.synchronize()
        comm.close()
        sharded = {"gpus": world, "parity": parity_ok, "moe_expert_parallel": moe_ep, "prompt_row_split": rows,
                   "timing": "median of 5 x 50 calls, device events, max over ranks; us_1gpu: the whole problem on one "
                             "GPU (full weights); us: NCCL combine, launched directly; us_p2p: combine fused into the "
                             "kernel (peer stores), the 50 calls in one CUDA graph",
                   "parity_how": "bit-identical to the one-GPU kernel on the same inputs, NCCL and fused combines, "
                                 "every rank; err_fp64: max |y - ref| / sum |x w| on a sampled slice, ref in float64"}

    if rank != 0:
        return None, parity_ok
    peak = float(peaks.get("hbm_gbs", 6650.0))
    traffic = None
    tf = os.path.join(ROOT, "profiles", "qmv_dram_traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get("step_bytes_per_launch")
        except (OSError, ValueError):
            traffic = None

    cpu, refk = None, None
    if world == 1:
        # the reference's kernels on this GPU (a child process), cuBLAS bf16 beside every decode case
        refk = reference_kernels_section()
        for key, rec in (refk.get("decode") or {}).items():
            if key in table:
                table[key]["cublas_bf16_us"] = rec.get("cublas_bf16_us")
        threads = os.cpu_count() or 1
        frac = cpu_plan(cases, threads, 1, budget_s=20.0)
        t_cpu, nb = cpu_reference(cases, threads, frac)
        cpu = {"value": round(nb / t_cpu / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": cpu_kind(),
               "sample": cpu_sample_text(frac, len(cases)), "s_per_step": round(t_cpu, 3)}

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
        "config": bench_config(),
        "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
        "launch": "one CUDA graph per step (48 vkb_gemv calls captured with vkb_graph_begin/end, programmatic "
                  "dependent launch between them)",
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu / peak, 4), "traffic": traffic,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else "fallback 6650"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "chunks": nch,
                "how": f"per step: one H2D copy of every activation block from pinned memory, the 48 vkb_gemv calls "
                f"as {nch} vkb_graph_launch (C ABI) of consecutive calls, each chunk's outputs copied D2H on a copy "
                "stream as soon as it is done (while the next chunk runs), sync; host wall clock"},
        "gpu_launches": 48 * args.steps,
        "clocks": clocks,
        "cases_us": table,
        "headline": headline,
        "prompt_gemm": prompt,
        "moe": moe1,
        "f32in_and_glu": glu1,
        "reference_kernels": refk,
        "sharded": sharded,
    }, parity_ok


# ---- the reference arm -----------------------------------------------------------------------------------------------

def run_reference(args, rank: int, world: int):
    """The reference's CPU path on this box's host cores (rank 0 only; the other ranks exit without work): every step
    runs the reference's ref_value over the step's outputs -- all of them when steps + warm-up fit the budget (the
    default run: 25 full steps), else the same leading rows of every case; value and ms_per_step are those outputs'
    bytes and time, unscaled. Inputs from the oracle (no libvkb.so)."""
    if rank != 0:
        return None
    cases = host_cases(source="oracle")
    threads = os.cpu_count() or 1
    frac = cpu_plan(cases, threads, args.steps + args.warmup, budget_s=150.0)
    for _ in range(args.warmup):
        cpu_reference(cases, threads, frac)
    t, nb = 0.0, 0.0
    for _ in range(args.steps):
        dt, b = cpu_reference(cases, threads, frac)
        t += dt
        nb += b
    value = nb / t / 1e9
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
        "config": bench_config(),
        "parallelism": "host CPU, rank 0 only",
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": cpu_kind(),
                         "sample": cpu_sample_text(frac, len(cases))},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-chunks", type=int, default=4,
                    help="graphs per end-to-end step; each chunk's outputs are read back while the next one runs")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    parity_ok = True
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
        res, parity_ok = run_ours(args, rank, world, local_rank, dist)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)
    if not parity_ok:   # a sharded result differs from the one-GPU kernel's
        sys.exit(1)


if __name__ == "__main__":
    main()
