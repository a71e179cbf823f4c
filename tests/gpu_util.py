"""Helpers shared by the GPU parity tests: build device-side weight sets from integer codes, run the library through
its C ABI, and score against the oracle with the reference's metric (src/bakeoff.cu:565-583)."""
from __future__ import annotations

import numpy as np

import vkb
from oracle import oracle as O

LO_HI = {O.FMT_Q4: (-8, 7), O.FMT_Q8: (-127, 127), O.FMT_Q2: (-2, 1)}


def random_codes(rng, fmt, N, K):
    lo, hi = LO_HI[fmt]
    codes = rng.integers(lo, hi + 1, size=(N, K)).astype(np.int8)
    # the reference's scale distribution: U[0.004, 0.02] (x0.06 for q8), src/bakeoff.cu:204-206
    mul = 0.06 if fmt == O.FMT_Q8 else 1.0
    scales = (rng.uniform(0.004, 0.02, size=(N, K // 32)) * mul).astype(np.float16).view(np.uint16)
    return codes, scales


def baseline_weights(fmt, N, K, seed=0):
    """BASELINE's synthetic weights: fp32 N(0, 0.02) from seed, quantised per 32-value block."""
    w = vkb.synth_normal(seed, (N, K), 0.02)
    return vkb.quantize(fmt, w)


def normal_x(M, K, seed=1):
    return vkb.to_f16_bits(vkb.synth_normal(seed, (M, K), 1.0))


def uniform_x(rng, M, K, mul=1.0):
    return (rng.uniform(-1.0, 1.0, size=(M, K)) * mul).astype(np.float16).view(np.uint16)


def device_weights(fmt, codes, scales, sabotage=False, device="cuda"):
    packed = O.pack(fmt, codes, sabotage=sabotage)
    return vkb.to_device_packed(packed, device), vkb.to_device_f16(scales, device)


def run_gemv(fmt, q, s, x_bits, out_f32, device="cuda"):
    import torch
    x = vkb.to_device_f16(x_bits, device)
    y = vkb.gemv(fmt, q, s, x, out_f32=out_f32)
    torch.cuda.synchronize()
    return y.float().cpu().numpy().astype(np.float64)


def score(y, codes, scales, x_bits):
    ref = O.ref_value(codes, scales, x_bits)
    mag = O.ref_scale(codes, scales, x_bits)
    return O.check_error(y, ref, mag), ref
