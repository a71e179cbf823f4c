"""The sabotage negative control for every packed-weight entry point that the decode, MoE and prompt parity files do
not already cover: broken packing must fail the check (the reference's BAKEOFF_SABOTAGE, src/bakeoff.cu:20-23,
:845-846: Q4 nibbles swapped, Q8 and 2-bit code pairs swapped), while the same call on correctly packed weights passes.

  Q8 prompt GEMM (vkb_gemm_q8_tc), gate + up + SwiGLU (vkb_gate_up_glu_q4[_f32in]), the fp32-in decode (pipelined and
  general kernels), the Q8 and 2-bit MoE, and the GGUF device repack (blocks whose nibbles / code pairs are swapped,
  repacked on the GPU, then multiplied, against the values of the intact blocks)."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

from gpu_util import device_weights, random_codes, uniform_x

pytestmark = pytest.mark.gpu


def _err(y, codes, scales, x_bits):
    return O.check_error(np.asarray(y, dtype=np.float64), O.ref_value(codes, scales, x_bits),
                         O.ref_scale(codes, scales, x_bits))[0]


@pytest.mark.parametrize("M", [64, 200])
def test_q8_prompt_gemm_sabotage(cuda, M):
    import torch
    rng = np.random.default_rng(300 + M)
    N, K = 1024, 2048
    codes, scales = random_codes(rng, O.FMT_Q8, N, K)
    x_bits = uniform_x(rng, M, K)
    x = vkb.to_device_f16(x_bits)
    for sab, ok in ((False, True), (True, False)):
        q, s = device_weights(O.FMT_Q8, codes, scales, sabotage=sab)
        y = vkb.gemm_tc(q, s, x, out_f32=True, fmt=O.FMT_Q8)
        torch.cuda.synchronize()
        err = _err(y.cpu().numpy(), codes, scales, x_bits)
        assert (err <= O.TOL_FP16) if ok else (err > 1e-2), (sab, err)


@pytest.mark.parametrize("f32in", [True, False])
def test_gate_up_glu_sabotage(cuda, f32in):
    import torch
    rng = np.random.default_rng(310 + int(f32in))
    N, K, M = 2048, 2048, 4
    codes, scales = random_codes(rng, O.FMT_Q4, 2 * N, K)
    x32 = rng.uniform(-1, 1, size=(M, K)).astype(np.float32)
    x_bits = x32.astype(np.float16).view(np.uint16)
    xd = torch.from_numpy(x32).cuda() if f32in else vkb.to_device_f16(x_bits)
    for sab, ok in ((False, True), (True, False)):
        q, s = device_weights(O.FMT_Q4, codes, scales, sabotage=sab)
        out, ys = vkb.gate_up_glu_q4(q, s, xd, out_f32=True)
        torch.cuda.synchronize()
        ys_np = ys.cpu().numpy().astype(np.float64)
        err = _err(ys_np, codes, scales, x_bits)
        # the SwiGLU output against silu(g) * u of the intact product: the reference's verdict combines both
        want = O.swiglu_ref(O.ref_value(codes, scales, x_bits), N)
        err_out = float(np.max(np.abs(out.cpu().numpy() - want) / (np.abs(want) + 1e-3)))
        if ok:
            assert err <= O.TOL_EXACT and O.glu_error(out.cpu().numpy(), ys_np, N) <= 1e-5, err
        else:
            assert err > 1e-2 and err_out > 1e-2, (err, err_out)


@pytest.mark.parametrize("K", [2048, 640])   # the pipelined kernel (fp32 read in-kernel) and the general path (xh)
def test_f32in_decode_sabotage(cuda, K):
    import torch
    rng = np.random.default_rng(320 + K)
    N, M = 1031, 3
    codes, scales = random_codes(rng, O.FMT_Q4, N, K)
    x32 = rng.uniform(-1, 1, size=(M, K)).astype(np.float32)
    x_bits = x32.astype(np.float16).view(np.uint16)
    for sab, ok in ((False, True), (True, False)):
        q, s = device_weights(O.FMT_Q4, codes, scales, sabotage=sab)
        y = vkb.gemv_q4_f32in(q, s, torch.from_numpy(x32).cuda())
        torch.cuda.synchronize()
        err = _err(y.cpu().numpy(), codes, scales, x_bits)
        assert (err <= O.TOL_EXACT) if ok else (err > 1e-2), (sab, err)


@pytest.mark.parametrize("fmt", [O.FMT_Q8, O.FMT_Q2])
@pytest.mark.parametrize("T", [1, 8])
def test_moe_q8_q2_sabotage(cuda, fmt, T):
    import torch
    rng = np.random.default_rng(330 + 10 * fmt + T)
    E, N, K, k = 16, 256, 1024, 4
    cs = [random_codes(rng, fmt, N, K) for _ in range(E)]
    codes = np.stack([c for c, _ in cs])
    scales = np.stack([s for _, s in cs])
    idx = vkb.synth_topk(40 + T, T, E, k)
    x_bits = uniform_x(rng, T, K)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x_bits)
    for sab, ok in ((False, True), (True, False)):
        packed = np.stack([O.pack(fmt, codes[e], sabotage=sab) for e in range(E)])
        q = vkb.to_device_packed(packed.reshape(E * N, -1), "cuda").view(E, N, -1)
        s = vkb.to_device_f16(scales.reshape(E * N, -1), "cuda").view(E, N, K // 32)
        y = vkb.moe(fmt, q, s, torch.from_numpy(idx).cuda(), vkb.to_device_f16(x_bits), out_f32=True)
        torch.cuda.synchronize()
        err = O.check_error(y.cpu().numpy().reshape(T * k, N).astype(np.float64), ref, mag)[0]
        assert (err <= O.TOL_EXACT) if ok else (err > 1e-2), (sab, err)


def _gguf_sabotage(fmt, blocks):
    """GGUF blocks with the reference's sabotage applied inside each block: Q4_0 nibbles of every byte swapped
    (element j <-> j + 16), Q8_0 every pair of codes swapped."""
    b = blocks.reshape(-1, 18 if fmt == O.FMT_Q4 else 34).copy()
    if fmt == O.FMT_Q4:
        qs = b[:, 2:]
        b[:, 2:] = ((qs & 15) << 4) | (qs >> 4)
    else:
        qs = b[:, 2:].reshape(-1, 16, 2)
        b[:, 2:] = qs[:, :, ::-1].reshape(-1, 32)
    return b.reshape(-1)


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8])
def test_gguf_device_repack_sabotage(cuda, fmt):
    import torch
    rng = np.random.default_rng(340 + fmt)
    N, K, M = 1024, 2048, 4
    codes, scales = random_codes(rng, fmt, N, K)
    blocks = O.gguf_blocks(fmt, codes, scales)
    w = O.gguf_values(fmt, blocks, N, K)              # the intact blocks' values
    x_bits = uniform_x(rng, M, K)
    xf = x_bits.view(np.float16).astype(np.float64)
    ref, mag = xf @ w.T, np.abs(xf) @ np.abs(w).T
    for sab, ok in ((False, True), (True, False)):
        blk = _gguf_sabotage(fmt, blocks) if sab else blocks
        qd, sd = vkb.gguf_to_vkb_device(fmt, torch.from_numpy(blk).cuda(), N, K)
        y = vkb.gemv(fmt, qd, sd, vkb.to_device_f16(x_bits), out_f32=True)
        torch.cuda.synchronize()
        err = O.check_error(y.cpu().numpy().astype(np.float64), ref, mag)[0]
        assert (err <= O.TOL_EXACT) if ok else (err > 1e-2), (sab, err)
    assert vkb.device_status() == 0
