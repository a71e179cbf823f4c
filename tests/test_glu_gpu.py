"""GPU parity of the fp32-activation decode entry (vkb_gemv_q4_f32in) and the fused gate + up + SwiGLU
(vkb_gate_up_glu_q4_f32in / vkb_gate_up_glu_q4) through the C ABI.

- fp32 in: the result must match the fp16-activation GEMV on the activations rounded to fp16 (the reference's
  conversion step, src/stage5_gap8.cuh:207-228) to fp32 summation-order differences, on both of the library's
  paths: rounding inside the pipelined kernel, and the separate conversion into xh followed by the general kernel
  (K = 640, not a multiple of 256), and the oracle.
- gate/up: the reference's own check (src/bakeoff.cu:370-406) on its table (Qwen3-1.7B MLP, gate and up 6144x2048
  stacked): the stacked product against the oracle (exact-code class here, 1e-4; the reference allows 2e-3), and
  out against silu(gate) * up recomputed from that product (1e-5).
"""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

from gpu_util import device_weights, random_codes

pytestmark = pytest.mark.gpu


def _x32(rng, M, K, mul=1.0):
    """fp32 activations that are not all fp16-representable (the kernel must round them)."""
    return (rng.uniform(-1.0, 1.0, size=(M, K)) * mul).astype(np.float32)


@pytest.mark.parametrize("N,K,M", [(8192, 2048, 1), (8192, 2048, 2), (4096, 2048, 4), (2048, 2048, 8),
                                   (1031, 2560, 3), (2048, 6144, 8), (640, 640, 1)])
def test_gemv_f32in_equals_rounded_f16(cuda, N, K, M):
    import torch
    rng = np.random.default_rng(N + 7 * K + M)
    codes, scales = random_codes(rng, O.FMT_Q4, N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x32 = _x32(rng, M, K)
    xd = torch.from_numpy(x32).cuda()
    y = vkb.gemv_q4_f32in(q, s, xd)
    xh_bits = x32.astype(np.float16).view(np.uint16)   # round to nearest even, as the reference's conversion
    y16 = vkb.gemv(O.FMT_Q4, q, s, vkb.to_device_f16(xh_bits), out_f32=True)
    torch.cuda.synchronize()
    mag = O.ref_scale(codes, scales, xh_bits)
    yn, y16n = y.cpu().numpy().astype(np.float64), y16.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(yn - y16n) / (mag + 1e-12)) <= 1e-6
    err = O.check_error(yn, O.ref_value(codes, scales, xh_bits), mag)[0]
    assert err <= O.TOL_EXACT, err
    assert vkb.device_status() == 0


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_gate_up_glu_reference_check(cuda, M):
    import torch
    N, K = 6144, 2048
    rng = np.random.default_rng(100 + M)
    codes, scales = random_codes(rng, O.FMT_Q4, 2 * N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x32 = _x32(rng, M, K)
    out, ys = vkb.gate_up_glu_q4(q, s, torch.from_numpy(x32).cuda())
    torch.cuda.synchronize()
    ys_np = ys.cpu().numpy().astype(np.float64)
    xh_bits = x32.astype(np.float16).view(np.uint16)
    err_mm = O.check_error(ys_np, O.ref_value(codes, scales, xh_bits), O.ref_scale(codes, scales, xh_bits))[0]
    err_glu = O.glu_error(out.cpu().numpy(), ys_np, N)
    assert err_mm <= O.TOL_EXACT, err_mm
    assert err_glu <= 1e-5, err_glu
    assert vkb.device_status() == 0


@pytest.mark.parametrize("N,K,M", [(1000, 2048, 5), (256, 6144, 8), (6144, 2048, 1)])
def test_gate_up_glu_shapes_and_outputs(cuda, N, K, M):
    """Ragged N (1000: the last output tile pair is partial in both halves), long rows (K = 6144), a single tile pair
    per CTA (N = 256), fp16 activations with fp16 and fp32 outputs, and no stacked output."""
    import torch
    rng = np.random.default_rng(N + K + M)
    codes, scales = random_codes(rng, O.FMT_Q4, 2 * N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x32 = _x32(rng, M, K)
    xh_bits = x32.astype(np.float16).view(np.uint16)
    ref = O.ref_value(codes, scales, xh_bits)
    mag = O.ref_scale(codes, scales, xh_bits)
    want = O.swiglu_ref(ref, N)
    # fp32 in, fp32 out, with the stacked product
    out, ys = vkb.gate_up_glu_q4(q, s, torch.from_numpy(x32).cuda())
    # fp16 in, fp32 out, no stacked product: the same numbers up to fp32 summation order
    x16 = vkb.to_device_f16(xh_bits)
    out_b, none = vkb.gate_up_glu_q4(q, s, x16, out_f32=True, want_stack=False)
    # fp16 in, fp16 out
    out_h, _ = vkb.gate_up_glu_q4(q, s, x16, out_f32=False, want_stack=False)
    torch.cuda.synchronize()
    assert none is None
    ys_np = ys.cpu().numpy().astype(np.float64)
    assert O.check_error(ys_np, ref, mag)[0] <= O.TOL_EXACT
    assert O.glu_error(out.cpu().numpy(), ys_np, N) <= 1e-5
    # gate / up errors of relative size `rel` (of sum |x w|) propagated through silu(g) * u
    g, u = ref[:, :N], ref[:, N:]
    sg = 1.0 / (1.0 + np.exp(-g))
    dsilu = sg * (1.0 + g * (1.0 - sg))

    def bound(rel):
        return rel * (np.abs(dsilu * u) * mag[:, :N] + np.abs(g * sg) * mag[:, N:]) + 1e-6 * np.abs(want) + 1e-7

    on, ob = out.cpu().numpy().astype(np.float64), out_b.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(on - ob) <= bound(1e-6))      # the two paths: summation order only
    assert torch.equal(out_h, out_b.half())
    assert np.all(np.abs(on - want) <= bound(O.TOL_EXACT))   # the float64 SwiGLU of the oracle's product
    assert vkb.device_status() == 0


def test_glu_rejects_unsupported(cuda):
    import torch
    N, K = 256, 2048
    rng = np.random.default_rng(3)
    codes, scales = random_codes(rng, O.FMT_Q4, 2 * N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    L = vkb.lib()
    x = torch.zeros((9, K), dtype=torch.float32, device="cuda")
    out = torch.zeros((9, N), dtype=torch.float32, device="cuda")
    xh = torch.zeros((9, K), dtype=torch.float16, device="cuda")
    # 9 tokens: unsupported, nothing launched, out untouched
    rc = L.vkb_gate_up_glu_q4_f32in(vkb._ptr(q), vkb._ptr(s), vkb._ptr(x), vkb._ptr(xh), None, vkb._ptr(out), N, K, 9,
                                    vkb._stream())
    assert rc == vkb.EUNSUPPORTED
    rc = L.vkb_gemv_q4_f32in(vkb._ptr(q), vkb._ptr(s), vkb._ptr(x), vkb._ptr(xh), vkb._ptr(out), N, K, 9,
                             vkb._stream())
    assert rc == vkb.EUNSUPPORTED
    # K % 256 != 0: the fused gate/up kernel is the pipelined one only
    rc = L.vkb_gate_up_glu_q4(vkb._ptr(q), vkb._ptr(s), vkb._ptr(xh), None, vkb._ptr(out), 1, N, 640, 1,
                              vkb._stream())
    assert rc == vkb.EUNSUPPORTED
    torch.cuda.synchronize()
    assert float(out.abs().sum()) == 0.0
