"""GPU checks of vkb_dequant (the reference's dequant_q4, src/bakeoff.cu:52-68, for every format) and of the
reference's dq4+cublas control built on it (src/bakeoff.cu:687-690): the dense copy is bit-exact against the host's
one rounding of code * scale (fp16 and bf16), and a plain PyTorch fp16 GEMM on it meets the oracle with the
reference's fp16-class tolerance."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

from gpu_util import device_weights, random_codes, uniform_x

pytestmark = pytest.mark.gpu


def _host_dense(codes, scales, bf16):
    import torch
    v = codes.astype(np.float32) * np.repeat(scales.view(np.float16).astype(np.float32), 32, axis=1)
    t = torch.from_numpy(v)
    return t.to(torch.bfloat16) if bf16 else t.to(torch.float16)   # round to nearest even, once


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2])
@pytest.mark.parametrize("N,K", [(1031, 768), (64, 2048), (3, 64)])
@pytest.mark.parametrize("bf16", [False, True])
def test_dequant_bit_exact(cuda, fmt, N, K, bf16):
    import torch
    rng = np.random.default_rng(N + K + fmt)
    codes, scales = random_codes(rng, fmt, N, K)
    q, s = device_weights(fmt, codes, scales)
    w = vkb.dequant(fmt, q, s, N, K, bf16=bf16)
    torch.cuda.synchronize()
    want = _host_dense(codes, scales, bf16)
    assert torch.equal(w.cpu().view(torch.int16), want.view(torch.int16))


def test_dequant_rejects_bad_arguments(cuda):
    import torch
    rng = np.random.default_rng(5)
    codes, scales = random_codes(rng, O.FMT_Q2, 16, 96)
    q, s = device_weights(O.FMT_Q2, codes, scales)
    w = torch.empty((16, 96), dtype=torch.float16, device="cuda")
    L = vkb.lib()
    assert L.vkb_dequant(O.FMT_Q2, vkb._ptr(q), vkb._ptr(s), vkb._ptr(w), 16, 96, 0, None) == vkb.EUNSUPPORTED  # K % 64
    assert L.vkb_dequant(7, vkb._ptr(q), vkb._ptr(s), vkb._ptr(w), 16, 96, 0, None) == vkb.EINVAL
    assert L.vkb_dequant(O.FMT_Q4, None, vkb._ptr(s), vkb._ptr(w), 16, 96, 0, None) == vkb.EINVAL


@pytest.mark.parametrize("N,K,M", [(2560, 6144, 64), (1031, 768, 8)])
def test_dq4_cublas_control(cuda, N, K, M):
    """The control path: GPU dequantisation, then a plain fp16 PyTorch GEMM (cuBLAS, fp32 accumulation)."""
    import torch
    rng = np.random.default_rng(N + M)
    codes, scales = random_codes(rng, O.FMT_Q4, N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x_bits = uniform_x(rng, M, K)
    w = vkb.dequant(O.FMT_Q4, q, s, N, K)
    x = vkb.to_device_f16(x_bits)
    y = torch.matmul(x, w.t()).float()   # fp16 in and out, fp32 accumulation (the reference control's class)
    torch.cuda.synchronize()
    err, m, n = O.check_error(y.cpu().numpy().astype(np.float64), O.ref_value(codes, scales, x_bits),
                              O.ref_scale(codes, scales, x_bits))
    assert err <= O.TOL_FP16, (err, m, n)
