"""GGUF Q4_0 / Q8_0 blocks repacked on the GPU (vkb_gguf_to_vkb_device): bit-identical to the host conversion, and a
decode GEMV on the repacked weights against the values the GGUF blocks encode (the oracle's gguf_values)."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

from gpu_util import uniform_x

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8])
@pytest.mark.parametrize("N,K", [(1031, 2048), (4096, 4096), (3, 32)])
def test_gguf_device_repack(cuda, fmt, N, K):
    import torch
    rng = np.random.default_rng(N + K + 10 * fmt)
    lo, hi = (-8, 7) if fmt == O.FMT_Q4 else (-127, 127)
    codes = rng.integers(lo, hi + 1, size=(N, K)).astype(np.int8)
    mul = 0.06 if fmt == O.FMT_Q8 else 1.0
    scales = (rng.uniform(0.004, 0.02, size=(N, K // 32)) * mul).astype(np.float16).view(np.uint16)
    blocks = O.gguf_blocks(fmt, codes, scales)
    qd, sd = vkb.gguf_to_vkb_device(fmt, torch.from_numpy(blocks).cuda(), N, K)
    qh, sh = vkb.gguf_to_vkb(fmt, blocks, N, K)
    torch.cuda.synchronize()
    assert np.array_equal(qd.cpu().numpy(), qh)
    assert np.array_equal(sd.cpu().numpy().view(np.uint16), sh)
    if N >= 16 and K % 256 == 0:   # decode on the repacked weights
        M = 4
        x_bits = uniform_x(rng, M, K)
        y = vkb.gemv(fmt, qd, sd, vkb.to_device_f16(x_bits), out_f32=True)
        torch.cuda.synchronize()
        w = O.gguf_values(fmt, blocks, N, K)
        xf = x_bits.view(np.float16).astype(np.float64)
        ref, mag = xf @ w.T, np.abs(xf) @ np.abs(w).T
        err = O.check_error(y.cpu().numpy().astype(np.float64), ref, mag)[0]
        assert err <= O.TOL_EXACT, err
    assert vkb.device_status() == 0
