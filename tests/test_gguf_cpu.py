"""GGUF Q4_0 / Q8_0 interop of libvkb.so's host functions (vkb_gguf_to_vkb / vkb_vkb_to_gguf): blocks built by the
oracle from the GGUF layout convert to exactly what vkb_pack writes from the same codes (and the scales unchanged),
and back to the same blocks. Host only: no GPU."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8])
@pytest.mark.parametrize("N,K", [(1, 32), (7, 96), (64, 2048)])
def test_gguf_round_trip(fmt, N, K):
    rng = np.random.default_rng(N * 1000 + K + fmt)
    lo, hi = (-8, 7) if fmt == O.FMT_Q4 else (-127, 127)
    codes = rng.integers(lo, hi + 1, size=(N, K)).astype(np.int8)
    scales = rng.uniform(0.004, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
    blocks = O.gguf_blocks(fmt, codes, scales)
    assert vkb.lib().vkb_gguf_bytes(fmt, N, K) == blocks.size
    q, s = vkb.gguf_to_vkb(fmt, blocks, N, K)
    assert np.array_equal(q, np.asarray(vkb.pack(fmt, codes)).view(np.uint8).reshape(-1))
    assert np.array_equal(s, scales)
    assert np.array_equal(vkb.vkb_to_gguf(fmt, q, s, N, K), blocks)


def test_gguf_rejects():
    L = vkb.lib()
    buf = np.zeros(64, np.uint8)
    assert L.vkb_gguf_to_vkb(O.FMT_Q2, buf.ctypes.data, 1, 32, buf.ctypes.data, buf.ctypes.data) != 0
    assert L.vkb_gguf_to_vkb(O.FMT_Q4, buf.ctypes.data, 1, 48, buf.ctypes.data, buf.ctypes.data) != 0
    assert L.vkb_gguf_bytes(O.FMT_Q4, 1, 40) == 0
