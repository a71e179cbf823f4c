"""Property tests (hypothesis) of libvkb.so's host functions against the oracle, on random shapes and values: the
packers for every format (with and without sabotage), the quantiser (the reference's absmax rules, src/bakeoff.cu:
200-219, :486-490, src/stage3_lut.cuh:90-97, restated in oracle/oracle.py), and the GGUF Q4_0 / Q8_0 converters
(both directions). Host only: no GPU; sizes stay small so the whole file runs in seconds."""
import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

import vkb
from oracle import oracle as O

FMTS = [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2]
RANGE = {O.FMT_Q4: (-8, 7), O.FMT_Q8: (-127, 127), O.FMT_Q2: (-2, 1)}
KUNIT = {O.FMT_Q4: 32, O.FMT_Q8: 32, O.FMT_Q2: 64}   # the smallest K each packed layout takes


@st.composite
def codes_case(draw):
    fmt = draw(st.sampled_from(FMTS))
    N = draw(st.integers(1, 40))
    K = KUNIT[fmt] * draw(st.integers(1, 12))
    seed = draw(st.integers(0, 2**31 - 1))
    lo, hi = RANGE[fmt]
    codes = np.random.default_rng(seed).integers(lo, hi + 1, size=(N, K)).astype(np.int8)
    return fmt, codes


@settings(max_examples=60, deadline=None)
@given(codes_case(), st.booleans())
def test_pack_matches_oracle_on_random_shapes(case, sabotage):
    fmt, codes = case
    mine = np.asarray(vkb.pack(fmt, codes, sabotage=sabotage))
    ref = np.asarray(O.pack(fmt, codes, sabotage=sabotage))
    assert np.array_equal(mine.view(np.uint8), ref.view(np.uint8))
    assert vkb.lib().vkb_packed_bytes(fmt, codes.shape[0], codes.shape[1]) == mine.nbytes


@settings(max_examples=40, deadline=None)
@given(st.sampled_from(FMTS), st.integers(1, 24), st.integers(1, 8), st.integers(0, 2**31 - 1),
       st.sampled_from([1e-4, 0.02, 1.0, 300.0]))
def test_quantize_matches_oracle_on_random_weights(fmt, N, kb, seed, scale):
    K = KUNIT[fmt] * kb
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * scale).astype(np.float32)
    w[rng.random((N, K)) < 0.05] = 0.0                     # sparse zeros, and now and then a whole zero block
    if N > 1:
        w[1, :32] = 0.0
    c1, s1 = vkb.quantize(fmt, w)
    c2, s2 = O.quantize(fmt, w)
    assert np.array_equal(s1, s2) and np.array_equal(c1, c2)
    lo, hi = RANGE[fmt]
    assert c1.min() >= lo and c1.max() <= hi


@settings(max_examples=40, deadline=None)
@given(st.sampled_from([O.FMT_Q4, O.FMT_Q8]), st.integers(1, 24), st.integers(1, 10), st.integers(0, 2**31 - 1))
def test_gguf_round_trip_on_random_shapes(fmt, N, kb, seed):
    K = 32 * kb
    rng = np.random.default_rng(seed)
    lo, hi = RANGE[fmt]
    codes = rng.integers(lo, hi + 1, size=(N, K)).astype(np.int8)
    scales = rng.uniform(1e-4, 4.0, size=(N, K // 32)).astype(np.float16).view(np.uint16)
    blocks = O.gguf_blocks(fmt, codes, scales)
    q, s = vkb.gguf_to_vkb(fmt, blocks, N, K)
    assert np.array_equal(q, np.asarray(vkb.pack(fmt, codes)).view(np.uint8).reshape(-1))
    assert np.array_equal(s, scales)
    assert np.array_equal(vkb.vkb_to_gguf(fmt, q, s, N, K), blocks)
    # the values the blocks encode are the ones the split layout encodes
    w = O.gguf_values(fmt, blocks, N, K)
    assert np.array_equal(w, codes.astype(np.float64) * np.repeat(scales.view(np.float16).astype(np.float64), 32,
                                                                   axis=1))


@pytest.mark.parametrize("fmt", FMTS)
def test_pack_rejects_ragged_k(fmt):
    """K not a multiple of the layout's unit: nothing written, an error code (the oracle's packers refuse it too)."""
    L = vkb.lib()
    N, K = 3, KUNIT[fmt] + 8
    codes = np.zeros((N, K), np.int8)
    out = np.zeros(1024, np.uint8)
    assert L.vkb_pack(fmt, codes.ctypes.data, N, K, 0, out.ctypes.data) != 0
    assert not out.any()
