"""Property tests (hypothesis) pinning the numpy oracle to the reference's own host code (oracle/_ref/libvkbref.so,
compiled from src/bakeoff.cu) on random shapes, codes, scales and activations, beyond the fixed golden vectors:

- pack_q4 / pack_q2 with and without sabotage (src/bakeoff.cu:210-219, src/stage3_lut.cuh:90-97): bit for bit;
- ref_value / ref_scale over M tokens (src/bakeoff.cu:221-235) and ref_q2 (src/stage2.cuh:261-270): to 1e-12 of
  sum |x w| (the sums are taken in another order);
- the multi-threaded CPU baseline (ref_gemv_mt in oracle/ref_shim.cu) over any row window and thread count: the same
  doubles as the single-threaded reference, bit for bit, and its checksum is their sum.

Host only; sizes stay small so the file runs in seconds."""
import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from oracle import oracle as O
from oracle import refbind

@pytest.fixture(autouse=True)
def _reference_library():
    # loaded when a test here runs, not at collection (a -m gpu run collects this file without loading it)
    if refbind.load() is None:
        pytest.skip("oracle/_ref/libvkbref.so not built")


RANGE = {O.FMT_Q4: (-8, 7), O.FMT_Q8: (-127, 127), O.FMT_Q2: (-2, 1)}


def _case(fmt, N, kb, M, seed, xscale):
    rng = np.random.default_rng(seed)
    lo, hi = RANGE[fmt]
    K = (64 if fmt == O.FMT_Q2 else 32) * kb
    codes = rng.integers(lo, hi + 1, size=(N, K)).astype(np.int8)
    scales = rng.uniform(1e-4, 0.05, size=(N, K // 32)).astype(np.float16).view(np.uint16)
    x = (rng.uniform(-1, 1, size=(M, K)) * xscale).astype(np.float16).view(np.uint16)
    return codes, scales, x


@settings(max_examples=40, deadline=None)
@given(st.sampled_from([O.FMT_Q4, O.FMT_Q2]), st.integers(1, 33), st.integers(1, 6), st.integers(0, 2**31 - 1),
       st.booleans())
def test_packers_match_the_reference(fmt, N, kb, seed, sabotage):
    codes, scales, _ = _case(fmt, N, kb, 1, seed, 1.0)
    mine = O.pack(fmt, codes, sabotage=sabotage)
    ref = (refbind.pack_q4 if fmt == O.FMT_Q4 else refbind.pack_q2)(codes, scales, sabotage=sabotage)
    assert np.array_equal(np.asarray(mine).view(np.uint8).reshape(-1), ref.view(np.uint8).reshape(-1))


@settings(max_examples=40, deadline=None)
@given(st.sampled_from([O.FMT_Q4, O.FMT_Q8]), st.integers(1, 33), st.integers(1, 6), st.integers(1, 8),
       st.integers(0, 2**31 - 1), st.sampled_from([1e-3, 1.0, 60.0, 6e4]))
def test_ref_value_and_scale_match_the_reference(fmt, N, kb, M, seed, xscale):
    codes, scales, x = _case(fmt, N, kb, M, seed, xscale)
    val, mag = refbind.values(codes, scales, x)
    v, m = O.ref_value(codes, scales, x), O.ref_scale(codes, scales, x)
    assert np.all(np.abs(m - mag) <= 1e-12 * (mag + 1e-300))
    assert np.all(np.abs(v - val) <= 1e-12 * (mag + 1e-300))


@settings(max_examples=30, deadline=None)
@given(st.integers(1, 33), st.integers(1, 4), st.integers(0, 2**31 - 1))
def test_ref_q2_matches_the_reference(N, kb, seed):
    codes, scales, x = _case(O.FMT_Q2, N, kb, 1, seed, 1.0)
    val, mag = refbind.q2_values(codes, scales, x[0])
    v = O.ref_q2(codes, scales, x)[0]
    m = O.ref_scale(codes, scales, x)[0]
    assert np.all(np.abs(m - mag) <= 1e-12 * (mag + 1e-300))
    assert np.all(np.abs(v - val) <= 1e-12 * (mag + 1e-300))


@settings(max_examples=30, deadline=None)
@given(st.integers(1, 40), st.integers(1, 4), st.integers(1, 8), st.integers(0, 2**31 - 1), st.integers(1, 9),
       st.data())
def test_cpu_baseline_is_the_reference(N, kb, M, seed, threads, data):
    codes, scales, x = _case(O.FMT_Q4, N, kb, M, seed, 1.0)
    row0 = data.draw(st.integers(0, N - 1))
    nrows = data.draw(st.integers(1, N - row0))
    out = np.full((M, nrows), np.nan)
    checksum = refbind.gemv_mt(codes, scales, x, row0, nrows, threads, out=out)
    val, _ = refbind.values(codes, scales, x)
    assert np.array_equal(out, val[:, row0:row0 + nrows])
    assert checksum == pytest.approx(float(out.sum()), rel=1e-12, abs=1e-9)
