"""CPU tests: the oracle pinned to the reference's own outputs (tests/golden), and the library's host-side format
code checked against the oracle. Mirrors the reference's --check inputs (src/bakeoff.cu:475-513): mt19937(1234)
weights, U[-1,1] activations, +bigx and +tinyx."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle import refbind


def _tables(golden, fmt):
    for name in ("a", "odd"):
        p = f"{name}_q{ {O.FMT_Q4: 4, O.FMT_Q8: 8, O.FMT_Q2: 2}[fmt] }_"
        yield p, golden[p + "codes"], golden[p + "scales"]


def test_probe_matches_survey(golden):
    # mt19937(1234), 8192x2048 Q4: first packed word 0xcc97d973 and y[0] = 1.79625016 (the reference run here)
    assert int(golden["probe_packed_row0"][0]) == 0xCC97D973
    assert golden["probe_val"][0, 0] == pytest.approx(1.79625016, abs=5e-9)
    assert np.array_equal(O.pack_q4(golden["probe_codes_row0"][None, :])[0], golden["probe_packed_row0"])


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q2])
def test_pack_matches_reference(golden, fmt):
    for p, codes, _ in _tables(golden, fmt):
        assert np.array_equal(O.pack(fmt, codes), golden[p + "packed"]), p
        assert np.array_equal(O.pack(fmt, codes, sabotage=True), golden[p + "packed_sab"]), p
        unpack = O.unpack_q4 if fmt == O.FMT_Q4 else O.unpack_q2
        assert np.array_equal(unpack(golden[p + "packed"], codes.shape[1]), codes)


def test_q8_pack_is_raw_codes_and_sabotage_swaps_pairs():
    codes = np.arange(-64, 64, dtype=np.int8).reshape(2, 64)
    assert np.array_equal(O.pack_q8(codes), codes)
    sab = O.pack_q8(codes, sabotage=True).reshape(-1)
    assert np.array_equal(sab[0::2], codes.reshape(-1)[1::2]) and np.array_equal(sab[1::2], codes.reshape(-1)[0::2])


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8])
def test_ref_value_matches_reference(golden, fmt):
    for p, codes, scales in _tables(golden, fmt):
        for ci in range(5):
            x = golden[p + f"x{ci}"]
            val, mag = O.ref_value(codes, scales, x), O.ref_scale(codes, scales, x)
            np.testing.assert_allclose(val, golden[p + f"val{ci}"], rtol=1e-12, atol=1e-12 * np.abs(mag).max())
            np.testing.assert_allclose(mag, golden[p + f"mag{ci}"], rtol=1e-12)


def test_ref_q2_matches_reference(golden):
    for p, codes, scales in _tables(golden, O.FMT_Q2):
        x = golden[p + "x0"]
        np.testing.assert_allclose(O.ref_q2(codes, scales, x), golden[p + "val0"], rtol=1e-12,
                                   atol=1e-12 * golden[p + "mag0"].max())
        np.testing.assert_allclose(O.ref_q2_mag(codes, scales, x), golden[p + "mag0"], rtol=1e-12)


def test_check_metric_is_the_references():
    ref = np.array([[1.0, -2.0]])
    mag = np.array([[2.0, 4.0]])
    err, m, n = O.check_error(np.array([[1.001, -2.0]]), ref, mag)
    assert err == pytest.approx(0.0005) and (m, n) == (0, 0)
    assert O.check_error(np.array([[np.nan, 0.0]]), ref, mag)[0] == np.inf


def test_golden_reproducible_from_reference():
    """The fixtures are what the reference computes (skipped where oracle/_ref could not be built)."""
    if refbind.load() is None:
        pytest.skip("oracle/_ref/libvkbref.so not built")
    rng = refbind.Rng(1234)
    codes, scales = rng.make_weights(64, 256, 4)
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.npz"))
    assert np.array_equal(codes, g["a_q4_codes"]) and np.array_equal(scales, g["a_q4_scales"])


def test_quantizer_rule():
    w = np.zeros((1, 64), np.float32)
    w[0, :32] = np.linspace(-1.0, 1.0, 32, dtype=np.float32)
    codes, scales = O.quantize(O.FMT_Q4, w)
    d = float(scales.view(np.float16)[0, 0])
    assert d == pytest.approx(1.0 / 8, rel=1e-3)
    assert codes[0, :32].min() == -8 and codes[0, :32].max() == 7      # +1/d = 8 rounds to 8, clamps to 7
    assert np.all(codes[0, 32:] == 0) and scales.view(np.float16)[0, 1] == 0
    for fmt, lo, hi in ((O.FMT_Q8, -127, 127), (O.FMT_Q2, -2, 1)):
        c, _ = O.quantize(fmt, w)
        assert c.min() >= lo and c.max() <= hi


def test_swiglu_ref_and_glu_error():
    """silu(g) * u over a stacked product (src/stage5_gap8.cuh:232-238) and the reference's relative check."""
    ys = np.array([[0.0, 1.0, 2.0, 3.0], [-2.0, 0.5, 4.0, -1.0]])
    want = np.array([[0.0, 3.0 / (1.0 + np.exp(-1.0))],
                     [-2.0 / (1.0 + np.exp(2.0)) * 4.0, 0.5 / (1.0 + np.exp(-0.5)) * -1.0]])
    assert np.allclose(O.swiglu_ref(ys, 2), want, rtol=1e-15, atol=0)
    assert O.glu_error(want, ys, 2) < 1e-12
    bad = want.copy()
    bad[1, 1] *= 1.001
    assert O.glu_error(bad, ys, 2) > 5e-4


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8])
def test_gguf_blocks_values(fmt):
    """The oracle's GGUF blocks encode exactly code * scale (the reference's value model, src/bakeoff.cu:5-7)."""
    rng = np.random.default_rng(11 + fmt)
    lo, hi = (-8, 7) if fmt == O.FMT_Q4 else (-127, 127)
    codes = rng.integers(lo, hi + 1, size=(5, 96)).astype(np.int8)
    scales = rng.uniform(0.004, 0.02, size=(5, 3)).astype(np.float16).view(np.uint16)
    blocks = O.gguf_blocks(fmt, codes, scales)
    assert blocks.size == 5 * 3 * (18 if fmt == O.FMT_Q4 else 34)
    want = codes.astype(np.float64) * np.repeat(scales.view(np.float16).astype(np.float64), 32, axis=1)
    assert np.array_equal(O.gguf_values(fmt, blocks, 5, 96), want)


def test_oracle_inputs_match_the_library():
    """bench.py's reference arm builds the benchmark's inputs without libvkb.so: the oracle's normal draws, numpy
    quantiser and fp16 rounding must equal the library's bit for bit (full configs[0] table, and odd lengths)."""
    if refbind.load() is None:
        pytest.skip("oracle/_ref/libvkbref.so not built")
    import vkb
    for seed, shape, std in ((0, (8192, 2048), 0.02), (3, (4, 2048), 1.0), (5, (7,), 1.0)):
        a, b = refbind.synth_normal(seed, shape, std), vkb.synth_normal(seed, shape, std)
        assert a.dtype == b.dtype == np.float32 and np.array_equal(a.view(np.uint32), b.view(np.uint32))
    w = refbind.synth_normal(0, (512, 2048), 0.02)
    for fmt in (O.FMT_Q4, O.FMT_Q8, O.FMT_Q2):
        c0, s0 = O.quantize(fmt, w)
        c1, s1 = vkb.quantize(fmt, w)
        assert np.array_equal(c0, c1) and np.array_equal(s0, s1), fmt
    x = refbind.synth_normal(2, (8, 2048), 1.0)
    assert np.array_equal(x.astype(np.float16).view(np.uint16), vkb.to_f16_bits(x))
