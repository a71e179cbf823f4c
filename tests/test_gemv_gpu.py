"""GPU parity of the decode GEMV family (Q4 / Q8 / Q2, 1..8 tokens) against the oracle, through the C ABI.

Mirrors the reference's --check (src/bakeoff.cu:475-649): the reference's own known-answer vectors (tests/golden),
its +bigx / +tinyx stress inputs, the sabotage negative control, the odd-row sentinel test with an unsupported token
count (run_check_odd_rows, :410-473), plus BASELINE's shapes at full size. Tolerances: fp32 output 1e-4 of
sum|x*w| (exact codes, fp32 sums); fp16 output 1e-3 (the fp16 rounding of y alone is up to 2^-11 of |y|) and
BASELINE's |y - ref| <= 1e-2 + 1e-3 |ref|."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

from gpu_util import baseline_weights, device_weights, normal_x, random_codes, run_gemv, score, uniform_x

pytestmark = pytest.mark.gpu

FMTS = [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2]
NAME = {O.FMT_Q4: "q4", O.FMT_Q8: "q8", O.FMT_Q2: "q2"}


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("table", ["a", "odd"])
def test_golden_vectors(cuda, golden, fmt, table):
    p = f"{table}_{NAME[fmt]}_"
    codes, scales = golden[p + "codes"], golden[p + "scales"]
    q, s = device_weights(fmt, codes, scales)
    ncase = 1 if fmt == O.FMT_Q2 else 5
    for ci in range(ncase):
        x = golden[p + f"x{ci}"]
        ref, mag = golden[p + f"val{ci}"], golden[p + f"mag{ci}"]
        y32 = run_gemv(fmt, q, s, x, out_f32=True)
        err, m, n = O.check_error(y32, ref, mag)
        assert err <= O.TOL_EXACT, (p, ci, err, m, n)
        y16 = run_gemv(fmt, q, s, x, out_f32=False)
        fin = np.abs(ref) < 60000.0            # +bigx can overflow fp16 in the output itself
        err16 = np.max(np.abs(y16 - ref)[fin] / (mag[fin] + 1e-12))
        assert err16 <= 1e-3, (p, ci, err16)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
def test_random_tokens(cuda, fmt, M):
    rng = np.random.default_rng(100 + 10 * fmt + M)
    N, K = 200, 1024
    codes, scales = random_codes(rng, fmt, N, K)
    q, s = device_weights(fmt, codes, scales)
    x = uniform_x(rng, M, K)
    (err, m, n), _ = score(run_gemv(fmt, q, s, x, True), codes, scales, x)
    assert err <= O.TOL_EXACT, (err, m, n)


BASELINE_SHAPES = [(8192, 2048), (12288, 2560), (2560, 6144), (6144, 2048), (2048, 6144)]


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("shape", BASELINE_SHAPES)
def test_baseline_shapes_full_size(cuda, fmt, shape):
    """BASELINE configs 0 and 1: N(0,0.02) weights seed 0, quantised; x N(0,1); 1/2/4/8 tokens; fp16 output."""
    N, K = shape
    codes, scales = baseline_weights(fmt, N, K)
    q, s = device_weights(fmt, codes, scales)
    ref_w = O._weights_f64(codes, scales)
    for M in (1, 2, 4, 8):
        x = normal_x(M, K, seed=1 + M)
        xd = x.view(np.float16).astype(np.float64)
        ref, mag = xd @ ref_w.T, np.abs(xd) @ np.abs(ref_w).T
        y16 = run_gemv(fmt, q, s, x, out_f32=False)
        err, m, n = O.check_error(y16, ref, mag)
        assert err <= 1e-3, (shape, M, err, m, n)
        assert O.allclose_f16out(y16, ref), (shape, M)
        if M == 1:
            y32 = run_gemv(fmt, q, s, x, out_f32=True)
            assert O.check_error(y32, ref, mag)[0] <= O.TOL_EXACT


@pytest.mark.parametrize("fmt", FMTS)
def test_sabotage_fails(cuda, golden, fmt):
    """BAKEOFF_SABOTAGE: broken packing must fail the check (src/bakeoff.cu:20-23, :845)."""
    p = f"a_{NAME[fmt]}_"
    codes, scales = golden[p + "codes"], golden[p + "scales"]
    q, s = device_weights(fmt, codes, scales, sabotage=True)
    x = golden[p + "x0"]
    err, _, _ = O.check_error(run_gemv(fmt, q, s, x, True), golden[p + "val0"], golden[p + "mag0"])
    assert err > 1e-2, err


@pytest.mark.parametrize("fmt", FMTS)
def test_odd_rows_sentinels_and_unsupported_m(cuda, fmt):
    """N = 1031 (odd, not a multiple of 16): every output checked, nothing written outside M x N (sentinel pads);
    then unsupported token counts launch nothing (src/bakeoff.cu:410-473)."""
    import torch
    rng = np.random.default_rng(7 + fmt)
    N, K, PAD = 1031, 2048, 1024
    codes, scales = random_codes(rng, fmt, N, K)
    q, s = device_weights(fmt, codes, scales)
    SENT = -12345.0
    for M in (1, 2, 4, 8):
        x = uniform_x(rng, M, K)
        buf = torch.full((M * N + 2 * PAD,), SENT, dtype=torch.float32, device="cuda")
        y = buf[PAD:PAD + M * N].view(M, N)
        vkb.gemv(fmt, q, s, vkb.to_device_f16(x), y=y, out_f32=True)
        torch.cuda.synchronize()
        out = buf.cpu().numpy()
        assert np.all(out[:PAD] == SENT) and np.all(out[PAD + M * N:] == SENT)
        (err, m, n), _ = score(out[PAD:PAD + M * N].reshape(M, N), codes, scales, x)
        assert err <= O.TOL_EXACT, (M, err, m, n)
    x = vkb.to_device_f16(uniform_x(rng, 9, K))
    y = torch.full((9, N), SENT, dtype=torch.float32, device="cuda")
    L = vkb.lib()
    for M in (9, 0, -1):
        rc = L.vkb_gemv(fmt, vkb._ptr(q), vkb._ptr(s), vkb._ptr(x), vkb._ptr(y), 1, N, K, M, vkb._stream())
        assert rc > 0, rc
    torch.cuda.synchronize()
    assert torch.all(y == SENT)


@pytest.mark.parametrize("fmt", FMTS)
def test_general_path_shapes(cuda, fmt):
    """K % 256 != 0 (the reference's 2560x640 expert-down table) and an unaligned activation pointer take the
    general kernel; same results."""
    import torch
    rng = np.random.default_rng(31 + fmt)
    for N, K in ((2560, 640), (100, 64 * 5)):
        codes, scales = random_codes(rng, fmt, N, K)
        q, s = device_weights(fmt, codes, scales)
        x = uniform_x(rng, 3, K)
        (err, m, n), _ = score(run_gemv(fmt, q, s, x, True), codes, scales, x)
        assert err <= O.TOL_EXACT, (N, K, err)
    # unaligned x (offset by one fp16 element) on a fast-path shape
    N, K = 96, 512
    codes, scales = random_codes(rng, fmt, N, K)
    q, s = device_weights(fmt, codes, scales)
    x = uniform_x(rng, 2, K)
    xbuf = torch.zeros(2 * K + 8, dtype=torch.float16, device="cuda")
    xbuf[1:1 + 2 * K] = vkb.to_device_f16(x).reshape(-1)
    xv = xbuf[1:1 + 2 * K].view(2, K)
    y = vkb.gemv(fmt, q, s, xv, out_f32=True)
    torch.cuda.synchronize()
    (err, _, _), _ = score(y.cpu().numpy().astype(np.float64), codes, scales, x)
    assert err <= O.TOL_EXACT


def test_pdl_chain_orders_activations_and_outputs(cuda):
    """Back-to-back calls under programmatic dependent launch: call i+1 reads call i's output as its activations
    (N == K), and many calls overwrite one output buffer; the results must be those of strictly ordered calls."""
    import torch
    rng = np.random.default_rng(5)
    K = 1024
    codes, scales = random_codes(rng, O.FMT_Q4, K, K)
    scales = (scales.view(np.float16).astype(np.float32) * 0.05).astype(np.float16).view(np.uint16)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x0 = uniform_x(rng, 1, K)
    xs = [vkb.to_device_f16(x0)]
    for _ in range(6):
        xs.append(vkb.gemv(O.FMT_Q4, q, s, xs[-1]))
    torch.cuda.synchronize()
    ref = x0.view(np.float16).astype(np.float64)
    W = O._weights_f64(codes, scales)
    for i in range(1, 7):
        ref = (ref @ W.T).astype(np.float16).astype(np.float64)   # each hop rounds to fp16 like the kernel output
        got = xs[i].float().cpu().numpy()
        assert np.allclose(got, ref, rtol=2e-2, atol=2e-2 * np.abs(ref).max()), i
    # WAW: 20 calls alternate between two inputs into the same y; the last one wins
    xa, xb = vkb.to_device_f16(uniform_x(rng, 1, K)), vkb.to_device_f16(uniform_x(rng, 1, K))
    y = torch.empty((1, K), dtype=torch.float32, device="cuda")
    for i in range(20):
        vkb.gemv(O.FMT_Q4, q, s, xa if i % 2 == 0 else xb, y=y, out_f32=True)
    torch.cuda.synchronize()
    want = vkb.gemv(O.FMT_Q4, q, s, xb, out_f32=True)
    torch.cuda.synchronize()
    assert torch.equal(y, want)


def test_pdl_off_gives_identical_results(cuda):
    import torch
    rng = np.random.default_rng(9)
    codes, scales = random_codes(rng, O.FMT_Q8, 512, 2048)
    q, s = device_weights(O.FMT_Q8, codes, scales)
    x = vkb.to_device_f16(uniform_x(rng, 4, 2048))
    a = vkb.gemv(O.FMT_Q8, q, s, x, out_f32=True)
    old = vkb.set_pdl(False)
    b = vkb.gemv(O.FMT_Q8, q, s, x, out_f32=True)
    vkb.set_pdl(old)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert vkb.device_status() == 0
