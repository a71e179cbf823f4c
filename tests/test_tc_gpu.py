"""GPU parity of the tcgen05 prompt GEMM (vkb_gemm_q4_tc) through the C ABI.

Two references: a plain PyTorch fp32 matmul over the same fp16-rounded weights ((code - 8) * scale, one rounding, as
the reference's tc_q4 unpack rounds them, src/stage4_tc.cuh:25-36) -- tight, isolates the tensor-core tile machinery
(descriptors, swizzles, TMEM) -- and the CPU oracle of the exact codes with the reference's tc tolerance (2e-3,
src/bakeoff.cu:575-579) plus BASELINE's fp16-output bound. Shapes: BASELINE's prompt tables at 64 and 512 tokens, and
ragged token counts / rows (1-512 tokens, N not a multiple of 128)."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

from gpu_util import baseline_weights, device_weights, normal_x, random_codes, uniform_x

pytestmark = pytest.mark.gpu


def _tc(q, s, x_bits, M, out_f32):
    import torch
    L = vkb.lib()
    N = s.shape[0]
    K = x_bits.shape[1]
    x = vkb.to_device_f16(x_bits)
    y = torch.empty((M, N), dtype=torch.float32 if out_f32 else torch.float16, device="cuda")
    fn = L.vkb_gemm_q4_tc_f32 if out_f32 else L.vkb_gemm_q4_tc
    rc = fn(vkb._ptr(q), vkb._ptr(s), vkb._ptr(x), vkb._ptr(y), N, K, M, vkb._stream())
    assert rc == 0, vkb.strerror(rc)
    torch.cuda.synchronize()
    return y


def _torch_ref(codes, scales, x_bits):
    """fp32 matmul over the fp16-rounded dequantised weights (what the kernel feeds the tensor cores)."""
    import torch
    w16 = (codes.astype(np.float32) * np.repeat(scales.view(np.float16).astype(np.float32), 32, axis=1))
    w16 = torch.from_numpy(w16.astype(np.float16)).cuda().float()
    x = torch.from_numpy(x_bits.view(np.float16).astype(np.float32)).cuda()
    return x @ w16.T


# (1031, 768, 200): ragged last row tile and a token tile that overruns M
@pytest.mark.parametrize("N,K,M", [(512, 256, 16), (256, 512, 64), (384, 1024, 128), (1031, 768, 65),
                                   (1024, 2048, 1), (640, 2560, 130), (2048, 2048, 511), (1031, 768, 200)])
def test_tc_vs_torch_fp32(cuda, N, K, M):
    rng = np.random.default_rng(N + K + M)
    codes, scales = random_codes(rng, O.FMT_Q4, N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x = uniform_x(rng, M, K)
    y = _tc(q, s, x, M, out_f32=True)
    ref = _torch_ref(codes, scales, x)
    err = ((y - ref).abs().max() / (ref.abs().max() + 1e-12)).item()
    assert err < 1e-5, err


@pytest.mark.parametrize("shape", [(12288, 2560), (8192, 2048)])
@pytest.mark.parametrize("M", [64, 512])
def test_tc_baseline_prompt(cuda, shape, M):
    """N(0,0.02) weights seed 0 quantised Q4_0, x fp16 N(0,1), 64 and 512 tokens, fp16 out."""
    N, K = shape
    codes, scales = baseline_weights(O.FMT_Q4, N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x = normal_x(M, K, seed=3)
    y = _tc(q, s, x, M, out_f32=False).float().cpu().numpy().astype(np.float64)
    ref, mag = O.ref_value(codes, scales, x), O.ref_scale(codes, scales, x)
    err, m, n = O.check_error(y, ref, mag)
    assert err <= O.TOL_FP16, (err, m, n)
    assert O.allclose_f16out(y, ref)


def test_tc_golden_and_sabotage(cuda, golden):
    codes, scales, x = golden["a_q4_codes"], golden["a_q4_scales"], golden["a_q4_x2"]   # 64 x 256, 8 tokens
    q, s = device_weights(O.FMT_Q4, codes, scales)
    y = _tc(q, s, x, 8, out_f32=True).cpu().numpy().astype(np.float64)
    err, _, _ = O.check_error(y, golden["a_q4_val2"], golden["a_q4_mag2"])
    assert err <= O.TOL_FP16, err
    qb, sb = device_weights(O.FMT_Q4, codes, scales, sabotage=True)
    yb = _tc(qb, sb, x, 8, out_f32=True).cpu().numpy().astype(np.float64)
    assert O.check_error(yb, golden["a_q4_val2"], golden["a_q4_mag2"])[0] > 1e-2


def test_tc_rejects_unsupported(cuda):
    import torch
    L = vkb.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = vkb._ptr(buf)
    assert L.vkb_gemm_q4_tc(p, p, p, p, 128, 320, 64, vkb._stream()) == vkb.EUNSUPPORTED   # K % 256 != 0
    assert L.vkb_gemm_q4_tc(p, p, p, p, 128, 256, 0, vkb._stream()) == vkb.EINVAL


_VARIANT_SCRIPT = r"""
import sys
import numpy as np
sys.path[:0] = sys.argv[1:4]
import vkb
from oracle import oracle as O
from gpu_util import device_weights, random_codes, uniform_x
from test_tc_gpu import _tc, _torch_ref
worst = 0.0
for N, K, M in [(384, 1024, 128), (1031, 768, 200), (2048, 2048, 511), (512, 256, 16), (12288, 2560, 512),
                (640, 2560, 130)]:
    rng = np.random.default_rng(N + K + M)
    codes, scales = random_codes(rng, O.FMT_Q4, N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x = uniform_x(rng, M, K)
    y = _tc(q, s, x, M, out_f32=True)
    ref = _torch_ref(codes, scales, x)
    worst = max(worst, ((y - ref).abs().max() / (ref.abs().max() + 1e-12)).item())
print("WORST", worst, "STATUS", vkb.device_status())
"""


@pytest.mark.parametrize("env", [{"VKB_TC_CG": "2"}, {"VKB_TC_RB": "2"}, {"VKB_TC_RB": "2", "VKB_TC_NT": "176"},
                                 {"VKB_TC_RB": "2", "VKB_TC_NT": "48"}, {"VKB_TC_RB": "1", "VKB_TC_NT": "176"},
                                 {"VKB_TC_RB": "1", "VKB_TC_NT": "80"}, {"VKB_TC_SPLIT": "2"},
                                 {"VKB_TC_SPLIT": "3", "VKB_TC_NT": "80"}, {"VKB_TC_SPLIT": "1"}],
                         ids=["pair", "rb2", "rb2_nt176", "rb2_nt48", "rb1_nt176", "rb1_nt80", "split2",
                              "split3_nt80", "nosplit"])
def test_tc_kernel_variants(cuda, env):
    """Every prompt-kernel variant the planner can pick, forced by its tuning overrides (read once per process, so in
    a child process) against torch fp32: the CTA pair (tcgen05 cta_group::2), two 128-row blocks per CTA, token
    tiles that are multiples of 16 but not of 32 (one accumulator, two blocks, or two accumulators), and split-K over
    2 or 3 CTAs (even and uneven shares of the K units; 640x2560 has 5 units) or none. A forced value that does not
    fit a shape leaves that shape to the planner."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = [root, os.path.join(root, "volta-kernel-bakeoff_b200"), os.path.join(root, "tests")]
    r = subprocess.run([sys.executable, "-c", _VARIANT_SCRIPT] + paths, env=dict(os.environ, **env),
                       capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("WORST")][-1].split()
    assert float(line[1]) < 1e-5 and int(line[3]) == 0, line


@pytest.mark.parametrize("N,K,M", [(2560, 6144, 64), (2560, 6144, 512), (2048, 6144, 64), (2048, 6144, 512),
                                   (1000, 6144, 77)])
def test_tc_split_k_small_tables(cuda, N, K, M):
    """The survey's small-N / large-K prompt tables (and a ragged one), which the planner runs as split-K clusters
    (each tile's K range shared by several CTAs, partials summed in rank order over distributed shared memory):
    against torch fp32 over the same fp16 weights (tight), the oracle with the reference's tc tolerance and fp16-output
    bound, and two calls bit-identical (the reduction order is fixed)."""
    import torch
    p = vkb.plan(vkb.PLAN_TC_SPLIT, O.FMT_Q4, N, K, M)
    assert p["splits"] > 1 and p["grid"] == p["tiles"] * p["splits"] <= vkb.B200_LIMITS["sm_count"], p
    rng = np.random.default_rng(N + M)
    codes, scales = random_codes(rng, O.FMT_Q4, N, K)
    q, s = device_weights(O.FMT_Q4, codes, scales)
    x = uniform_x(rng, M, K)
    y = _tc(q, s, x, M, out_f32=True)
    ref = _torch_ref(codes, scales, x)
    err = ((y - ref).abs().max() / (ref.abs().max() + 1e-12)).item()
    assert err < 1e-5, err
    y2 = _tc(q, s, x, M, out_f32=True)
    assert torch.equal(y, y2)
    yh = _tc(q, s, x, M, out_f32=False).float().cpu().numpy().astype(np.float64)
    ref64, mag = O.ref_value(codes, scales, x), O.ref_scale(codes, scales, x)
    e, m, n = O.check_error(yh, ref64, mag)
    assert e <= O.TOL_FP16, (e, m, n)
    assert vkb.device_status() == 0


@pytest.mark.parametrize("N,K,M", [(512, 256, 16), (1031, 768, 65), (2048, 2048, 511), (12288, 2560, 512),
                                   (8192, 2048, 64), (2560, 6144, 512), (2048, 6144, 64)])   # (the last two: split-K)
def test_tc_q8_vs_torch_fp32_and_oracle(cuda, N, K, M):
    """The Q8 prompt GEMM (vkb_gemm_tc with Q8 weights): against torch fp32 over the fp16-rounded weights (tight) and
    the CPU oracle of the exact codes with the fp16-class tolerance."""
    import torch
    rng = np.random.default_rng(3 * N + K + M)
    codes, scales = random_codes(rng, O.FMT_Q8, N, K)
    q, s = device_weights(O.FMT_Q8, codes, scales)
    x = uniform_x(rng, M, K)
    y = vkb.gemm_tc(q, s, vkb.to_device_f16(x), out_f32=True, fmt=O.FMT_Q8)
    yh = vkb.gemm_tc(q, s, vkb.to_device_f16(x), out_f32=False, fmt=O.FMT_Q8)
    torch.cuda.synchronize()
    ref = _torch_ref(codes, scales, x)
    assert ((y - ref).abs().max() / (ref.abs().max() + 1e-12)).item() < 1e-5
    if N * K <= 2048 * 2048:
        yo = y.cpu().numpy().astype(np.float64)
        err = O.check_error(yo, O.ref_value(codes, scales, x), O.ref_scale(codes, scales, x))[0]
        assert err <= O.TOL_FP16, err
    assert torch.equal(yh, y.half())
    assert vkb.device_status() == 0
