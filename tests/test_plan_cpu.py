"""CPU tests of the launch planners (vkb_plan_describe: host only, no device): every plan the library would launch on a
B200 keeps the resource limits the kernels rely on, over the reference's tables and ragged shapes.

- decode GEMV / gate + up (csrc/qmv.cuh): shared memory within the opt-in limit, at least two ring stages, stages that
  cover K in 256-value units, conflict-free pitches, warp groups the ring can feed, and the two-CTA footprint only with
  at least 4 stages;
- prompt GEMM (csrc/tc_gemm.cuh): shared memory within the limit, TMEM accumulators and A ring inside the 512-column
  allocation, token tiles that are UMMA N values, X stages of at most 32 KB in an even count (two producers), chunk
  and stage sizes that divide the K steps, and a grid of at most one CTA per SM."""
import itertools

import pytest

import vkb
from oracle import oracle as O

LIM = vkb.B200_LIMITS
TABLES = [(12288, 2560), (2560, 6144), (6144, 2048), (2048, 6144), (8192, 2048), (512, 2048), (2048, 512),
          (640, 2560), (2560, 640)]
RAGGED = [(1031, 768), (16, 256), (33, 1024), (4096, 14336), (151936, 2048)]


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2])
def test_decode_plans_fit(fmt):
    n = 0
    for (N, K), M in itertools.product(TABLES + RAGGED, range(1, 9)):
        p = vkb.plan(vkb.PLAN_GEMV, fmt, N, K, M)
        if K % 256 != 0:
            assert p is None
            continue
        if p is None:   # only when the activation buffer leaves no room for two stages (general-shape kernel)
            assert M * 2 * K > 128 * 1024, (N, K, M)
            continue
        n += 1
        bits = {O.FMT_Q4: 4, O.FMT_Q8: 8, O.FMT_Q2: 2}[fmt]
        assert p["smem"] <= LIM["smem_optin"], (N, K, M, p)
        assert p["nstage"] >= 2
        assert p["KS"] % 256 == 0 and p["KS"] * p["nchunks"] >= K and p["KS"] * (p["nchunks"] - 1) < K
        assert p["KS"] * bits // 8 <= 2048                      # one TMA box row of 8-byte elements
        # conflict-free fragment reads: code rows an odd number of 16-byte units apart (Q8: of 32-byte units)
        unit = 32 if fmt == O.FMT_Q8 else 16
        assert p["cpitch"] % unit == 0 and (p["cpitch"] // unit) % 2 == 1, (N, K, M, p)
        assert p["spitch"] % 16 == 0 and (p["spitch"] // 16) % 2 == 1, (N, K, M, p)
        assert p["wg"] in (1, 2, 4) and (p["wg"] == 1 or p["nstage"] >= p["wg"] * p["nchunks"])
        assert p["tiles"] == (N + 15) // 16 and p["grid"] == min(p["tiles"], LIM["sm_count"])
        two_per_sm = 2 * p["smem"] <= LIM["smem_per_sm"]
        assert not two_per_sm or p["nstage"] >= 4 or p["nstage"] == 16, (N, K, M, p)
        # the two-CTA footprint (the 56-register kernel instances) only for K <= 2048 covered by one stage; the host
        # launches the one-CTA instances when two CTAs (plus the runtime's 1 KB each) do not fit an SM
        if 2 * (p["smem"] + 1024) <= LIM["smem_per_sm"]:
            assert p["nchunks"] == 1 and K <= 2048, (N, K, M, p)
    assert n > 100


def test_gate_up_plans_fit():
    for (N, K), M in itertools.product([(6144, 2048), (2048, 6144), (1031, 768), (8192, 2048)], range(1, 9)):
        p = vkb.plan(vkb.PLAN_GLU, O.FMT_Q4, N, K, M)
        assert p is not None and p["smem"] <= LIM["smem_optin"]
        assert p["tiles"] == 2 * ((N + 15) // 16)                # gate / up tile pairs
        assert p["wg"] in (1, 2, 4) and (p["wg"] == 1 or p["nstage"] >= p["wg"] * p["nchunks"])


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8])
def test_prompt_plans_fit(fmt):
    n = 0
    for (N, K), M in itertools.product(TABLES + RAGGED, [1, 7, 16, 33, 64, 100, 128, 200, 256, 384, 511, 512, 1000]):
        p = vkb.plan(vkb.PLAN_TC, fmt, N, K, M)
        if K % 256 != 0:
            assert p is None
            continue
        assert p is not None, (N, K, M)
        n += 1
        assert p["smem"] <= LIM["smem_optin"], (N, K, M, p)
        assert p["cg"] == 1 and p["rb"] == 1                    # the defaults: one CTA, one 128-row block per tile
        NT = p["NT"]
        assert 32 <= NT <= 256 and NT % 16 == 0 and (NT > 128 or NT % 32 == 0), (N, K, M, p)
        assert NT <= max(32, -(-M // 32) * 32)                  # no wider than the tokens need
        # TMEM: accumulators at columns 0 (and 128), A ring of na 128-column slots from a_col0, all inside 512
        assert p["tmem_cols"] == 512
        assert p["nacc"] in (1, 2) and (p["nacc"] == 1 or NT <= 128)
        assert (p["nacc"] - 1) * 128 + NT <= p["a_col0"] and p["a_col0"] + p["na"] * 128 <= 512
        nk = K // 64
        assert nk % p["pk"] == 0 and nk % p["xk"] == 0 and p["pk"] in (4, 8)
        assert p["x_stage"] == p["xk"] * NT * 128 and p["x_stage"] <= 32768
        assert p["nx"] >= 2 and p["nx"] % 2 == 0 and p["np"] >= 2
        assert p["tiles_n"] == -(-N // 128) and p["tiles"] == p["tiles_n"] * -(-M // NT)
        assert p["grid"] == min(p["tiles"], LIM["sm_count"])
    assert n > 100


def test_split_k_plans():
    """Kind 3, the prompt planner with split-K: the small-N / large-K tables (20 and 16 row tiles; Q4 and Q8) take
    clusters of 2-8 CTAs per tile, one tile per cluster, all within the SM count, K units (8 K steps) to spare for
    every CTA, and the fp32 partial (128 rows x NT) inside the shared memory the rings used; large tables keep the
    one-CTA plan."""
    for (N, K), M, fmt in itertools.product([(2560, 6144), (2048, 6144)], [16, 64, 128, 512], [O.FMT_Q4, O.FMT_Q8]):
        p = vkb.plan(vkb.PLAN_TC_SPLIT, fmt, N, K, M)
        assert 2 <= p["splits"] <= 8 and p["splits"] <= K // 64 // 8, (N, K, M, p)
        assert p["grid"] == p["tiles"] * p["splits"] <= LIM["sm_count"], (N, K, M, p)
        assert 128 * p["NT"] * 4 <= p["nx"] * p["x_stage"] + p["np"] * 128 * (32 * p["pk"] + 16 + 48), p
    for (N, K), M in itertools.product([(12288, 2560), (8192, 2048), (6144, 2048)], [64, 128, 512]):
        p, q = vkb.plan(vkb.PLAN_TC_SPLIT, O.FMT_Q4, N, K, M), vkb.plan(vkb.PLAN_TC, O.FMT_Q4, N, K, M)
        assert p["splits"] == 1 and {k: v for k, v in p.items() if k != "splits"} == \
            {k: v for k, v in q.items() if k != "cg"}, (N, K, M, p, q)
    # Q8 weights split too; K without whole 8-step units stays unsplit
    assert vkb.plan(vkb.PLAN_TC_SPLIT, O.FMT_Q8, 2560, 6144, 512)["splits"] > 1
    assert vkb.plan(vkb.PLAN_TC_SPLIT, O.FMT_Q4, 2560, 768, 64)["splits"] == 1


def test_prompt_plans_for_baseline_shapes():
    """the tile shapes the measurements in the profiles were taken with."""
    p = vkb.plan(vkb.PLAN_TC, O.FMT_Q4, 12288, 2560, 512)
    assert (p["NT"], p["tiles"], p["nacc"], p["grid"]) == (176, 288, 1, 148)
    p = vkb.plan(vkb.PLAN_TC, O.FMT_Q4, 8192, 2048, 512)
    assert (p["NT"], p["tiles"], p["grid"]) == (256, 128, 128)


def test_plan_rejects_bad_arguments():
    import ctypes
    info = (ctypes.c_int * 16)()
    L = vkb.lib()
    ptr = ctypes.cast(info, ctypes.c_void_p)
    assert L.vkb_plan_describe(0, 0, 0, 2048, 1, 148, 232448, 233472, ptr) == vkb.EINVAL
    assert L.vkb_plan_describe(7, 0, 64, 2048, 1, 148, 232448, 233472, ptr) == vkb.EINVAL
    assert L.vkb_plan_describe(2, 1, 64, 2048, 1, 148, 232448, 233472, ptr) == vkb.EINVAL      # gate/up: Q4 only
    assert L.vkb_plan_describe(1, 2, 64, 2048, 1, 148, 232448, 233472, ptr) == vkb.EINVAL      # prompt: Q4 / Q8
    assert L.vkb_plan_describe(0, 0, 64, 2048, 9, 148, 232448, 233472, ptr) == vkb.EUNSUPPORTED
    assert L.vkb_plan_describe(0, 0, 64, 2048, 1, 148, 232448, 233472, None) == vkb.EINVAL


_RB2_SCRIPT = r"""
import itertools, sys
sys.path[:0] = sys.argv[1:3]
import vkb
bad = []
for (N, K), M in itertools.product([(12288, 2560), (8192, 2048), (1031, 768), (2048, 6144)], [16, 64, 200, 512]):
    p = vkb.plan(vkb.PLAN_TC, 0, N, K, M)
    NT, r32 = p["NT"], -(-p["NT"] // 32) * 32
    ok = (p["rb"] == 2 and p["nacc"] == 1 and p["pk"] == 4 and p["a_col0"] >= r32 + NT and p["a_col0"] % 64 == 0
          and 2 <= p["na"] <= 4 and p["a_col0"] + 64 * p["na"] <= 512 and p["tiles_n"] == -(-N // 256)
          and p["smem"] <= 232448)
    if not ok:
        bad.append((N, K, M, p))
print("BAD", bad)
"""


def test_two_block_plans_fit():
    """VKB_TC_RB=2 (two 128-row blocks per CTA): both accumulators (columns 0 and NT rounded up to 32) and at least two
    64-column A slots inside the 512 TMEM columns, 256-row tiles, 4-step chunks."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = [root, os.path.join(root, "volta-kernel-bakeoff_b200")]
    r = subprocess.run([sys.executable, "-c", _RB2_SCRIPT] + paths, env=dict(os.environ, VKB_TC_RB="2"),
                       capture_output=True, text=True, timeout=120, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().splitlines()[-1] == "BAD []", r.stdout[-2000:]
