"""The bakeoff harness's parity contract, run as the reference's runner runs it before every sweep
(bench/overnight.sh:37-38): `bakeoff --check` must pass, and `BAKEOFF_SABOTAGE=1 bakeoff --check` must fail.

  --check              every row ok, exit 0 (the reference: src/bakeoff.cu:475-649, exit code :839-852). The rows cover
                       the decode GEMV (Q4/Q8/2-bit, fp32 and fp16 output, 1/2/4/8 tokens, +bigx, +tinyx), the prompt
                       GEMM on tcgen05 (Q4 and Q8 weights, 1-512 tokens and 65), the fp32-in decode, gate + up +
                       SwiGLU, the one-launch MoE (1/8/64 tokens), the odd-rows sentinel case (N = 1031, 1-100
                       tokens) and the refused token count, on every table of the reference (src/bakeoff.cu:300-311);
  sabotage             the packing is broken (Q4 nibbles, Q8 and 2-bit code pairs swapped; src/bakeoff.cu:20-23): every
                       packed-weight row FAILs, exit 1; the cuBLAS controls (unpacked weights) and the refused-call
                       checks (nothing launched) stay ok.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BAKEOFF = os.path.join(ROOT, "volta-kernel-bakeoff_b200", "bin", "bakeoff")
PACKED = {"vkb_q4", "vkb_q8", "vkb_q2", "vkb_q4_f16out", "vkb_q8_f16out", "vkb_q2_f16out", "vkb_tc_q4",
          "vkb_tc_q4_f16out", "vkb_tc_q8", "vkb_q4_f32in", "vkb_glu_q4_f32in", "vkb_moe_q4", "dq4+cublas"}


def _run(sabotage: bool):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(BAKEOFF):
        pytest.fail(f"{BAKEOFF} is not built")
    env = dict(os.environ, BAKEOFF_SABOTAGE="1" if sabotage else "0")
    r = subprocess.run([BAKEOFF, "--check"], capture_output=True, text=True, timeout=900, env=env)
    rows = []
    for line in r.stdout.splitlines():
        f = line.split(",")
        if len(f) == 8 and f[0] == "check" and f[1] != "contender":
            rows.append({"who": f[1], "shape": f[2], "M": int(f[3]), "err": f[4], "verdict": f[7]})
    return r, rows


def test_check_passes():
    r, rows = _run(False)
    bad = [x for x in rows if x["verdict"] != "ok"]
    assert r.returncode == 0 and not bad, (r.returncode, bad[:10], r.stderr[-2000:])
    who = {x["who"] for x in rows}
    assert PACKED | {"cublas_fp16"} <= who, sorted(who)
    ms = {x["M"] for x in rows if x["who"].startswith("vkb_tc")}
    assert {1, 2, 4, 8, 64, 65, 128, 256, 512} <= ms, sorted(ms)
    assert any(x["shape"] == "odd_rows_1031x2048" for x in rows)
    assert len(rows) > 900, len(rows)


def test_sabotage_fails_every_packed_kernel():
    r, rows = _run(True)
    assert r.returncode == 1, (r.returncode, r.stderr[-2000:])
    controls = [x for x in rows if x["who"].startswith("cublas") or x["who"].endswith("_unsupported_M")]
    packed = [x for x in rows if x not in controls]
    assert controls and all(x["verdict"] == "ok" for x in controls), [x for x in controls if x["verdict"] != "ok"]
    survivors = [x for x in packed if x["verdict"] != "FAIL"]
    assert not survivors, survivors[:10]
    assert PACKED <= {x["who"] for x in packed}, sorted({x["who"] for x in packed})
