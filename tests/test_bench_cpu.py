"""bench.py's reference arm on the host CPU (no GPU needed): the driver's JSON contract, the same `config` as the GPU
arm, inputs built without libvkb.so, and the torchrun rule that ranks other than 0 exit 0 without work."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Runs bench.py as __main__ in this process and reports afterwards whether libvkb.so was ever mapped into it.
_RUN = """
import runpy, sys
sys.argv = ["bench.py"] + sys.argv[1:]
try:
    runpy.run_path("bench.py", run_name="__main__")
finally:
    maps = open("/proc/self/maps").read()
    print("LIBVKB_MAPPED" if "libvkb.so" in maps else "LIBVKB_NOT_MAPPED", flush=True)
"""

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(env_extra, *args, timeout=600):
    env = dict(os.environ, **env_extra)
    env.pop("CUDA_VISIBLE_DEVICES", None)
    return subprocess.run([sys.executable, "-c", _RUN, *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_line():
    if not os.path.exists("/proc/self/maps"):
        pytest.skip("needs /proc/self/maps")
    r = _run({}, "--impl", "reference", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    assert lines[-1] == "LIBVKB_NOT_MAPPED", "the reference arm loaded the library it is compared against"
    rows = [json.loads(ln) for ln in lines if ln.startswith("{")]
    assert len(rows) == 1
    res = rows[0]
    assert KEYS <= set(res), KEYS - set(res)
    assert res["impl"] == "reference" and res["unit"] == "GB/s" and res["higher_is_better"] is True
    assert res["steps"] == 1 and res["n_gpus"] == 1 and res["value"] > 0
    import bench
    assert res["config"] == json.loads(json.dumps(bench.bench_config())), "config differs from the GPU arm's"
    assert res["metric"] == bench.METRIC
    cb = res["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == res["value"] and cb["sample"]
    assert res["e2e"] == {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the timed work fits the wall clock that ran it: ms_per_step x steps is the CPU time of the outputs reported
    assert res["ms_per_step"] * res["steps"] / 1e3 < 600


def test_reference_arm_other_ranks_exit_without_work():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--impl", "reference", "--steps", "1",
             "--warmup", "0", timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
