"""The B200 load judge (vkb.load_judge), the counterpart of the reference's bench/load_flag.py, on hand-written
nvidia-smi sample files (tests/fixtures_load/): which timed regions are rejected, which are kept with a note, and
the CLI contract (one line, exit 0; wrong arguments exit 2)."""
import os
import subprocess
import sys

import pytest

from vkb import load_judge as J

FX = os.path.join(os.path.dirname(__file__), "fixtures_load")


def _judge(name):
    with open(os.path.join(FX, name)) as f:
        return J.judge(f.read())


def test_good_and_partial_tail():
    v = _judge("good.csv")
    assert not v.flagged and v.busy == 8 and v.min_clock == 1965 and v.max_clock == 1965 and v.max_temp == 46
    line = J.format_line("r1", v)
    assert line.startswith("round r1 under load: 8 busy samples") and "FLAGGED" not in line
    v = _judge("partial_tail.csv")   # the cut-off last line is dropped, not counted as malformed
    assert not v.flagged and v.busy == 4


def test_power_cap_is_noted_not_flagged():
    v = _judge("power_cap.csv")
    assert not v.flagged and v.power_cap == 6 and v.low == 0
    assert "sw_power_cap" in v.reason_names()
    assert "6 on the sw power cap" in J.format_line("r", v)


@pytest.mark.parametrize("name,check", [
    ("hw_slowdown.csv", lambda v: v.rejected == 1 and v.reasons == J.HW_SLOWDOWN),
    ("thermal.csv", lambda v: v.rejected == 1 and v.reasons == J.SW_THERMAL and v.max_temp == 88),
    ("clock_stuck.csv", lambda v: v.low == 6 and v.rejected == 0),
    ("idle_only.csv", lambda v: v.busy == 0 and "no usable busy samples" in v.notes),
    ("ecc_rise.csv", lambda v: "ecc uncorrected 0->2" in v.notes),
    ("ecc_na.csv", lambda v: "ecc uncorrected unreadable" in v.notes),
    ("util_na.csv", lambda v: any("unreadable utilization" in n for n in v.notes) and v.low == 1),
    ("malformed.csv", lambda v: "1 malformed sample" in v.notes),
])
def test_rejected_regions(name, check):
    v = _judge(name)
    assert v.flagged and check(v), (name, v)
    assert J.format_line("r", v).endswith("** FLAGGED **")


def test_cli():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=os.path.join(root, "volta-kernel-bakeoff_b200"))
    r = subprocess.run([sys.executable, "-m", "vkb.load_judge", "7", os.path.join(FX, "hw_slowdown.csv")],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0 and r.stdout.startswith("round 7 under load:") and "FLAGGED" in r.stdout
    r = subprocess.run([sys.executable, "-m", "vkb.load_judge", "7", os.path.join(FX, "missing.csv")],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0 and "could not read samples" in r.stdout and "FLAGGED" in r.stdout
    r = subprocess.run([sys.executable, "-m", "vkb.load_judge", "7"], capture_output=True, text=True, env=env)
    assert r.returncode == 2


def test_nvml_rows_inside_the_timed_region():
    """bench.py's NVML sampler polls only while the timed work runs: a zero utilization reading (NVML's counter
    averages over a longer window) still counts as busy with assume_busy, and a slowdown reason still rejects."""
    ok = "0,1965,1965,612.0,0x0000000000000000,-,-,-,-,0,41,0\n" * 5
    v = J.judge(ok, assume_busy=True)
    assert v.busy == 5 and not v.flagged and v.median_clock == 1965
    assert J.judge(ok).busy == 0 and J.judge(ok).flagged          # without it: idle samples only
    bad = "0,1965,1965,612.0,0x0000000000000008,-,-,-,-,0,41,0\n"
    v = J.judge(bad, assume_busy=True)
    assert v.flagged and v.reason_names() == ["hw_slowdown"]
    low = "0,1100,1965,300.0,0x0000000000000000,-,-,-,-,0,41,0\n"
    assert J.judge(low, assume_busy=True).low == 1                   # a low clock with no reason: a leftover lock
