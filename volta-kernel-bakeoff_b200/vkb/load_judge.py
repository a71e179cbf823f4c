"""One line about a timed region from its nvidia-smi samples: did the B200 run at its own clocks?

The reference's judge (bench/load_flag.py) checks a V100 whose SM clock was locked at 1380 MHz. Clocks are never
locked on a shared B200, so this judge compares every busy sample with the GPU's own maximum SM clock instead, and
applies the rules a B200 timing must pass:

  rejected (FLAGGED): a hardware slowdown, hardware or software thermal slowdown or power-brake reason; an SM clock
      below LOW_FRAC of the maximum with no reason that explains it (a leftover clock lock); uncorrected ECC errors
      (non-zero or rising); no usable busy sample; unreadable fields on busy samples; malformed rows
  kept and noted: the software power cap (a 1 kW part under a dense GEMM sits on it), with its sample count

Input: nvidia-smi --query-gpu=<SAMPLE_FIELDS> --format=csv,noheader,nounits -lms <period> (ClockSampler in bench.py
writes exactly this). A last line without its newline (the sampler was stopped mid-write) is dropped, as the
reference does. CLI: python -m vkb.load_judge ROUND FILE prints the line (exit 0); wrong arguments exit 2.
"""
from __future__ import annotations

import sys
from dataclasses import dataclass, field

SAMPLE_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
                 "utilization.gpu,temperature.gpu,ecc.errors.uncorrected.volatile.total")
SM, SM_MAX, POWER, REASON, UTIL, TEMP, ECC = 1, 2, 3, 4, 9, 10, 11
COLUMNS = 12

LOW_FRAC = 0.8
# clocks_event_reasons.active bits
IDLE, APP_CLOCKS, SW_POWER_CAP, HW_SLOWDOWN = 0x1, 0x2, 0x4, 0x8
SW_THERMAL, HW_THERMAL, HW_POWER_BRAKE = 0x20, 0x40, 0x80
REJECT = HW_SLOWDOWN | SW_THERMAL | HW_THERMAL | HW_POWER_BRAKE
EXPLAINS_LOW = IDLE | SW_POWER_CAP | REJECT   # a low clock with one of these is not a leftover lock


def _num(text: str) -> float | None:
    """A number at the start of an nvidia-smi field ('1965', '1965 MHz', '612.3 W', '[N/A]' -> None)."""
    parts = text.strip().split()
    if not parts:
        return None
    word = parts[0]
    for suffix in ("MHz", "W", "C", "%"):
        if word.endswith(suffix):
            word = word[: -len(suffix)]
    try:
        return float(word)
    except ValueError:
        return None


def _hex(text: str) -> int | None:
    parts = text.strip().split()
    if not parts:
        return None
    try:
        return int(parts[0], 16)
    except ValueError:
        return None


@dataclass
class Verdict:
    busy: int = 0
    min_clock: float | None = None
    max_clock: float | None = None
    median_clock: float | None = None
    max_temp: float = 0.0
    low: int = 0            # busy samples below LOW_FRAC of the maximum with no explaining reason
    rejected: int = 0       # busy samples with a rejecting reason
    power_cap: int = 0      # busy samples on the software power cap (noted only)
    reasons: int = 0        # union of the rejecting reason bits seen
    notes: list = field(default_factory=list)

    @property
    def flagged(self) -> bool:
        return bool(self.low or self.rejected or self.notes)

    def reason_names(self) -> list:
        names = {HW_SLOWDOWN: "hw_slowdown", SW_THERMAL: "sw_thermal_slowdown", HW_THERMAL: "hw_thermal_slowdown",
                 HW_POWER_BRAKE: "hw_power_brake_slowdown"}
        out = [n for b, n in names.items() if self.reasons & b]
        if self.power_cap:
            out.append("sw_power_cap")
        return out


def _rows(text: str) -> tuple[list, int]:
    malformed = 0
    if text and not text.endswith("\n"):
        head, nl, _ = text.rpartition("\n")
        if not nl:
            return [], int(bool(text.strip()))
        text = head + "\n"
    rows = []
    for line in text.splitlines():
        if not line.strip():
            continue
        f = [p.strip() for p in line.split(",")]
        if len(f) < COLUMNS:
            malformed += 1
            continue
        rows.append(f)
    return rows, malformed


def _plural(n: int, what: str) -> str:
    return f"{n} {what}" if n == 1 else f"{n} {what}s"


def judge(text: str, assume_busy: bool = False) -> Verdict:
    """assume_busy: every sample was taken while the timed work ran (bench.py's NVML sampler polls only inside the
    timed region), so a zero utilization reading -- NVML averages it over a longer window than a short burst -- does
    not make a sample idle."""
    v = Verdict()
    rows, malformed = _rows(text)
    clocks, ecc_vals = [], []
    bad_util = bad_clock = bad_reason = bad_ecc = 0
    for f in rows:
        util, clk, mx = _num(f[UTIL]), _num(f[SM]), _num(f[SM_MAX])
        why, temp, ecc = _hex(f[REASON]), _num(f[TEMP]), _num(f[ECC])
        if ecc is None:
            bad_ecc += 1
        else:
            ecc_vals.append(ecc)
        if util == 0 and not assume_busy:
            continue   # idle: the GPU may clock down
        if util == 0:
            util = 100.0
        if util is None:
            bad_util += 1
        else:
            v.busy += 1
            if temp is not None:
                v.max_temp = max(v.max_temp, temp)
        if mx is not None:
            v.max_clock = mx if v.max_clock is None else max(v.max_clock, mx)
        if why is None:
            bad_reason += 1
        else:
            if why & REJECT:
                v.rejected += 1
                v.reasons |= why & REJECT
            if why & SW_POWER_CAP:
                v.power_cap += 1
        if clk is None or mx is None:
            bad_clock += 1
            continue
        clocks.append(clk)
        if clk < LOW_FRAC * mx and (why is None or not why & EXPLAINS_LOW):
            v.low += 1
    if clocks:
        clocks.sort()
        v.min_clock, v.median_clock = clocks[0], clocks[len(clocks) // 2]
    if v.busy == 0:
        v.notes.append("no usable busy samples")
    if bad_util:
        v.notes.append(f"unreadable utilization on {_plural(bad_util, 'sample')}")
    if bad_clock:
        v.notes.append(f"unreadable SM clock on {_plural(bad_clock, 'sample')}")
    if bad_reason:
        v.notes.append(f"unreadable clock-event reasons on {_plural(bad_reason, 'sample')}")
    if malformed:
        v.notes.append(_plural(malformed, "malformed sample"))
    if bad_ecc and not ecc_vals:
        v.notes.append("ecc uncorrected unreadable")
    elif bad_ecc:
        v.notes.append(f"ecc uncorrected unreadable on {_plural(bad_ecc, 'sample')}")
    if ecc_vals:
        peak = max(ecc_vals)
        if peak > ecc_vals[0]:
            v.notes.append(f"ecc uncorrected {ecc_vals[0]:g}->{peak:g}")
        elif peak != 0:
            v.notes.append(f"ecc uncorrected {peak:g}")
    return v


def format_line(round_id: str, v: Verdict) -> str:
    clk = "-" if v.min_clock is None else f"{v.min_clock:g}"
    mx = "-" if v.max_clock is None else f"{v.max_clock:g}"
    reasons = f" (0x{v.reasons:x})" if v.reasons else ""
    cap = f", {v.power_cap} on the sw power cap" if v.power_cap else ""
    extra = (", " + ", ".join(v.notes)) if v.notes else ""
    mark = "  ** FLAGGED **" if v.flagged else ""
    return (f"round {round_id} under load: {v.busy} busy samples, SM clock min {clk} of max {mx} MHz, "
            f"max {v.max_temp:g} C, {v.low} below {int(LOW_FRAC * 100)}% of max without a reason, "
            f"{v.rejected} with slowdown reasons{reasons}{cap}{extra}{mark}")


def main(argv: list) -> int:
    if len(argv) != 3:
        sys.stderr.write("usage: python -m vkb.load_judge ROUND SAMPLES.csv\n")
        return 2
    round_id, path = argv[1], argv[2]
    try:
        with open(path, encoding="utf-8", errors="replace") as fh:
            text = fh.read()
    except OSError as err:
        v = Verdict()
        v.notes.append(f"could not read samples ({err.strerror or 'unknown error'})")
        print(format_line(round_id, v))
        return 0
    print(format_line(round_id, judge(text)))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
