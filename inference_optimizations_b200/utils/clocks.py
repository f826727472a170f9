"""Samples SM clocks, power and throttle reasons with nvidia-smi during a timed region (read-only queries).

Start before the timed region, stop after; `summary()` gives the median SM clock under load, the max clock and every
throttle reason seen active.  A run that saw hw_slowdown / hw_thermal_slowdown / sw_thermal_slowdown, or SM clocks
stuck far below max with no reason, is not a valid measurement; sw_power_cap is normal under a dense load.
"""
from __future__ import annotations

import csv
import os
import subprocess
import tempfile
from statistics import median
from typing import Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int, interval_ms: int = 200, log_path: Optional[str] = None):
        self.gpu = gpu_index
        self.path = log_path or tempfile.mktemp(prefix="iob_clocks_", suffix=".csv")
        self.proc = None
        self.interval = interval_ms

    def start(self) -> "ClockSampler":
        try:
            self._fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits",
                 f"-lms", str(self.interval)], stdout=self._fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._fh.close()
        return self.summary()

    def summary(self) -> dict:
        rows = []
        if os.path.exists(self.path):
            with open(self.path) as f:
                for r in csv.reader(f):
                    if len(r) >= 9:
                        rows.append([x.strip() for x in r])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].replace(".", "", 1).isdigit()]
        reasons = sorted({name for r in rows for name, v in zip(REASONS, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "reasons": reasons, "samples": len(rows)}


def rejected(summary: dict) -> Optional[str]:
    bad = [r for r in summary.get("reasons", []) if r != "sw_power_cap"]
    if bad:
        return "throttled: " + ",".join(bad)
    sm, mx = summary.get("sm_mhz"), summary.get("sm_max_mhz")
    if sm and mx and sm < 0.5 * mx and "sw_power_cap" not in summary.get("reasons", []):
        return f"SM clock {sm} MHz far below max {mx} with no reason (clock lock?)"
    return None
