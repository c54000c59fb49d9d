"""Sample GPU clocks and throttle reasons with nvidia-smi while a timed region runs.

Reads only (`nvidia-smi --query-gpu ... -lms`); never changes a clock, power limit or mode.
"""

from __future__ import annotations

import csv
import io
import os
import shutil
import subprocess
import tempfile

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, period_ms: int = 200, gpu: int | None = None):
        self.period_ms, self.gpu = period_ms, gpu
        self.proc = None
        self.path = None

    def start(self):
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"]
        if self.gpu is not None:
            cmd.insert(1, f"--id={self.gpu}")
        self.out = open(self.path, "w")
        self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        with open(self.path) as f:
            text = f.read()
        os.unlink(self.path)
        return summarize(text)


def summarize(text: str) -> dict:
    sm, smax, power, reasons = [], [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for row in csv.reader(io.StringIO(text)):
        if len(row) < 9:
            continue
        try:
            sm.append(float(row[1]))
            smax.append(float(row[2]))
            power.append(float(row[3]))
        except ValueError:
            continue
        for name, val in zip(names, row[5:9]):
            if val.strip().lower() == "active":
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
    busy = [s for s in sm if s > 0.5 * max(sm)] or sm
    busy.sort()
    return {
        "sm_mhz": busy[len(busy) // 2],
        "sm_max_mhz": max(smax),
        "power_w_max": max(power),
        "samples": len(sm),
        "reasons": sorted(reasons),
    }
