"""Sample GPU SM clocks and throttle reasons with nvidia-smi while a region runs.

Read-only: queries ``clocks.sm``, ``clocks.max.sm``, power and ``clocks_event_reasons.*``;
never changes a clock or any other GPU setting.
"""
from __future__ import annotations

import shutil
import statistics
import subprocess
import tempfile
from typing import Optional

_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    def __init__(self, gpu_index: Optional[int] = None, period_ms: int = 200):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.file = None

    def __enter__(self):
        self.start()
        return self

    def __exit__(self, *exc):
        self.stop()

    def start(self):
        if shutil.which("nvidia-smi") is None:
            return
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = ["nvidia-smi", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits",
               f"-lms={self.period}"]
        if self.gpu is not None:
            cmd.append(f"--id={self.gpu}")
        self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:  # pragma: no cover
                self.proc.kill()
            self.proc = None

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        self.file.seek(0)
        sm, mx, reasons, power = [], [], set(), []
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(_REASONS, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s, p in zip(sm, power) if p > 250] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx),
                "samples": len(sm), "power_w_max": max(power), "reasons": sorted(reasons)}
