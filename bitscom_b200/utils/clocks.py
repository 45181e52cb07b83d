"""Samples GPU clocks and throttle reasons with nvidia-smi while a timed region runs.

Read-only: it only queries ``nvidia-smi --query-gpu`` (it never changes a
clock or any other GPU setting).
"""

from __future__ import annotations

import statistics
import subprocess
import tempfile
from typing import Dict, List, Optional

_FIELDS = (
    "index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
    "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
    "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
)
_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """Context manager: ``with ClockSampler([0]) as cs: ...; cs.summary()``."""

    def __init__(self, gpus: Optional[List[int]] = None, period_ms: int = 200):
        self.gpus = gpus
        self.period_ms = period_ms
        self.proc = None
        self.file = None
        self.rows: List[List[str]] = []

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=True)
            cmd = ["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits", "-lms", str(self.period_ms)]
            if self.gpus is not None:
                cmd += ["-i", ",".join(str(g) for g in self.gpus)]
            self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.file.flush()
            self.file.seek(0)
            for line in self.file.read().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 10:
                    self.rows.append(parts)
            self.file.close()
        return False

    def summary(self) -> Dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        loaded = [r for r in self.rows if (num(r[4]) or 0) >= 50] or self.rows
        sm = [num(r[1]) for r in loaded if num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if num(r[2]) is not None]
        reasons = set()
        for r in loaded:
            for name, val in zip(_REASONS, r[6:10]):
                if val.strip().lower() in ("active", "0x1", "1"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(self.rows),
            "samples_under_load": len(loaded),
            "power_w_max": max((num(r[3]) or 0.0) for r in self.rows),
        }
