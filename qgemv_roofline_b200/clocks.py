"""Samples SM clocks and throttle reasons with nvidia-smi while a timed region
runs (read-only: nothing here changes any GPU setting)."""

from __future__ import annotations

import shutil
import subprocess
import tempfile

QUERY = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_COLS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """``with ClockSampler(uuid) as s: ...`` then ``s.summary()``."""

    def __init__(self, uuid: str | None = None, period_ms: int = 100):
        self.uuid = uuid
        self.period_ms = period_ms
        self.proc = None
        self.out = None
        self.rows = []

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        self.out = tempfile.TemporaryFile(mode="w+")
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               f"-lms={self.period_ms}"]
        if self.uuid:
            cmd.append(f"--id={self.uuid}")
        self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return False
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.seek(0)
        for line in self.out.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 10:
                self.rows.append(parts)
        self.out.close()
        return False

    def summary(self) -> dict | None:
        if not self.rows:
            return None
        sm = []
        mx = 0.0
        reasons = set()
        for r in self.rows:
            try:
                sm.append(float(r[2]))
                mx = max(mx, float(r[3]))
            except ValueError:
                continue
            for name, val in zip(REASON_COLS, r[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        sm.sort()
        # median over the samples in the upper half of the range (under load)
        loaded = [v for v in sm if v >= 0.5 * sm[-1]] or sm
        return {"sm_mhz": loaded[len(loaded) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}
