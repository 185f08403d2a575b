"""Samples SM clocks and throttle reasons with nvidia-smi while a timed region
runs (read-only: nothing here changes any GPU setting)."""

from __future__ import annotations

import shutil
import subprocess
import threading
import time

QUERY = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_COLS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """``with ClockSampler(uuid) as s: ...`` then ``s.summary()``.

    A reader thread collects the samples as nvidia-smi prints them, so
    ``count()`` tells a caller whether the region seen so far has enough of
    them (``keep_busy`` runs more work until it does)."""

    def __init__(self, uuid: str | None = None, period_ms: int = 50):
        self.uuid = uuid
        self.period_ms = period_ms
        self.proc = None
        self.rows = []
        self._lock = threading.Lock()
        self._thread = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               f"-lms={self.period_ms}"]
        if self.uuid:
            cmd.append(f"--id={self.uuid}")
        self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                     text=True, bufsize=1)
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 10:
                with self._lock:
                    self.rows.append(parts)

    def count(self) -> int:
        with self._lock:
            return len(self.rows)

    def keep_busy(self, work, min_samples: int = 5, max_seconds: float = 5.0) -> int:
        """Runs ``work()`` (untimed, e.g. more calls of the timed workload)
        until ``min_samples`` samples exist or ``max_seconds`` pass; returns
        how many times it ran.  A timed region of a few milliseconds ends
        before nvidia-smi prints its first sample."""
        if self.proc is None:
            return 0
        n, t0 = 0, time.perf_counter()
        while self.count() < min_samples and time.perf_counter() - t0 < max_seconds:
            work()
            n += 1
        return n

    def __exit__(self, *exc):
        if self.proc is None:
            return False
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)
        return False

    def summary(self) -> dict | None:
        with self._lock:
            rows = list(self.rows)
        if not rows:
            return None
        sm = []
        mx = 0.0
        reasons = set()
        for r in rows:
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
