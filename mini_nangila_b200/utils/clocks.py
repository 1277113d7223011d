"""Sample SM clocks and throttle reasons with ``nvidia-smi`` while a timed
region runs (read-only queries; no GPU setting is changed)."""
from __future__ import annotations

import os
import signal
import statistics
import subprocess
import tempfile

FIELDS = [
    "index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
    "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
    "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap",
]
REASON_KEYS = {
    "clocks_event_reasons.hw_slowdown": "hw_slowdown",
    "clocks_event_reasons.hw_thermal_slowdown": "hw_thermal_slowdown",
    "clocks_event_reasons.sw_thermal_slowdown": "sw_thermal_slowdown",
    "clocks_event_reasons.sw_power_cap": "sw_power_cap",
}


class ClockSampler:
    """``nvidia-smi -lms`` in the background.  ``begin()`` / ``end()`` mark
    the timed region: the statistics of ``stop()`` come from the samples
    written between the marks (or, for a region shorter than the period,
    the samples on either side of it), so the sampler can be started before
    the warm-up steps and be producing samples when the region starts
    (``nvidia-smi`` takes a noticeable time to print its first sample on a
    multi-GPU query).  Without marks, every sample counts."""

    def __init__(self, gpus: list[int] | None = None, period_ms: int = 200):
        self.gpus = gpus
        self.period_ms = period_ms
        self.proc = None
        self.path = None
        self._marks: list[int] = []

    def _lines(self) -> int:
        try:
            with open(self.path) as fh:
                return sum(1 for line in fh if line.endswith("\n"))
        except (OSError, TypeError):
            return 0

    def begin(self) -> None:
        """Mark the start of the timed region."""
        self._marks = [self._lines()]

    def end(self) -> None:
        """Mark the end of the timed region."""
        if self._marks:
            self._marks = self._marks[:1] + [self._lines()]

    def start(self) -> "ClockSampler":
        fd, self.path = tempfile.mkstemp(prefix="ngl_clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={','.join(FIELDS)}", "--format=csv,noheader,nounits", "-lms",
               str(self.period_ms)]
        if self.gpus:
            cmd += ["-i", ",".join(str(g) for g in self.gpus)]
        try:
            with open(self.path, "w") as log:  # the child keeps its own descriptor
                self.proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.DEVNULL, start_new_session=True)
        except OSError:
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is not None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
            self.proc.wait(timeout=10)
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if not self.path or not os.path.exists(self.path):
            return out
        with open(self.path) as fh:
            lines = [line for line in fh if line.endswith("\n")]
        os.unlink(self.path)
        if len(self._marks) == 2:
            # the timed region's lines (the marks count complete lines), or
            # the samples just before and after a region shorter than the period
            a, b = self._marks
            lines = lines[a:b] or lines[max(0, a - 1): b + 1] or lines
        rows = []
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(FIELDS):
                rows.append(dict(zip(FIELDS, parts)))
        if not rows:
            return out
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r["clocks.sm"]) for r in rows if num(r["clocks.sm"])]
        mx = [num(r["clocks.max.sm"]) for r in rows if num(r["clocks.max.sm"])]
        pw = [num(r["power.draw"]) for r in rows if num(r["power.draw"])]
        reasons = set()
        for r in rows:
            for k, name in REASON_KEYS.items():
                if r.get(k, "").lower().startswith("active"):
                    reasons.add(name)
        # Median under load: samples above 50% of max (idle samples at the
        # edges of the window excluded).
        peak = max(mx) if mx else None
        loaded = [s for s in sm if peak is None or s >= 0.5 * peak] or sm
        out.update(sm_mhz=statistics.median(loaded) if loaded else None, sm_max_mhz=peak,
                   reasons=sorted(reasons), samples=len(rows), power_w_max=max(pw) if pw else None)
        return out
