"""Sample GPU clocks and throttle reasons with ``nvidia-smi`` while a region runs.

Read-only: it queries clocks, power and the active clock-event reasons; it
never changes any GPU setting.
"""

from __future__ import annotations

import os
import signal
import statistics
import subprocess
import tempfile

QUERY = (
    "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
    "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
    "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
)
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int, period_ms: int = 200) -> None:
        self.gpu_index = int(gpu_index)
        self.period_ms = int(period_ms)
        self.proc: subprocess.Popen | None = None
        self.path = ""

    def __enter__(self) -> "ClockSampler":
        fd, self.path = tempfile.mkstemp(prefix="atlas_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", "-lms",
                 str(self.period_ms), "-i", str(self.gpu_index)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL, start_new_session=True,
            )
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                os.killpg(self.proc.pid, signal.SIGKILL)

    def summary(self) -> dict[str, object]:
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        except OSError:
            pass
        finally:
            if self.path:
                try:
                    os.unlink(self.path)
                except OSError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x: str) -> float | None:
            try:
                return float(x)
            except ValueError:
                return None

        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        power = [v for v in (num(r[3]) for r in rows) if v is not None]
        active = set()
        for r in rows:
            for name, val in zip(REASONS, r[5:9]):
                if val.lower() == "active":
                    active.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "power_w_max": max(power) if power else None,
            "reasons": sorted(active),
            "samples": len(rows),
        }
