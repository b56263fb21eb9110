"""Sample GPU clocks and throttle reasons with nvidia-smi while a timed region runs."""
from __future__ import annotations

import os
import statistics
import subprocess
import tempfile

_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """`with ClockSampler(gpus) as s: ...` then `s.summary()`.  Reads settings only."""

    def __init__(self, gpus: list[int] | None = None, period_ms: int = 200):
        self.gpus = gpus
        self.period_ms = period_ms
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits",
               "-lms", str(self.period_ms)]
        if self.gpus is not None:
            cmd += ["-i", ",".join(str(g) for g in self.gpus)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # nvidia-smi needs a moment before its first sample; wait for it so a short timed region
        # is still covered.
        import time

        deadline = time.time() + 5.0
        while self.proc is not None and time.time() < deadline:
            self.out.flush()
            if os.path.getsize(self.out.name) > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.out.flush()

    def summary(self) -> dict:
        self.out.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}
