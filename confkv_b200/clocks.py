"""SM clock and throttle-reason sampling (nvidia-smi) around a timed region.

Reading clocks only: nothing here changes a GPU setting.
"""

from __future__ import annotations

import statistics
import subprocess
import time


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return summarize(out)


REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def summarize(text: str) -> dict | None:
    """Summary of `nvidia-smi --query-gpu=<ClockSampler.FIELDS> --format=csv,noheader,nounits`
    output: median SM clock, the highest max clock seen, and every throttle
    reason that was Active in any sample. Lines that do not parse (a line cut
    off when the sampler was stopped) are skipped; None when no line parses."""
    sm, mx, reasons = [], 0.0, set()
    for line in text.strip().splitlines():
        r = [f.strip() for f in line.split(",")]
        try:
            clk, top = float(r[1]), float(r[2])
            flags = r[5:9]
        except (ValueError, IndexError):
            continue
        if len(flags) != len(REASONS):
            continue
        sm.append(clk)
        mx = max(mx, top)
        reasons.update(nm for nm, v in zip(REASONS, flags) if v.lower() == "active")
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}
