"""Samples SM clocks and throttle reasons with nvidia-smi while a timed region
runs (read-only queries; no GPU setting is changed)."""
from __future__ import annotations

import csv
import io
import os
import signal
import statistics
import subprocess

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int | None = None, period_ms: int = 200):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               f"-lms", str(self.period_ms)]
        if self.gpu_index is not None:
            cmd += ["-i", str(self.gpu_index)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True, start_new_session=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"available": False}
        try:
            os.killpg(self.proc.pid, signal.SIGTERM)
        except ProcessLookupError:
            pass
        out, _ = self.proc.communicate(timeout=10)
        return summarize(out)


def summarize(text: str) -> dict:
    rows = []
    for rec in csv.reader(io.StringIO(text)):
        if len(rec) < 9:
            continue
        try:
            rows.append({"sm": float(rec[1]), "max": float(rec[2]), "power": float(rec[3]),
                         "hw_slowdown": rec[5].strip() == "Active",
                         "hw_thermal_slowdown": rec[6].strip() == "Active",
                         "sw_thermal_slowdown": rec[7].strip() == "Active",
                         "sw_power_cap": rec[8].strip() == "Active"})
        except ValueError:
            continue
    if not rows:
        return {"available": False}
    loaded = [r for r in rows if r["power"] > 300] or rows
    reasons = sorted({k for r in loaded for k in REASONS if r[k]})
    return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
            "sm_max_mhz": max(r["max"] for r in rows),
            "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded),
            "power_w_max": max(r["power"] for r in rows)}
