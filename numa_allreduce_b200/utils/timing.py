"""Device timing, bandwidth arithmetic and clock sampling for benchmarks.

Conventions (nccl-tests): for a message of S bytes per rank on n ranks taking
t seconds, algbw = S / t and busbw = algbw * 2 (n - 1) / n. The reference
reported 2 S / t (examples/profile_nsys_ncu.py:180-185), which is neither.
Multi-GPU times are the maximum over ranks of CUDA-event device times.
"""

from __future__ import annotations

import os
import statistics
import subprocess
import tempfile

import torch

CLOCK_FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REJECT_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def busbw_gbs(nbytes: int, seconds: float, n: int) -> float:
    if seconds <= 0 or n <= 1:
        return 0.0
    return nbytes / seconds * 2 * (n - 1) / n / 1e9


def algbw_gbs(nbytes: int, seconds: float) -> float:
    return nbytes / seconds / 1e9 if seconds > 0 else 0.0


def percentile(values: list[float], q: float) -> float:
    if not values:
        return float("nan")
    v = sorted(values)
    k = (len(v) - 1) * q
    lo, hi = int(k), min(int(k) + 1, len(v) - 1)
    return v[lo] + (v[hi] - v[lo]) * (k - lo)


def flush_l2(buf: torch.Tensor | None = None) -> torch.Tensor:
    """Writes a buffer larger than the 126 MB L2 (returns it for reuse)."""
    if buf is None:
        buf = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    buf.fill_(1)
    return buf


def pci_bus_id(device: int) -> str:
    p = torch.cuda.get_device_properties(device)
    return f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0".upper()


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons every 200 ms while active.

    ``stop()`` returns ``{"sm_mhz": median, "sm_max_mhz": ..., "power_w_max":
    ..., "reasons": [...], "samples": n}`` for the GPUs whose PCI bus ids were
    given (all GPUs if none). Nothing is changed on the GPU: it only reads.
    """

    def __init__(self, bus_ids: list[str] | None = None, interval_ms: int = 200):
        self.bus_ids = {b.upper().lstrip("0") for b in bus_ids} if bus_ids else None
        self.interval_ms = interval_ms
        self.proc = None
        self.path = None

    def start(self) -> "ClockSampler":
        fd, self.path = tempfile.mkstemp(prefix="nab_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 f"--loop-ms={self.interval_ms}", f"--filename={self.path}"],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"available": False}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    bus = parts[0].upper().lstrip("0")
                    if self.bus_ids and bus not in self.bus_ids:
                        continue
                    rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return {"available": False}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return float("nan")

        sm = [num(r[1]) for r in rows]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(num(r[2]) for r in rows),
                "power_w_max": max(num(r[3]) for r in rows), "reasons": sorted(reasons),
                "samples": len(rows)}


def clocks_ok(clocks: dict) -> bool:
    """False for a run that saw hardware/thermal slowdown or a clock stuck low."""
    if not clocks.get("available", True):
        return True
    if any(r in clocks.get("reasons", []) for r in REJECT_REASONS):
        return False
    return True
