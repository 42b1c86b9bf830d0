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


# NVML clock-event reason bits (nvmlClocksEventReason*), public NVML API values.
_NVML_REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                 "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}


def _summarise(rows: list[tuple[float, float, float, set]]) -> dict:
    if not rows:
        return {"available": False, "samples": 0}
    reasons = set()
    for r in rows:
        reasons |= r[3]
    return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
            "power_w_max": round(max(r[2] for r in rows), 1), "reasons": sorted(reasons), "samples": len(rows)}


_SAMPLER_SRC = r"""
import sys, time, pynvml
out, interval, ids = sys.argv[1], float(sys.argv[2]), sys.argv[3:]
pynvml.nvmlInit()
hs = [pynvml.nvmlDeviceGetHandleByPciBusId(b) for b in ids] if ids else \
     [pynvml.nvmlDeviceGetHandleByIndex(i) for i in range(pynvml.nvmlDeviceGetCount())]
get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
mx = [pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in hs]
pw = [0.0] * len(hs)
with open(out, "w", buffering=1) as f:
    print("ready", file=f)
    k = 0
    while True:
        # SM clock and event reasons every pass; power every 8th pass (slower call)
        for i, h in enumerate(hs):
            if k % 8 == 0:
                pw[i] = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
            f.write("%.6f,%d,%d,%.1f,%d\n" % (time.time(), pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                    mx[i], pw[i], int(get(h))))
        k += 1
        time.sleep(interval)
"""


class ClockSampler:
    """Samples SM clocks, power and throttle reasons while active.

    Runs in a separate process (NVML, a pass over the GPUs every
    ``interval_ms``; ``nvidia-smi`` if NVML is missing), so the sampling never
    competes with the benchmark's own kernel launches. ``stop(t0, t1)``
    returns ``{"sm_mhz": median, "sm_max_mhz", "power_w_max", "reasons":
    [...], "samples"}`` over the GPUs whose PCI bus ids were given, counting
    only the samples taken between the host times ``t0`` and ``t1``
    (``time.time()``; the whole run when omitted). It only reads; nothing on
    the GPU changes.
    """

    def __init__(self, bus_ids: list[str] | None = None, interval_ms: float = 1.0):
        self.bus_ids = list(bus_ids) if bus_ids else []
        self.interval_ms = interval_ms
        self.proc = None
        self.path = None
        self.kind = None

    def start(self, wait_s: float = 5.0) -> "ClockSampler":
        import sys
        import time

        fd, self.path = tempfile.mkstemp(prefix="nab_clocks_", suffix=".csv")
        os.close(fd)
        try:
            import pynvml  # noqa: F401

            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_SRC, self.path,
                                          str(self.interval_ms / 1000.0), *self.bus_ids],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            self.kind = "nvml"
        except (ImportError, OSError):
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                     f"--loop-ms={max(100, self.interval_ms)}", f"--filename={self.path}"],
                    stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
                self.kind = "nvidia-smi"
            except OSError:
                self.proc = None
        # wait until the sampler is producing, so the timed region is covered
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < wait_s:
            if self.proc.poll() is not None:
                break
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.01)
        return self

    def stop(self, t0: float | None = None, t1: float | None = None) -> dict:
        if self.proc is None:
            return {"available": False, "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        rows = []
        try:
            with open(self.path) as f:
                lines = f.read().splitlines()
        finally:
            os.unlink(self.path)
        if self.kind == "nvml":
            for line in lines:
                parts = line.split(",")
                if len(parts) != 5:
                    continue
                ts = float(parts[0])
                if (t0 is not None and ts < t0) or (t1 is not None and ts > t1):
                    continue
                bits = int(parts[4])
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]),
                             {k for k, b in _NVML_REASONS.items() if bits & b}))
        else:
            want = {b.upper().lstrip("0") for b in self.bus_ids}
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            for line in lines:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or (want and parts[0].upper().lstrip("0") not in want):
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]),
                                 {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}))
                except ValueError:
                    continue
        out = _summarise(rows)
        out["source"] = self.kind
        return out


def clocks_ok(clocks: dict | None, min_samples: int = 10) -> bool | None:
    """False for a run that saw hardware/thermal slowdown or SM clocks well
    below the maximum with no reason given (a leftover clock lock); None
    ("unknown") when fewer than ``min_samples`` samples cover the run."""
    if not clocks or not clocks.get("available", True) or clocks.get("samples", 0) < min_samples:
        return None
    if any(r in clocks.get("reasons", []) for r in REJECT_REASONS):
        return False
    mhz, top = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    if mhz and top and mhz < 0.8 * top and not clocks.get("reasons"):
        return False
    return True
