"""Shared pieces of the benchmarks: clock sampling during timed regions, lane
calibration, the reference project's runtime (for its arm) and JSON output."""

from __future__ import annotations

import json
import statistics
import subprocess
import sys
import threading
from pathlib import Path

REPO_ROOT = Path(__file__).resolve().parents[2]


class ClockSampler:
    """``nvidia-smi`` SM clock / power / throttle-reason samples every 200 ms
    while a timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpus):
        """``gpus``: a GPU count (indices 0..gpus-1) or the indices sampled."""
        self.devices = set(range(gpus)) if isinstance(gpus, int) else {int(g) for g in gpus}
        self.gpus = len(self.devices)
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, reasons, power = [], [], set(), []
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.devices:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                pass
            for name, val in zip(self.REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": max(power) if power else None}


def fill_random_torch(host_t, seed: int = 0, device: int = 0) -> None:
    """Uniform-random bytes into a host uint8 tensor, generated on the GPU
    with torch and copied back.  The reference arms use this one: nothing of
    this project's native code may run on their path."""
    import torch

    g = torch.Generator(device=f"cuda:{device}").manual_seed(int(seed))
    step = 1 << 30
    n = host_t.numel()
    for o in range(0, n, step):
        k = min(step, n - o)
        host_t[o:o + k].copy_(torch.randint(0, 256, (k,), dtype=torch.uint8, device=f"cuda:{device}", generator=g))
    torch.cuda.synchronize(device)


def fill_random(arr, seed: int = 0, threads: int = 0) -> None:
    """Uniform-random bytes into a numpy uint8 array (native, multithreaded)."""
    from .._native import native

    native().fill_random_bytes(arr.ctypes.data, arr.size, seed, threads)


def calibrate(engine, target: int, devices, nbytes: int, chunk: int, direction: str = "h2d"):
    """Probe the lanes solo and together; return (lane_set, weights,
    balancer, profile).  One lane needs no probe."""
    from ..parallel.balance import LaneBalancer

    balancer = LaneBalancer(alpha=0.5)
    devices = list(devices)
    if len(devices) == 1:
        return devices, None, balancer, None
    from ..parallel.linkprobe import concurrent_lane_plan, probe_profile

    relays = [d for d in devices if d != target]
    profile = probe_profile(engine, target, relays, nbytes=min(nbytes, 1 << 30), chunk=chunk)
    lane_set, weights = devices, None
    picked = concurrent_lane_plan(profile, direction)
    if picked is not None:
        lane_set, weights = picked
        balancer.seed(target, direction, dict(zip(lane_set, weights)))
    return list(lane_set), weights, balancer, profile


def reference_runtime(n_gpus: int, chunk: int):
    """The reference's native Runtime on GPU0 with relays 1..N-1 and its own
    profile, or (None, reason)."""
    ref = REPO_ROOT / "baseline" / "_ref"
    if not (ref / "turbobus").exists():
        return None, "reference not installed under baseline/_ref"
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    from turbobus import runtime_engine
    from turbobus.runtime_engine import RuntimeOptions

    native = runtime_engine._turbobus
    if native is None:
        return None, "reference native extension failed to import"
    rt = native.Runtime(RuntimeOptions(chunk_bytes=chunk).to_native())
    rt.init(0, list(range(1, n_gpus)))
    return rt, None


def reference_plan(rt, nbytes: int, chunk: int, direction: str = "h2d"):
    from turbobus import runtime_engine
    from turbobus.planner_engine import PlannerEngine

    profile = rt.profile(256 << 20, False)
    plan = PlannerEngine().plan(nbytes, chunk, profile, "pool", direction=direction)
    return runtime_engine._native_transfer_plan(plan), profile


def emit(line: dict, json_out: str = "") -> None:
    s = json.dumps(line)
    print(s, flush=True)
    if json_out:
        Path(json_out).write_text(s + "\n")


__all__ = ["ClockSampler", "REPO_ROOT", "calibrate", "emit", "fill_random", "reference_plan", "reference_runtime"]
