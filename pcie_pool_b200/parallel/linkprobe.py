"""Link probe: measured bandwidth for the planner.

The reference measures each link once, alone, with one 256 MiB copy and no
warm-up (cpp/src/profiler_cuda.cu:31-160), so it cannot see lanes that share
host resources, and its daemon never calls it (profiles arrive only through
PUT_PROFILE).  This probe measures, on the engine the transfers will use:

  1. solo: the target's direct lane and every relay lane alone, H2D and D2H
     (warm-up, then the median of repeats);
  2. concurrent: all lanes together, re-split by the measured rates until
     they finish together (``LaneBalancer`` fixed point);
  3. lane sets: prefixes of the lanes ordered by concurrent rate, each
     balanced the same way; the set with the highest aggregate wins, per
     direction (adding lanes can lower the aggregate when they share an
     oversubscribed host link).

The result is a daemon profile entry (GiB/s in ``*_gbps`` fields, as in the
reference) with a ``concurrent`` section the planner uses when present.
"""

from __future__ import annotations

import statistics
import time
from typing import Sequence

from .balance import LaneBalancer
from .engine import D2H, H2D, PoolEngine
from .planning import plan_lanes

GIB = float(1 << 30)


def _run(eng: PoolEngine, direction: int, target: int, host, dev_ptr: int, nbytes: int, lanes,
         repeats: int = 3):
    out = []
    for _ in range(repeats):
        r = eng.run(direction, target, host.ptr, nbytes, dev_ptr, nbytes, lanes)
        r.raise_for_status()
        out.append(r)
    out.sort(key=lambda r: r.cuda_ms)
    return out[len(out) // 2]


def _balanced(eng: PoolEngine, direction: int, target: int, host, dev_ptr: int, nbytes: int,
              devices: Sequence[int], chunk: int, rounds: int = 3):
    """Run ``rounds`` balancing iterations over ``devices``; returns
    (aggregate GB/s, per-device GiB/s rate estimates)."""
    bal = LaneBalancer(alpha=1.0)
    w = None
    best = None
    for _ in range(rounds):
        lanes = plan_lanes(nbytes, chunk, list(devices), target, bw_gibps=w)
        r = eng.run(direction, target, host.ptr, nbytes, dev_ptr, nbytes, lanes)
        r.raise_for_status()
        bal.observe(target, "x", r)
        w = bal.weights(target, "x", list(devices))
        if best is None or r.cuda_ms < best.cuda_ms:
            best = r
    return best.gb_per_s, bal.rates(target, "x")


def probe_profile(eng: PoolEngine, target: int, relays: Sequence[int], nbytes: int = 256 << 20,
                  chunk: int | None = None, concurrent: bool = True, choose_lanes: bool = True) -> dict:
    """Measure and return a daemon-format profile for ``target``."""
    import torch

    from ..utils.host_memory import PinnedHostBuffer

    chunk = int(chunk or min(eng.slot_bytes, 16 << 20))
    relays = [int(r) for r in relays if int(r) != int(target)]
    host = PinnedHostBuffer(nbytes, fill=0)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{target}")
    t0 = time.perf_counter()
    solo: dict[str, dict[int, float]] = {"h2d": {}, "d2h": {}}
    for dname, d in (("h2d", H2D), ("d2h", D2H)):
        for lane_dev in [target, *relays]:
            lanes = plan_lanes(nbytes, chunk, [lane_dev], target)
            _run(eng, d, target, host, dev.data_ptr(), nbytes, lanes, repeats=1)  # warm-up
            r = _run(eng, d, target, host, dev.data_ptr(), nbytes, lanes)
            solo[dname][lane_dev] = (nbytes / GIB) / (r.cuda_ms / 1e3)
    p2p: dict[int, float] = {}
    for rly in relays:
        src = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{rly}")
        dev.copy_(src)
        torch.cuda.synchronize()
        ms = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.device(target):
                e0.record()
                dev.copy_(src, non_blocking=True)
                e1.record()
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        p2p[rly] = (nbytes / GIB) / (statistics.median(ms) / 1e3)
        del src
    conc: dict[str, dict] = {}
    if concurrent and relays:
        for dname, d in (("h2d", H2D), ("d2h", D2H)):
            _gbs, rates = _balanced(eng, d, target, host, dev.data_ptr(), nbytes, [target, *relays], chunk)
            order = sorted(rates, key=lambda k: (-rates[k], k != target))
            if target in order:  # the direct lane always leads
                order.remove(target)
                order.insert(0, target)
            best_set, best_gbs, best_rates = [target, *relays], _gbs, rates
            if choose_lanes:
                for k in range(1, len(order) + 1):
                    cand = order[:k]
                    gbs, r = _balanced(eng, d, target, host, dev.data_ptr(), nbytes, cand, chunk)
                    if gbs > best_gbs * 1.02:
                        best_set, best_gbs, best_rates = cand, gbs, r
            conc[dname] = {"lanes": [int(x) for x in best_set], "aggregate_gb_per_s": round(best_gbs, 3),
                           "lane_gibps": {str(k): round(v, 3) for k, v in best_rates.items()},
                           "all_lane_gibps": {str(k): round(v, 3) for k, v in rates.items()}}
    profile = {
        "target_device": int(target),
        "direct_h2d_bw_gbps": solo["h2d"][target],
        "direct_d2h_bw_gbps": solo["d2h"][target],
        "relays": [{"relay_device": r, "target_device": int(target), "h2d_bw_gbps": solo["h2d"][r],
                    "d2h_bw_gbps": solo["d2h"][r], "p2p_bw_gbps": p2p.get(r, 0.0),
                    "effective_bw_gbps": solo["h2d"][r], "effective_d2h_bw_gbps": solo["d2h"][r],
                    "p2p_enabled": True} for r in relays],
        "concurrent": conc,
        "measured_by": {"probe": "pcie_pool_b200.linkprobe", "bytes": int(nbytes), "chunk_bytes": chunk,
                        "seconds": round(time.perf_counter() - t0, 3)},
    }
    host.release()
    return profile


def concurrent_lane_plan(profile: dict, direction: str) -> tuple[list[int], list[float]] | None:
    """Lane devices and their concurrent GiB/s from a probed profile."""
    c = (profile or {}).get("concurrent", {}).get(direction)
    if not c:
        return None
    lanes = [int(x) for x in c["lanes"]]
    rates = c.get("lane_gibps", {})
    if not all(str(l) in rates for l in lanes):
        return None
    return lanes, [float(rates[str(l)]) for l in lanes]


def profile_daemon(daemon, targets: Sequence[int], relays: Sequence[int], nbytes: int = 256 << 20) -> list[dict]:
    """Probe every target with the daemon's relays and PUT the profiles."""
    import torch

    out = []
    devs = sorted({int(t) for t in targets} | {int(r) for r in relays})
    eng = PoolEngine(devs, slot_bytes=16 << 20, slots=3)
    for t in targets:
        rl = [r for r in relays if r != t]
        prof = probe_profile(eng, int(t), rl, nbytes)
        daemon.put_profile(int(t), rl, prof, profile_bytes=nbytes)
        out.append(prof)
    del eng
    torch.cuda.synchronize()
    return out


__all__ = ["concurrent_lane_plan", "probe_profile", "profile_daemon"]
