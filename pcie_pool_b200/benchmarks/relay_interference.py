"""Pooled transfers while other work loads the GPUs: relay idle versus busy,
target busy, and the target's own PCIe link busy.

    python -m pcie_pool_b200.benchmarks.relay_interference --gpus 4 --bytes 4G --repeats 5

One pooled H2D transfer of ``--bytes`` into GPU0 over the direct lane plus
every other GPU as a relay (equal split), timed with CUDA events (median of
``--repeats`` after one warm-up) under each scenario:

* ``idle``           nothing else runs;
* ``relays_busy``    the load kernel (``ops.interference``: every SM streaming
                     FMAs over a ``--load-bytes`` fp32 buffer, so both SMs and
                     HBM are busy) runs on every relay GPU;
* ``target_busy``    the load kernel runs on the target GPU, where the
                     landing kernel shares SMs and HBM with it;
* ``all_busy``       both;
* ``target_link_busy`` a background host->GPU0 copy stream keeps the target's
                     own PCIe link busy (another tenant on the same link).

The load is queued back to back for about ``--load-factor`` times the idle
transfer time before the timed transfer starts, so it covers the transfer;
every launch is a plain kernel of bounded length.  Each line reports GB/s,
the slowdown against ``idle`` and whether the landed bytes' checksums match
the host's.  The scenario list follows the reference's benchmark notes
(relay idle versus busy, target link saturated versus not).
"""

from __future__ import annotations

import argparse
import json
import statistics

SCENARIOS = ("idle", "relays_busy", "target_busy", "all_busy", "target_link_busy")
UNITS = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}


def parse_size(s: str) -> int:
    s = str(s).strip().upper()
    return int(float(s[:-1]) * UNITS[s[-1]]) if s and s[-1] in UNITS else int(s)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=0, help="GPUs to use (0 = all visible)")
    p.add_argument("--bytes", default="4G")
    p.add_argument("--chunk", default="16M")
    p.add_argument("--repeats", type=int, default=5)
    p.add_argument("--scenarios", default=",".join(SCENARIOS))
    p.add_argument("--load-bytes", default="1G", help="fp32 buffer the load kernel streams over, per GPU")
    p.add_argument("--load-iters", type=int, default=16, help="FMAs per element per load launch")
    p.add_argument("--load-factor", type=float, default=2.0, help="queued load / idle transfer time")
    a = p.parse_args(argv)
    a.scenario_list = [s for s in a.scenarios.split(",") if s]
    bad = [s for s in a.scenario_list if s not in SCENARIOS]
    if bad:
        p.error(f"unknown scenarios: {bad}")
    return a


def loaded_devices(scenario: str, target: int, relays: list[int]) -> list[int]:
    """GPUs that run the load kernel in a scenario."""
    return {"relays_busy": list(relays), "target_busy": [target], "all_busy": [target, *relays]}.get(scenario, [])


def main(argv=None) -> int:
    import torch

    from .._native import native
    from ..ops import interference
    from ..parallel.engine import H2D, PoolEngine, split_even
    from ..utils.checksum import combine, rebase_chunk_sums
    from ..utils.host_memory import PinnedHostBuffer
    from .common import ClockSampler, fill_random

    a = parse_args(argv)
    n, chunk = parse_size(a.bytes), parse_size(a.chunk)
    ngpu = torch.cuda.device_count() if a.gpus <= 0 else min(a.gpus, torch.cuda.device_count())
    devices = list(range(ngpu))
    target, relays = 0, devices[1:]
    host = PinnedHostBuffer(n, fill=None)
    fill_random(host.numpy(), seed=3)
    want = tuple(int(x) for x in native().checksum_host(host.ptr, n))
    dev = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    eng = PoolEngine(devices, slot_bytes=chunk, slots=3, ctas_per_lane=4, timeout_s=30.0)
    lanes = split_even(n, chunk, devices)
    load_elems = parse_size(a.load_bytes) // 4
    loads = {g: torch.zeros(load_elems, dtype=torch.float32, device=f"cuda:{g}") for g in devices}
    streams = {g: torch.cuda.Stream(device=g) for g in devices}
    bg_host = PinnedHostBuffer(min(n, 1 << 30), fill=0)
    bg_src = bg_host.torch()  # page-locked: the background copies are asynchronous
    bg_dev = torch.empty(bg_host.nbytes, dtype=torch.uint8, device="cuda:0")

    def transfer():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = eng.run(H2D, target, host.ptr, n, dev.data_ptr(), n, lanes, checksum=True)
        e1.record()
        e1.synchronize()
        r.raise_for_status()
        return e0.elapsed_time(e1), r

    def launch_ms(g: int) -> float:
        s = streams[g]
        with torch.cuda.stream(s):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            interference(loads[g], iters=a.load_iters)
            e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1)

    transfer()
    idle_ms = statistics.median(transfer()[0] for _ in range(max(1, a.repeats)))
    per_launch = {g: max(launch_ms(g), 1e-3) for g in devices}
    clocks = ClockSampler(ngpu).start()
    base = None
    for sc in a.scenario_list:
        times, last = [], None
        for _ in range(max(1, a.repeats)):
            for g in loaded_devices(sc, target, relays):
                k = max(1, int(a.load_factor * idle_ms / per_launch[g]) + 1)
                with torch.cuda.stream(streams[g]):
                    for _ in range(k):
                        interference(loads[g], iters=a.load_iters)
            if sc == "target_link_busy":
                with torch.cuda.stream(streams[target]):
                    for _ in range(max(1, int(a.load_factor * n / bg_dev.numel()) + 1)):
                        bg_dev.copy_(bg_src, non_blocking=True)
            ms, last = transfer()
            times.append(ms)
            for g in devices:
                streams[g].synchronize()
        med = statistics.median(times)
        base = med if sc == "idle" else (base or idle_ms)
        ok = combine(rebase_chunk_sums(last.checksums, lanes)) == want
        print(json.dumps({"scenario": sc, "gpus": ngpu, "bytes": n, "chunk_bytes": chunk, "ms": round(med, 3),
                          "gb_per_s": round(n / 1e9 / (med / 1e3), 2), "slowdown_vs_idle": round(med / base, 3),
                          "loaded_gpus": loaded_devices(sc, target, relays), "verified": ok,
                          "lane_ms": [(l.device, round(l.cuda_ms, 2)) for l in last.lanes]}), flush=True)
    print(json.dumps({"clocks": clocks.stop()}), flush=True)
    del eng
    host.release()
    bg_host.release()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
