"""Measured uplink groups: which GPUs' PCIe links share host-side bandwidth.

NVML and sysfs name each GPU's socket, root port and switches, but inside a
VM or a container the sharing that matters may be invisible: on this pool's
8-GPU nodes every GPU reports its own root port and one NUMA node, yet with
all eight links busy GPUs 0-3 get ~18 GiB/s each and GPUs 4-7 ~30 GiB/s, and
GPUs 0-3 alone top out at ~114 GB/s together -- they share an uplink the
topology does not show.  This probe measures it directly, without the
engine: every GPU first copies host -> device alone, then all at once
(plain ``cudaMemcpyAsync`` from page-locked memory, CUDA events on each
GPU's stream).  When the solo rates agree but the concurrent rates fall into
clearly separated levels, the levels are contention groups, and lanes are
spread across them before the topology keys are consulted.
"""

from __future__ import annotations

from typing import Sequence


def contention_groups(solo: dict[int, float], concurrent: dict[int, float], *, solo_tol: float = 0.12,
                      gap: float = 1.2) -> dict[int, str]:
    """GPU -> group label from measured rates (any unit), or {} when the
    measurement shows no shared-uplink structure: the solo rates must agree
    within ``solo_tol`` (a GPU that is slow on its own has a slow link, not a
    shared one), and the sorted concurrent rates are cut where one exceeds the
    previous by more than ``gap``x."""
    devs = sorted(set(solo) & set(concurrent))
    if len(devs) < 2:
        return {}
    s = [solo[d] for d in devs]
    if min(s) <= 0 or max(s) > (1 + solo_tol) * min(s):
        return {}
    order = sorted(devs, key=lambda d: concurrent[d])
    groups, cur = [], [order[0]]
    for prev, d in zip(order, order[1:]):
        if concurrent[prev] > 0 and concurrent[d] > gap * concurrent[prev]:
            groups.append(cur)
            cur = []
        cur.append(d)
    groups.append(cur)
    if len(groups) < 2:
        return {}
    return {d: f"g{k}" for k, members in enumerate(groups) for d in members}


def probe_rates(devices: Sequence[int], nbytes: int = 256 << 20, reps: int = 2) -> dict[str, dict[int, float]]:
    """Host -> device GB/s of each GPU alone and of all of them at once
    (median of ``reps`` after one warm-up), with torch copies only."""
    import statistics

    import torch

    devices = [int(d) for d in devices]
    host = {d: torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) for d in devices}
    dev = {d: torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{d}") for d in devices}
    streams = {d: torch.cuda.Stream(device=d) for d in devices}

    def run(group: list[int]) -> dict[int, float]:
        ev = {}
        for d in group:
            with torch.cuda.device(d), torch.cuda.stream(streams[d]):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                dev[d].copy_(host[d], non_blocking=True)
                e1.record()
                ev[d] = (e0, e1)
        for d in group:
            torch.cuda.synchronize(d)
        return {d: nbytes / 1e9 / (e0.elapsed_time(e1) / 1e3) for d, (e0, e1) in ev.items()}

    def measured(group: list[int]) -> dict[int, float]:
        run(group)
        samples = [run(group) for _ in range(max(1, reps))]
        return {d: statistics.median(x[d] for x in samples) for d in group}

    try:
        solo = {}
        for d in devices:
            solo.update(measured([d]))
        return {"solo": solo, "concurrent": measured(devices)}
    finally:
        del host, dev
        torch.cuda.empty_cache()


__all__ = ["contention_groups", "probe_rates"]
