"""Pooled-transfer sweep and per-link probe.

    python -m pcie_pool_b200.benchmarks.pool_sweep --relays 0,1,3,7 \\
        --sizes 4M,64M,1G,8G --chunks 1M,4M,16M,64M --directions h2d,d2h

Moves uniform-random bytes between a page-locked host buffer and GPU0 over
the direct lane plus the first R relay GPUs (equal split, then the
balancer's weights after two calibration transfers), for every size, chunk
size and direction; each point is the median of ``--repeats`` timings and is
verified byte-exactly.  ``ms`` brackets the whole ``PoolEngine.run`` call with
CUDA events on the caller's stream (the Python submit, the engine's work and
the host noticing completion); ``engine_ms`` is the engine's own event pair
around the transfer's device work.  Verification: H2D compares the per-chunk
checksums of the landing kernels with the host checksum, D2H the host buffer
with the device buffer.  ``--solo`` adds one line per GPU with its own link alone
(the isolated-link roofline); the largest size with all lanes gives the
concurrent aggregate.  One JSON line per point.
"""

from __future__ import annotations

import argparse
import json
import statistics


UNITS = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}


def parse_size(s: str) -> int:
    s = s.strip().upper()
    return int(float(s[:-1]) * UNITS[s[-1]]) if s[-1] in UNITS else int(s)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--relays", default="0,1,3,7")
    p.add_argument("--sizes", default="4M,64M,1G,8G")
    p.add_argument("--chunks", default="1M,4M,16M,64M")
    p.add_argument("--directions", default="h2d,d2h")
    p.add_argument("--repeats", type=int, default=3)
    p.add_argument("--solo", action="store_true")
    p.add_argument("--no-verify", action="store_true")
    return p.parse_args(argv)


def main(argv=None) -> int:
    import torch

    from .._native import native
    from ..parallel.balance import LaneBalancer
    from ..parallel.engine import D2H, H2D, PoolEngine
    from ..parallel.planning import plan_lanes
    from ..utils.checksum import combine, rebase_chunk_sums
    from ..utils.host_memory import PinnedHostBuffer
    from .common import fill_random

    a = parse_args(argv)
    C = native()
    ngpu = torch.cuda.device_count()
    sizes = [parse_size(x) for x in a.sizes.split(",") if x]
    chunks = [parse_size(x) for x in a.chunks.split(",") if x]
    relays = [int(x) for x in a.relays.split(",") if x and int(x) < ngpu]
    nmax = max(sizes)
    host = PinnedHostBuffer(nmax, fill=None)
    fill_random(host.numpy(), seed=7)
    dev = torch.empty(nmax, dtype=torch.uint8, device="cuda:0")
    torch.cuda.set_device(0)
    for chunk in chunks:
        eng = PoolEngine(list(range(ngpu)), slot_bytes=chunk, slots=3, ctas_per_lane=4, timeout_s=30.0)
        for r in relays:
            devices = list(range(r + 1))
            for dname in [d for d in a.directions.split(",") if d]:
                direction = H2D if dname == "h2d" else D2H
                bal = LaneBalancer(alpha=0.5)
                for n in sizes:
                    if n < chunk:
                        continue
                    w = bal.weights(0, dname, devices) if r else None
                    lanes = plan_lanes(n, chunk, devices, target=0, bw_gibps=w)
                    for _ in range(2):  # warm-up and lane-weight calibration
                        res = eng.run(direction, 0, host.ptr, n, dev.data_ptr(), n, lanes, checksum=True)
                        res.raise_for_status()
                        if r:
                            bal.observe(0, dname, res)
                            lanes = plan_lanes(n, chunk, devices, target=0, bw_gibps=bal.weights(0, dname, devices))
                    ms, dev_ms = [], []
                    for _ in range(a.repeats):
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                        res = eng.run(direction, 0, host.ptr, n, dev.data_ptr(), n, lanes, checksum=True)
                        e1.record()
                        e1.synchronize()
                        res.raise_for_status()
                        ms.append(e0.elapsed_time(e1))
                        dev_ms.append(res.cuda_ms)
                    ok = None
                    if not a.no_verify:
                        if direction == H2D:
                            want = tuple(int(x) for x in C.checksum_host(host.ptr, n))
                            ok = combine(rebase_chunk_sums(res.checksums, lanes)) == want
                        else:
                            ok = bool(torch.equal(dev[:n].cpu(), torch.from_numpy(host.numpy()[:n])))
                    med = statistics.median(ms)
                    dmed = statistics.median(dev_ms)
                    print(json.dumps({"direction": dname, "relays": r, "lanes": len(devices), "bytes": n,
                                      "chunk_bytes": chunk, "ms": round(med, 3),
                                      "gb_per_s": round(n / 1e9 / (med / 1e3), 2),
                                      "engine_ms": round(dmed, 3),
                                      "engine_gb_per_s": round(n / 1e9 / (dmed / 1e3), 2) if dmed > 0 else None,
                                      "verified": ok,
                                      "lane_ms": [(l.device, round(l.cuda_ms, 2), l.bytes) for l in res.lanes]}),
                          flush=True)
        del eng
    if a.solo:
        n = min(nmax, 2 << 30)
        for g in range(ngpu):
            eng = PoolEngine([g], slot_bytes=32 << 20, slots=3, timeout_s=30.0)
            d = torch.empty(n, dtype=torch.uint8, device=f"cuda:{g}")
            for dname, direction in (("h2d", H2D), ("d2h", D2H)):
                lanes = plan_lanes(n, 32 << 20, [g], target=g)
                eng.run(direction, g, host.ptr, n, d.data_ptr(), n, lanes).raise_for_status()
                r = eng.run(direction, g, host.ptr, n, d.data_ptr(), n, lanes)
                r.raise_for_status()
                print(json.dumps({"solo_gpu": g, "direction": dname, "gb_per_s": round(r.gb_per_s, 2)}), flush=True)
            del eng, d
    host.release()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
