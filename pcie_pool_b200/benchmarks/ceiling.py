"""The host's PCIe ceiling, measured without this framework's engine.

    python -m pcie_pool_b200.benchmarks.ceiling --gpus 1,2,4,8 --bytes 1G

Each GPU of a set copies ``--bytes`` between its own page-locked host buffer
and its own memory with one plain ``cudaMemcpyAsync`` per repetition on its
own stream -- no relay, no kernel, no staging -- all GPUs of the set at
once, H2D and then D2H.  The host buffers are placed on one NUMA node
(``node0``, ``node1``, ...) or interleaved over all nodes (``mbind`` before
the pages are touched, then ``cudaHostRegister``), so the figures show what
the host's memory and root complexes deliver to that many links at once.
GPU sets are the first N of the daemon's uplink-spread order (GPU0, then
relays spread over sockets, root complexes and switches) and, with
``--orders index,spread``, also GPUs 0..N-1.

Per set: each GPU's rate from CUDA events on its own stream, and the
aggregate = all bytes / the slowest GPU's time.  Pooled H2D into one GPU can
approach the aggregate of its lane set but not exceed it, so this is the
ceiling the pooled bench value is compared with, next to the sum of
isolated link rates.  One JSON line per (order, N, placement, direction).
"""

from __future__ import annotations

import argparse
import ctypes
import glob
import json
import mmap
import os

UNITS = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
MPOL_BIND, MPOL_INTERLEAVE = 2, 3
SYS_MBIND = 237  # x86_64


def parse_size(s: str) -> int:
    s = str(s).strip().upper()
    return int(float(s[:-1]) * UNITS[s[-1]]) if s and s[-1] in UNITS else int(s)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", default="1,2,4,8", help="GPU-set sizes")
    p.add_argument("--bytes", default="1G", help="bytes per GPU per repetition")
    p.add_argument("--reps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--placements", default="auto", help="node0,node1,...,interleave or auto (all of them)")
    p.add_argument("--orders", default="spread", help="spread and/or index")
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


def numa_nodes() -> list[int]:
    nodes = sorted(int(os.path.basename(p)[4:]) for p in glob.glob("/sys/devices/system/node/node[0-9]*"))
    return nodes or [0]


class HostBuffer:
    """Anonymous memory placed by ``mbind`` before first touch, then
    page-locked for CUDA."""

    def __init__(self, nbytes: int, policy: str, nodes: list[int]) -> None:
        import numpy as np

        from .._native import native

        self.n = nbytes
        self.mm = mmap.mmap(-1, nbytes, flags=mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
        self.arr = np.frombuffer(self.mm, dtype=np.uint8)
        self.ptr = int(self.arr.ctypes.data)
        self.placed = self._mbind(policy, nodes)
        self.arr[::4096] = 1  # fault every page in under the policy
        self.arr[:] = 7
        native().host_register(self.ptr, nbytes)

    def _mbind(self, policy: str, nodes: list[int]) -> str:
        if policy == "default":
            return "first-touch"
        mode = MPOL_INTERLEAVE if policy == "interleave" else MPOL_BIND
        want = nodes if policy == "interleave" else [int(policy[4:])]
        mask = (ctypes.c_ulong * 4)()
        for n in want:
            mask[n // 64] |= 1 << (n % 64)
        libc = ctypes.CDLL(None, use_errno=True)
        rc = libc.syscall(SYS_MBIND, ctypes.c_void_p(self.ptr), ctypes.c_ulong(self.n), ctypes.c_int(mode),
                          mask, ctypes.c_ulong(256 + 1), ctypes.c_uint(0))
        return policy if rc == 0 else f"first-touch (mbind failed: errno {ctypes.get_errno()})"

    def release(self) -> None:
        from .._native import native

        native().host_unregister(self.ptr)
        del self.arr
        self.mm.close()


def run_set(devices, hosts, n: int, reps: int, warmup: int, direction: str) -> dict:
    import torch

    dev_bufs, streams = {}, {}
    for d in devices:
        dev_bufs[d] = torch.empty(n, dtype=torch.uint8, device=f"cuda:{d}")
        streams[d] = torch.cuda.Stream(device=d)
    host_t = {d: torch.from_numpy(hosts[d].arr) for d in devices}

    def launch():
        ev = {}
        for d in devices:
            with torch.cuda.device(d), torch.cuda.stream(streams[d]):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    if direction == "h2d":
                        dev_bufs[d].copy_(host_t[d], non_blocking=True)
                    else:
                        host_t[d].copy_(dev_bufs[d], non_blocking=True)
                e1.record()
                ev[d] = (e0, e1)
        for d in devices:
            torch.cuda.synchronize(d)
        return {d: e0.elapsed_time(e1) for d, (e0, e1) in ev.items()}

    for _ in range(warmup):
        launch()
    ms = launch()
    per = {str(d): round(n * reps / 1e9 / (t / 1e3), 2) for d, t in ms.items()}
    slowest = max(ms.values())
    return {"per_gpu_gb_per_s": per, "aggregate_gb_per_s": round(n * reps * len(devices) / 1e9 / (slowest / 1e3), 2),
            "sum_of_per_gpu_gb_per_s": round(sum(per.values()), 2)}


def main(argv=None) -> int:
    import torch

    from ..topology.cuda_nvml import cuda_lane_set

    a = parse_args(argv)
    n = parse_size(a.bytes)
    count = torch.cuda.device_count()
    sizes = [k for k in (int(x) for x in a.gpus.split(",") if x) if k <= count]
    nodes = numa_nodes()
    placements = ([f"node{x}" for x in nodes] + (["interleave"] if len(nodes) > 1 else [])
                  if a.placements == "auto" else [p for p in a.placements.split(",") if p])
    orders = {}
    if "spread" in a.orders:
        orders["spread"] = cuda_lane_set(max(sizes), 0)[0]
    if "index" in a.orders:
        orders["index"] = list(range(max(sizes)))
    out = []
    for place in placements:
        hosts = {d: HostBuffer(n, place, nodes) for d in range(max(sizes))}
        try:
            for oname, order in orders.items():
                for k in sizes:
                    devs = order[:k]
                    for direction in ("h2d", "d2h"):
                        r = run_set(devs, hosts, n, a.reps, a.warmup, direction)
                        rec = {"probe": "pcie ceiling (plain cudaMemcpyAsync per GPU, no engine)", "order": oname,
                               "gpus": devs, "n": k, "placement": place, "placed": hosts[0].placed,
                               "direction": direction, "bytes_per_gpu": n * a.reps, **r}
                        print(json.dumps(rec), flush=True)
                        out.append(rec)
        finally:
            for h in hosts.values():
                h.release()
    if a.json_out:
        with open(a.json_out, "w") as fh:
            json.dump(out, fh, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
