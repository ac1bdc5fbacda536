"""Landing-kernel throughput with the source already in HBM.

``python -m pcie_pool_b200.benchmarks.land_kernel --bytes 1073741824``
times the fused landing kernel (TMA bulk global->shared->global with the
per-chunk checksum) on one GPU, with no PCIe or NVLink leg, so the kernel is
measured against the HBM copy roofline: bytes read + bytes written per
second.  Buffers are larger than L2 by default; each timed launch reads a
different source/destination pair (two pairs alternate) so L2 cannot carry
data between iterations.  One JSON line per configuration.
"""

from __future__ import annotations

import argparse
import json
import pathlib

import torch

from ..ops import noalloc


def _peak_hbm() -> float | None:
    p = pathlib.Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return None


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--bytes", type=int, default=1 << 30)
    ap.add_argument("--chunk", type=int, default=16 << 20)
    ap.add_argument("--ctas", default="4,16,74,148")
    ap.add_argument("--op", choices=["copy", "scatter"], default="copy")
    ap.add_argument("--unit", type=int, default=32 << 10, help="scatter unit bytes (a paged-KV block lane)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-checksum", action="store_true")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    noalloc.setup(0)
    n = a.bytes
    srcs = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev) for _ in range(2)]
    dsts = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(2)]
    tables = [None, None]
    if a.op == "scatter":
        units = n // a.unit
        for i in range(2):
            perm = torch.randperm(units, device=dev)
            tables[i] = dsts[i].data_ptr() + perm.to(torch.int64) * a.unit
    peak = _peak_hbm()
    for ctas in [int(x) for x in a.ctas.split(",")]:
        def launch(i):
            noalloc.land(srcs[i % 2], None if a.op == "scatter" else dsts[i % 2], chunk_bytes=a.chunk, ctas=ctas,
                         unit_addrs=tables[i % 2], unit_bytes=a.unit if a.op == "scatter" else 0,
                         checksum=not a.no_checksum)
        for i in range(a.warmup):
            launch(i)
        status, _ = noalloc.result(0, 0)
        if status[0] != 0:
            raise RuntimeError(f"landing kernel status {status}")
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for i in range(a.iters):
            launch(i)
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / a.iters
        status, _ = noalloc.result(0, 0)
        gbs = 2 * n / (ms / 1e3) / 1e9
        print(json.dumps({"kernel": "land_kernel", "op": a.op, "bytes": n, "chunk": a.chunk, "ctas": ctas,
                          "checksum": not a.no_checksum, "ms": round(ms, 4), "rw_gb_per_s": round(gbs, 1),
                          "frac_of_measured_hbm": None if peak is None else round(gbs / peak, 3),
                          "status": status[0]}), flush=True)


if __name__ == "__main__":
    main()
