"""The fused lane kernels on one GPU with their data already in HBM.

    python -m pcie_pool_b200.benchmarks.lane_kernels --ops land_copy,land_scatter,land_unpack,land_fp8,land_adamw,push_copy,push_gather,push_pack

Each op runs as an engine transfer on GPU0's direct lane, staged through the
landing ring, in the engine's serialised mode: for a landing op every chunk
is copied into the staging slots first and the landing kernel then runs
alone, reading the slots from HBM; for a push op the push kernel runs alone
(HBM source -> slots) before any copy-out.  So the kernel is measured
without a PCIe leg and without waiting on a copy engine.  Its device time is
taken from its own per-chunk ``%globaltimer`` stamps (first chunk start to
last chunk done), and the algorithmic bytes it must move give GB/s against
the measured HBM copy bandwidth (``MEASURED_PEAKS.json``).  Two transfers
with different buffers alternate, each larger than the 126 MB L2 with the
default size.  The same command with ``--iters 1`` is the case to capture
under ncu (``-k regex:land_kernel`` / ``push_kernel``).

Algorithmic bytes per transfer of ``B`` payload bytes: copy / scatter /
gather / pack / unpack read B and write B; fp8 reads B (bf16) and writes
B/2 codes plus the scales; adamw reads the 12-byte state and the 2-byte
gradient and writes the 12-byte state and the 2-byte parameter per element.
"""

from __future__ import annotations

import argparse
import json
import pathlib

OPS = ("land_copy", "land_scatter", "land_unpack", "land_fp8", "land_adamw", "push_copy", "push_gather",
       "push_pack")


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--ops", default=",".join(OPS))
    p.add_argument("--bytes", type=int, default=256 << 20, help="payload bytes per transfer")
    p.add_argument("--chunk", type=int, default=32 << 20)
    p.add_argument("--unit", type=int, default=32 << 10, help="KV unit (block lane) bytes")
    p.add_argument("--ctas", type=int, default=0, help="CTAs of the lane (0: the engine's direction budget)")
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--no-checksum", action="store_true")
    a = p.parse_args(argv)
    a.op_list = [o for o in a.ops.split(",") if o]
    bad = [o for o in a.op_list if o not in OPS]
    if bad:
        p.error(f"unknown ops: {bad}")
    return a


def traffic(op: str, payload: int) -> int:
    if op == "land_fp8":
        n = payload // 2
        return payload + n + 4 * (n // (128 * 128))
    if op == "land_adamw":
        n = payload // 12
        return payload + 2 * n + payload + 2 * n
    return 2 * payload


def _peak_hbm() -> float | None:
    p = pathlib.Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return None


def main(argv=None) -> int:
    import numpy as np
    import torch

    from .._native import native
    from ..parallel.engine import D2H, H2D, Lane, PoolEngine

    a = parse_args(argv)
    C = native()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    n = a.bytes - a.bytes % max(a.unit, 24576 * 16)
    chunk = a.chunk
    slots = -(-n // chunk)
    eng = PoolEngine([0], slot_bytes=chunk, slots=slots, ctas_per_lane=max(1, a.ctas or 512), timeout_s=20.0)
    peak = _peak_hbm()
    host = [torch.empty(n, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    for h in host:
        h.copy_(torch.randint(0, 256, (n,), dtype=torch.uint8))
    out = []
    for op in a.op_list:
        h2d = op.startswith("land")
        kw: dict = {}
        offs = np.arange(0, n, chunk, dtype=np.uint64)
        sizes = np.minimum(chunk, n - offs).astype(np.uint64)
        unit0 = None
        devbufs = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(2)]
        tables = [None, None]
        if op in ("land_scatter", "push_gather", "land_unpack", "push_pack"):
            units = n // a.unit
            for i in range(2):
                perm = torch.randperm(units, device=dev, generator=g).cpu().numpy().astype(np.uint64)
                tables[i] = np.uint64(devbufs[i].data_ptr()) + perm * np.uint64(a.unit)
            if op in ("land_scatter", "push_gather"):
                kw = {"op": C.OP_SCATTER_UNITS if h2d else C.OP_GATHER_UNITS, "unit_bytes": a.unit}
                unit0 = (offs // np.uint64(a.unit)).astype(np.uint32)
            else:  # ranges: one per unit, at most one 32 KiB tile each
                rb = np.full(units, a.unit, dtype=np.uint32)
                pos_in_chunk = (np.arange(units, dtype=np.uint64) * np.uint64(a.unit)) % np.uint64(chunk)
                kw = {"op": C.OP_SCATTER_RANGES if h2d else C.OP_GATHER_RANGES}
                unit0 = (offs // np.uint64(a.unit)).astype(np.uint32)
        if op == "land_fp8":
            cols = 4096
            rows = n // (2 * cols) // 128 * 128
            n_op = rows * cols * 2
            offs = np.arange(0, n_op, chunk, dtype=np.uint64)
            sizes = np.minimum(chunk, n_op - offs).astype(np.uint64)
            qs = [torch.empty(rows * cols, dtype=torch.uint8, device=dev) for _ in range(2)]
            scs = [torch.empty((rows // 128) * (cols // 128), dtype=torch.float32, device=dev) for _ in range(2)]
            kw = {"op": C.OP_FP8_QUANT}
            unit0 = (offs // np.uint64(2 * cols)).astype(np.uint32)
            tensor = np.zeros(offs.size, dtype=np.uint32)
        if op == "land_adamw":
            tile = int(C.ADAM_TILE_BYTES)
            ntiles = n // tile
            n_op = ntiles * tile
            per = chunk // tile * tile
            offs = np.arange(0, n_op, per, dtype=np.uint64)
            sizes = np.minimum(per, n_op - offs).astype(np.uint64)
            nparams = ntiles * int(C.ADAM_TILE_PARAMS)
            grads = [torch.randn(nparams, device=dev, generator=g).bfloat16() * 1e-3 for _ in range(2)]
            params = [torch.empty(nparams, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            for h in host:  # sane fp32 state: master ~ N(0, 0.02), moments 0
                st = h[:n_op].view(torch.float32).view(ntiles, 3, -1)
                st[:, 0].normal_(0.0, 0.02)
                st[:, 1:].zero_()
            kw = {"op": C.OP_ADAMW}
            unit0 = (offs // np.uint64(tile)).astype(np.uint32)
        payload = int(sizes.sum())

        def run(i):
            extra = dict(kw)
            if tables[i % 2] is not None and "unit_bytes" in kw:
                extra["unit_addrs"] = tables[i % 2]
            if kw.get("op") in (getattr(C, "OP_SCATTER_RANGES"), getattr(C, "OP_GATHER_RANGES")):
                extra["ranges"] = (tables[i % 2], rb, pos_in_chunk)
            if op == "land_fp8":
                extra["tensors"] = [(qs[i % 2].data_ptr(), scs[i % 2].data_ptr(), rows, cols)]
            if op == "land_adamw":
                extra["adam"] = {"grads": grads[i % 2].data_ptr(), "params": params[i % 2].data_ptr(),
                                 "nparams": nparams, "lr": 1e-4, "step": i + 1}
            lane = Lane(0, offs.copy(), offs.copy(), sizes.copy(), unit0=None if unit0 is None else unit0.copy(),
                        tensor=tensor.copy() if op == "land_fp8" else None,
                        count=(sizes // np.uint64(a.unit)).astype(np.uint32)
                        if op in ("land_unpack", "push_pack") else None)
            r = eng.run(H2D if h2d else D2H, 0, host[i % 2].data_ptr(), n, devbufs[i % 2].data_ptr(), n, [lane],
                        checksum=not a.no_checksum and op != "land_adamw", stage_direct=True, serialize=True,
                        trace=True, ctas_per_lane=a.ctas, **extra)
            r.raise_for_status()
            tr = r.trace
            return (float(tr[:, 2].max()) - float(tr[:, 0].min())) / 1e6, int(tr[:, 3].max())

        for i in range(a.warmup):
            run(i)
        torch.cuda.synchronize()
        times, ctas = [], 0
        for i in range(a.iters):
            ms, ctas = run(a.warmup + i)
            times.append(ms)
        ms = float(np.median(times))
        gbs = traffic(op, payload) / 1e9 / (ms / 1e3)
        rec = {"op": op, "payload_bytes": payload, "algorithmic_bytes": traffic(op, payload),
               "kernel_ms_median": round(ms, 4), "gb_per_s": round(gbs, 1), "ctas": ctas,
               "frac_of_measured_hbm": None if peak is None else round(gbs / peak, 3),
               "checksum": not a.no_checksum and op != "land_adamw"}
        print(json.dumps(rec), flush=True)
        out.append(rec)
        del devbufs
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
