"""Standalone sm_100a op kernels on one GPU, against the HBM copy roofline.

    python -m pcie_pool_b200.benchmarks.op_kernels --kernels adamw,gather,scatter,pack,unpack,fp8,checksum

Each kernel runs on buffers larger than the 126 MB L2 (two input sets
alternate between iterations, so L2 carries nothing over), is timed with CUDA
events on its stream after warm-up, and reports the bytes it must move
(algorithmic traffic: every operand read once and every result written
once), GB/s and the fraction of the measured HBM copy bandwidth
(``MEASURED_PEAKS.json``).  The same command with a small ``--bytes`` is the
case to capture under ncu (``-k regex:<kernel>_kernel``).

Kernels (``pcie_pool_b200.ops``):

* ``adamw``     fused AdamW over fp32 master/m/v and bf16 grads, writing bf16
                params: reads 3x4 + 2 and writes 3x4 + 2 bytes per element;
* ``gather``    paged-KV gather: permuted fixed-size units into one packed
                buffer (read + write every byte);
* ``scatter``   the inverse, into a permuted block table;
* ``pack`` / ``unpack``  variable-size ranges to / from one packed buffer;
* ``fp8``       bf16 -> e4m3 with fp32 scales per 128x128 block (reads 2,
                writes 1 byte per element plus the scales);
* ``checksum``  the per-chunk checksum reduction (reads every byte once).
"""

from __future__ import annotations

import argparse
import json
import pathlib

KERNELS = ("adamw", "gather", "scatter", "pack", "unpack", "fp8", "checksum")


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--kernels", default=",".join(KERNELS))
    p.add_argument("--bytes", type=int, default=1 << 30, help="size of the main operand (bytes)")
    p.add_argument("--unit", type=int, default=32 << 10, help="gather/scatter unit bytes (one KV block lane)")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args(argv)
    a.kernel_list = [k for k in a.kernels.split(",") if k]
    bad = [k for k in a.kernel_list if k not in KERNELS]
    if bad:
        p.error(f"unknown kernels: {bad}")
    return a


def traffic_bytes(kernel: str, nbytes: int) -> int:
    """Algorithmic bytes one launch must move for a main operand of ``nbytes``."""
    if kernel == "adamw":
        n = nbytes // 4  # elements of the fp32 master copy
        return n * (4 * 3 + 2) + n * (4 * 3 + 2)
    if kernel == "fp8":
        n = nbytes // 2  # bf16 elements
        return 2 * n + n + 4 * (n // (128 * 128))
    if kernel == "checksum":
        return nbytes
    return 2 * nbytes  # gather / scatter / pack / unpack: read and write every byte


def _peak_hbm() -> float | None:
    p = pathlib.Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return None


def main(argv=None) -> int:
    import torch

    from .. import ops

    a = parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    n = int(a.bytes)
    peak = _peak_hbm()

    def two(make):
        return [make() for _ in range(2)]

    runs = {}
    if "adamw" in a.kernel_list:
        e = n // 4
        sets = two(lambda: (torch.randn(e, device=dev, generator=g), torch.zeros(e, device=dev),
                            torch.zeros(e, device=dev), torch.randn(e, device=dev, generator=g).bfloat16(),
                            torch.empty(e, dtype=torch.bfloat16, device=dev)))
        runs["adamw"] = lambda i: ops.fused_adamw(*sets[i % 2][:4], sets[i % 2][4], lr=1e-3, step=i + 1)
    if any(k in a.kernel_list for k in ("gather", "scatter", "pack", "unpack")):
        units = n // a.unit
        pools = two(lambda: torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g))
        flat = two(lambda: torch.empty(n, dtype=torch.uint8, device=dev))
        tables = [ops.unit_addresses(pools[i], a.unit, torch.randperm(units, device=dev, generator=g).cpu().numpy())
                  for i in range(2)]
        runs["gather"] = lambda i: ops.gather_units(tables[i % 2], a.unit, flat[i % 2])
        runs["scatter"] = lambda i: ops.scatter_units(flat[i % 2], tables[i % 2], a.unit)
        # ranges: two-unit pieces at permuted places (the range kernels take any sizes)
        sizes = torch.full((units // 2,), 2 * a.unit, dtype=torch.int64, device=dev)
        raddr = [ops.unit_addresses(pools[i], 2 * a.unit, torch.randperm(units // 2, device=dev,
                                                                         generator=g).cpu().numpy())
                 for i in range(2)]
        runs["pack"] = lambda i: ops.pack_ranges(raddr[i % 2], sizes, flat[i % 2])
        runs["unpack"] = lambda i: ops.unpack_ranges(flat[i % 2], raddr[i % 2], sizes)
    if "fp8" in a.kernel_list:
        side = int((n // 2) ** 0.5) // 128 * 128
        xs = two(lambda: torch.randn(side, side, device=dev, generator=g).bfloat16())
        runs["fp8"] = lambda i: ops.fp8_block_quant(xs[i % 2])
    if "checksum" in a.kernel_list:
        from .._native import native

        bufs = two(lambda: torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g))
        sums = torch.zeros(2, dtype=torch.int64, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        # the device reduction alone (ops.checksum also reads the result back to the host)
        runs["checksum"] = lambda i: native().checksum_device(bufs[i % 2].data_ptr(), n, sums.data_ptr(), stream)
    for k in a.kernel_list:
        fn = runs[k]
        for i in range(a.warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(a.iters):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / a.iters
        size = n if k != "fp8" else int((int((n // 2) ** 0.5) // 128 * 128) ** 2 * 2)
        gbs = traffic_bytes(k, size) / 1e9 / (ms / 1e3)
        print(json.dumps({"kernel": k, "bytes": size, "ms": round(ms, 4), "gb_per_s": round(gbs, 1),
                          "frac_of_measured_hbm": None if peak is None else round(gbs / peak, 3)}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
