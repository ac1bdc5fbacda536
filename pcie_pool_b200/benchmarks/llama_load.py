"""Llama-3-8B-shape weight load into GPU0 (BASELINE configs 3a / 3b).

    python -m pcie_pool_b200.benchmarks.llama_load --gpus 8 --variant bf16
    python -m pcie_pool_b200.benchmarks.llama_load --gpus 8 --variant fp8
    python -m pcie_pool_b200.benchmarks.llama_load --gpus 8 --variant bf16 --impl reference

The packed host image (8,030,261,248 bf16 parameters, N(0, 0.02), 16.06 GB,
page-locked) is loaded into GPU0 over the direct lane plus ``gpus-1`` relay
lanes.  ``bf16`` lands the image as-is (plain copy, per-chunk checksums);
``fp8`` lands every matrix as e4m3 codes with fp32 scales per 128x128 block,
quantized inside the landing kernel, and the 1-D norm weights as bf16.
``--api`` also times the bf16 load through the public API
(``ModelWeightLoader`` -> ``TurboBusClient`` -> daemon -> executor -> engine).
Each timed load is bracketed by CUDA events on GPU0 after warm-up loads; the
reported ``value`` is seconds per load (lower is better).  ``--impl
reference`` loads the same image through the reference's own runtime and
planner (bf16 only: the reference has no quantizing landing).
"""

from __future__ import annotations

import argparse
import time

import numpy as np

from .common import ClockSampler, calibrate, emit, reference_plan, reference_runtime


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--variant", choices=["bf16", "fp8"], default="bf16")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--chunk", type=int, default=16 << 20)
    p.add_argument("--api", action="store_true", help="also time the bf16 load through the public API")
    p.add_argument("--via", choices=["engine", "daemon"], default="engine",
                   help="ours: drive the engine directly, or submit each load as a daemon intent "
                        "(fp8: landing spec with the tensor table; relays from leases)")
    p.add_argument("--layers", type=int, default=0, help="override the layer count (smaller smoke runs)")
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


def _manifest(layers: int):
    from dataclasses import replace

    from ..models.llama import llama3_8b, weight_manifest

    cfg = llama3_8b()
    if layers:
        cfg = replace(cfg, layers=int(layers), name=f"llama-3-8b-shape-{layers}L")
    return weight_manifest(cfg)


def _host_image(manifest):
    from .._native import native
    from ..utils.host_memory import PinnedHostBuffer

    host = PinnedHostBuffer(manifest.total_bytes, fill=None)
    native().fill_normal_bf16(host.ptr, manifest.total_bytes // 2, 0.0, 0.02, 20240601, 0)
    return host


def _verify_bf16(host, res, lanes, total) -> bool:
    from .._native import native
    from ..utils.checksum import combine, rebase_chunk_sums

    want = tuple(int(x) for x in native().checksum_host(host.ptr, total))
    return combine(rebase_chunk_sums(res.checksums, lanes)) == want


def _verify_fp8(host, manifest, loaded) -> bool:
    import torch

    from ..utils.fp8 import block_quant

    raw = host.numpy()
    ok = True
    pick = [t for t in manifest.matrices() if ".k_proj." in t.name][:1] + manifest.matrices()[-1:]
    for t in pick:
        rows, cols = t.shape
        w = raw[t.offset:t.offset + t.nbytes].view(np.uint16).reshape(rows, cols)
        f = torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16).float().numpy()
        if rows > 4096:  # the vocab matrices: check the first 2048 rows (16 row-blocks)
            f = f[:2048]
        q_ref, s_ref = block_quant(f)
        q = loaded.tensors[t.name][:f.shape[0]].cpu().numpy()
        s = loaded.scales[t.name][:s_ref.shape[0]].cpu().numpy()
        ok &= bool(np.array_equal(q, q_ref)) and bool(np.array_equal(s, s_ref))
    for t in manifest.vectors()[:3]:
        got = loaded.tensors[t.name].view(torch.int16).cpu().numpy().view(np.uint16)
        ok &= bool(np.array_equal(got, raw[t.offset:t.offset + t.nbytes].view(np.uint16)))
    return ok


def run_ours(a) -> dict:
    import torch

    from ..models.loader import PooledWeightLoader
    from ..parallel.engine import PoolEngine

    manifest = _manifest(a.layers)
    total = manifest.total_bytes
    devices = list(getattr(a, "devices", None) or range(a.gpus))
    torch.cuda.set_device(0)
    host = _host_image(manifest)
    eng = PoolEngine(devices, slot_bytes=a.chunk, slots=3, ctas_per_lane=4, timeout_s=30.0)
    lane_set, weights, balancer, profile = calibrate(eng, 0, devices, total, a.chunk)
    relays = [d for d in lane_set if d != 0]
    loader = PooledWeightLoader(eng, 0, relays, chunk_bytes=a.chunk, balancer=balancer)
    dst = torch.empty(total, dtype=torch.uint8, device="cuda:0") if a.variant == "bf16" else None
    if a.via == "daemon":
        from .. import TurboBusClient
        from ..e2e import build_inprocess_node, nominal_profile
        from ..models.loader import DaemonWeightLoader

        prof = profile if profile is not None else (nominal_profile(0, relays) if relays else None)
        _daemon, dc = build_inprocess_node(eng, list(lane_set), 0, prof)
        sid = dc.register_session(0, relays, max_inflight_chunks=1 << 16).payload["session"]["session_id"]
        dc.register_job("llama-load", session_id=sid)
        dloader = DaemonWeightLoader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="llama-load", target=0,
                                     chunk_bytes=a.chunk)
        host_t = torch.from_numpy(host.numpy())  # the same page-locked image, as a tensor

    def load():
        if a.via == "daemon":
            if a.variant == "bf16":
                return dloader.load_bf16(host_t, manifest, device_buffer=dst)
            return dloader.load_fp8(host_t, manifest)
        if a.variant == "bf16":
            return loader.load_bf16(host.ptr, total, manifest, device_buffer=dst)
        return loader.load_fp8(host.ptr, total, manifest)

    for _ in range(a.warmup):
        last = load()
    torch.cuda.synchronize()
    clocks = ClockSampler(a.gpus).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(a.steps):
        last = load()
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / a.steps
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / a.steps
    if a.variant == "bf16":
        # one more load with its lanes kept: the per-chunk checksums, re-based
        # onto the image, must equal the host checksum of the whole image
        from ..parallel.engine import H2D

        lanes = loader.bf16_lanes(total)
        r = eng.run(H2D, 0, host.ptr, total, dst.data_ptr(), total, lanes, checksum=True)
        verified = r.ok and _verify_bf16(host, r, lanes, total)
    else:
        verified = _verify_fp8(host, manifest, last)
    out = {"ms": ms, "wall_ms": wall * 1e3, "verified": verified, "clocks": clk, "bytes": total,
           "lane_set": lane_set, "lanes": last.stats.lanes, "transfers_per_load": last.stats.transfers,
           "probe": None if profile is None else profile.get("concurrent")}
    if a.api and a.variant == "bf16":
        out["api"] = _api_load(a, eng, host, dst, manifest, profile)
    del last, dst
    host.release()
    return out


def _api_load(a, eng, host, dst, manifest, profile) -> dict:
    """bf16 load through ModelWeightLoader on an in-process daemon."""
    import torch

    from ..adapters import AdapterTransferContext, ModelWeightLoader
    from ..api import TurboBusClient
    from ..e2e import build_inprocess_node
    from ..schema import WorkloadKind

    total = manifest.total_bytes
    devices = list(getattr(a, "devices", None) or range(a.gpus))
    _daemon, dc = build_inprocess_node(eng, devices, 0, profile)
    sid = dc.register_session(0, devices[1:], max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    dc.register_job("llama-load", session_id=sid)
    dc.register_buffer("weights-host", "llama-load", "cpu_pinned", total, address=host.ptr, pinned=True)
    dc.register_buffer("weights-gpu0", "llama-load", "gpu", total, device_index=0, address=dst.data_ptr())

    def ctx(i):  # a fresh intent prefix per load: intent ids are idempotent in the daemon
        return AdapterTransferContext("llama-load", sid, "weights-host", "weights-gpu0",
                                      workload_kind=WorkloadKind.MODEL_WEIGHTS, metadata={"chunk_bytes": a.chunk},
                                      intent_prefix=f"llama-load-{i}", wait_timeout_seconds=600)

    class _Mem:  # byte-count stand-in for the packed image (the loader reads offsets only)
        def __init__(self, n):
            self.n = n

        def numel(self):
            return self.n

        def element_size(self):
            return 1

    bucket = 512 << 20
    count = (total + bucket - 1) // bucket

    def load(i):
        ld = ModelWeightLoader(TurboBusClient(daemon=dc), ctx(i))
        hb, rest = _Mem(total), total
        for k in range(count):
            n = min(bucket, rest)
            ld.add_bucket(f"w{k}", hb, hb, bucket_id=k, cpu_offset=k * bucket, gpu_offset=k * bucket, byte_count=n)
            rest -= n
        ld.load_all()
        ld.wait_all()
        return ld

    load(0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(a.steps):
        ld = load(i + 1)
    torch.cuda.synchronize()
    s = (time.perf_counter() - t0) / a.steps
    st = ld.transfer_stats_many(ld.names())
    return {"load_s": round(s, 4), "gb_per_s": round(total / 1e9 / s, 3), "buckets": count,
            "direct_chunks": st.direct_chunks, "relay_chunks": st.relay_chunks,
            "path": "ModelWeightLoader -> TurboBusClient -> daemon -> executor -> PoolEngine"}


def run_reference(a) -> dict:
    import torch

    if a.variant != "bf16":
        return {"unavailable": "the reference has no quantizing landing path (bf16 only)"}
    manifest = _manifest(a.layers)
    total = manifest.total_bytes
    torch.cuda.set_device(0)
    rt, why = reference_runtime(a.gpus, a.chunk)
    if rt is None:
        return {"unavailable": why}
    host_t = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    # random-init image made with torch only: nothing of this project's
    # native code runs on the reference's path
    g = torch.Generator(device="cuda:0").manual_seed(20240601)
    step = 1 << 30
    for o in range(0, total, step):
        n = min(step, total - o)
        w = torch.randn(n // 2, device="cuda:0", generator=g, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)
        host_t[o:o + n].copy_(w.view(torch.uint8))
    del w
    dst = torch.empty(total, dtype=torch.uint8, device="cuda:0")
    nplan, _profile = reference_plan(rt, total, a.chunk)

    def load():
        h = rt.fetch_plan_to_gpu(host_t.data_ptr(), total, dst.data_ptr(), total, nplan)
        rt.wait(h)

    for _ in range(a.warmup):
        load()
    torch.cuda.synchronize()
    clocks = ClockSampler(a.gpus).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        load()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / a.steps
    verified = bool(torch.equal(dst[:1 << 24].cpu(), host_t[:1 << 24])) and bool(
        torch.equal(dst[-(1 << 24):].cpu(), host_t[-(1 << 24):]))
    del rt
    return {"ms": ms, "verified": verified, "clocks": clk, "bytes": total}


def main(argv=None) -> int:
    a = parse_args(argv)
    res = run_reference(a) if a.impl == "reference" else run_ours(a)
    if "unavailable" in res:
        emit({"impl": a.impl, "unavailable": res["unavailable"]}, a.json_out)
        return 0
    ms = res["ms"]
    line = {"metric": "Llama-3-8B-shape weight load into GPU0", "value": round(ms / 1e3, 4), "unit": "s",
            "higher_is_better": False, "gb_per_s": round(res["bytes"] / 1e9 / (ms / 1e3), 3),
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "impl": a.impl, "variant": a.variant,
            "via": a.via if a.impl == "ours" else "reference runtime",
            "verified": res.get("verified"), "clocks": res.get("clocks"),
            "config": {"model": _manifest(a.layers).config.name, "params": _manifest(a.layers).param_count,
                       "image_bytes": res["bytes"], "chunk_bytes": a.chunk, "target_gpu": 0,
                       "relay_gpus": list(range(1, a.gpus)),
                       "landing": "bf16 copy" if a.variant == "bf16" else "fp8 e4m3 + fp32 128x128 scales",
                       "data": "synthetic bf16 N(0, 0.02), seeded"}}
    for k in ("wall_ms", "lane_set", "lanes", "transfers_per_load", "probe", "api"):
        if k in res:
            line[k] = res[k]
    emit(line, a.json_out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
