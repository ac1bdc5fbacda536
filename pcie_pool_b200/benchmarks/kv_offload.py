"""Paged-KV offload and reload latency on GPU0.

    python -m pcie_pool_b200.benchmarks.kv_offload --gpus 8
    python -m pcie_pool_b200.benchmarks.kv_offload --gpus 8 --impl reference

Llama-3-8B KV shapes: 32 layers, each a vLLM cache tensor
``[2, num_blocks, 16, 8, 128]`` bf16 N(0, 1) (one block-lane = 32 KiB, one
32k-token request = 2048 blocks x 2 lanes x 32 layers = 4 GiB).  Eight
requests are offloaded from a seeded random block table into page-locked
host memory (one region per request, CPU layout ``[layer][K/V][block]``),
then reloaded into a second, disjoint random block table.  Each request is
ONE pooled transfer (direct + relay lanes): the push kernel gathers through
the block table on offload and the landing kernel scatters through it on
reload.  Latency per request is timed with CUDA events around the call after
warm-up; ``value`` is the reload p50 in ms.  After the timed reloads every
request's blocks are compared with their source blocks on the device.

``--impl reference`` moves the same bytes through the reference's own
runtime with a plan from its planner: every (layer, lane, block) unit is a
32 KiB range (a permuted table coalesces nothing), i.e. 131,072 chunks per
request, each a separate copy.
"""

from __future__ import annotations

import argparse
import statistics
import time

import numpy as np

from .common import ClockSampler, calibrate, emit, reference_runtime

LAYERS, KV_HEADS, HEAD_DIM, BLOCK = 32, 8, 128, 16


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--requests", type=int, default=8)
    p.add_argument("--tokens", type=int, default=32768)
    p.add_argument("--layers", type=int, default=LAYERS)
    p.add_argument("--steps", type=int, default=2, help="timed passes over all requests")
    p.add_argument("--warmup", type=int, default=1, help="untimed passes over all requests")
    p.add_argument("--chunk", type=int, default=4 << 20, help="bytes per pooled chunk (whole block-lanes)")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--via", choices=["engine", "daemon"], default="engine",
                   help="ours: drive the engine directly, or submit every save / restore as a daemon intent "
                        "(fused gather / scatter landing spec, relays from leases)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


class KVWorld:
    def __init__(self, a):
        import torch

        self.blocks_per_req = (a.tokens + BLOCK - 1) // BLOCK
        need = a.requests * self.blocks_per_req
        self.num_blocks = 2 * need
        self.layers = a.layers
        shape = (a.layers, 2, self.num_blocks, BLOCK, KV_HEADS, HEAD_DIM)
        self.kv = torch.empty(shape, dtype=torch.bfloat16, device="cuda:0")
        g = torch.Generator(device="cuda:0").manual_seed(a.seed)
        for l in range(a.layers):
            self.kv[l].normal_(0.0, 1.0, generator=g)
        self.caches = [self.kv[l] for l in range(a.layers)]
        perm = np.random.default_rng(a.seed).permutation(self.num_blocks)
        self.src = [perm[r * self.blocks_per_req:(r + 1) * self.blocks_per_req] for r in range(a.requests)]
        self.dst = [perm[need + r * self.blocks_per_req:need + (r + 1) * self.blocks_per_req]
                    for r in range(a.requests)]
        self.unit = BLOCK * KV_HEADS * HEAD_DIM * 2
        self.req_bytes = a.layers * 2 * self.blocks_per_req * self.unit

    def verify(self) -> bool:
        import torch

        ok = True
        for s, d in zip(self.src, self.dst):
            si = torch.as_tensor(s, device="cuda:0")
            di = torch.as_tensor(d, device="cuda:0")
            for l in range(self.layers):
                ok &= bool(torch.equal(self.kv[l].index_select(1, si), self.kv[l].index_select(1, di)))
        return ok


def _timed(fn):
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1)


def run_ours(a) -> dict:
    import torch

    from ..adapters.kv_offload import PagedKVOffloader
    from ..parallel.engine import PoolEngine
    from ..utils.host_memory import PinnedHostBuffer

    torch.cuda.set_device(0)
    w = KVWorld(a)
    devices = list(getattr(a, "devices", None) or range(a.gpus))
    eng = PoolEngine(devices, slot_bytes=a.chunk, slots=3, ctas_per_lane=4, timeout_s=30.0)
    lane_set, _weights, balancer, profile = calibrate(eng, 0, devices, w.req_bytes, a.chunk)
    relays = [d for d in lane_set if d != 0]
    if a.via == "daemon":
        from .. import TurboBusClient
        from ..adapters.kv_offload import DaemonKVOffloader
        from ..e2e import build_inprocess_node, nominal_profile

        prof = profile if profile is not None else (nominal_profile(0, relays) if relays else None)
        _daemon, dc = build_inprocess_node(eng, list(lane_set), 0, prof)
        sid = dc.register_session(0, relays, max_inflight_chunks=1 << 16).payload["session"]["session_id"]
        dc.register_job("kv-bench", session_id=sid)
        off = DaemonKVOffloader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="kv-bench",
                                kv_caches=w.caches, units_per_chunk=a.chunk // w.unit)
        hosts = [torch.empty(w.req_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(a.requests)]
        save = lambda r: off.save(list(w.src[r]), hosts[r])  # noqa: E731
        load = lambda r: off.restore(list(w.dst[r]), hosts[r])  # noqa: E731
    else:
        off = PagedKVOffloader(eng, w.caches, 0, relays, units_per_chunk=a.chunk // w.unit, checksum=True,
                               balancer=balancer)
        hosts = [PinnedHostBuffer(w.req_bytes, fill=None) for _ in range(a.requests)]
        save = lambda r: off.save(list(w.src[r]), hosts[r].ptr, w.req_bytes)  # noqa: E731
        load = lambda r: off.restore(list(w.dst[r]), hosts[r].ptr, w.req_bytes)  # noqa: E731
    save_ms, load_ms, save_dev, load_dev = [], [], [], []
    try:
        for _ in range(a.warmup):
            for r in range(a.requests):
                save(r)
                load(r)
        torch.cuda.synchronize()
        clocks = ClockSampler(a.gpus).start()
        for _ in range(a.steps):
            for r in range(a.requests):
                st = {}
                save_ms.append(_timed(lambda: st.setdefault("s", save(r))))
                save_dev.append(st["s"].cuda_ms)
            for r in range(a.requests):
                st = {}
                load_ms.append(_timed(lambda: st.setdefault("l", load(r))))
                load_dev.append(st["l"].cuda_ms)
        clk = clocks.stop()
        verified = w.verify()
        last_lanes = st["l"].lanes
    finally:
        for h in hosts:
            if hasattr(h, "release"):
                h.release()
    return {"reload_ms": load_ms, "offload_ms": save_ms, "reload_dev_ms": load_dev, "offload_dev_ms": save_dev,
            "verified": verified, "clocks": clk, "lane_set": lane_set, "lanes": last_lanes,
            "req_bytes": w.req_bytes, "units_per_request": w.req_bytes // w.unit,
            "probe": None if profile is None else profile.get("concurrent")}


def run_reference(a) -> dict:
    import torch

    torch.cuda.set_device(0)
    rt, why = reference_runtime(a.gpus, 32 << 10)
    if rt is None:
        return {"unavailable": why}
    from turbobus import runtime_engine
    from turbobus.planner_engine import PlannerEngine

    w = KVWorld(a)
    base = w.kv.data_ptr()
    dev_bytes = w.kv.numel() * 2
    profile = rt.profile(256 << 20, False)
    eng = PlannerEngine()
    hosts = [torch.empty(w.req_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(a.requests)]
    stride_l = w.kv.stride(0) * 2
    stride_lane = w.kv.stride(1) * 2

    def ranges(ids, h2d: bool):
        out, hoff = [], 0
        for l in range(a.layers):
            for lane in range(2):
                for b in ids:
                    d = l * stride_l + lane * stride_lane + int(b) * w.unit
                    out.append((hoff, d, w.unit) if h2d else (d, hoff, w.unit))
                    hoff += w.unit
        return out

    plans = {}

    def plan(r, h2d):
        key = (r, h2d)
        if key not in plans:
            rs = ranges(w.dst[r] if h2d else w.src[r], h2d)
            p = eng.plan_ranges(rs, w.unit, profile, "pool", direction="h2d" if h2d else "d2h")
            plans[key] = runtime_engine._native_transfer_plan(p)
        return plans[key]

    def save(r):
        h = rt.offload_plan_to_cpu(base, dev_bytes, hosts[r].data_ptr(), w.req_bytes, plan(r, False))
        rt.wait(h)

    def load(r):
        h = rt.fetch_plan_to_gpu(hosts[r].data_ptr(), w.req_bytes, base, dev_bytes, plan(r, True))
        rt.wait(h)

    for _ in range(a.warmup):
        for r in range(a.requests):
            save(r)
            load(r)
    torch.cuda.synchronize()
    clocks = ClockSampler(a.gpus).start()
    save_ms, load_ms = [], []
    for _ in range(a.steps):
        for r in range(a.requests):
            save_ms.append(_timed(lambda: save(r)))
        for r in range(a.requests):
            load_ms.append(_timed(lambda: load(r)))
    clk = clocks.stop()
    verified = w.verify()
    del rt
    return {"reload_ms": load_ms, "offload_ms": save_ms, "verified": verified, "clocks": clk,
            "req_bytes": w.req_bytes, "units_per_request": w.req_bytes // w.unit,
            "reference_chunks_per_request": w.req_bytes // w.unit}


def _pct(xs, q):
    xs = sorted(xs)
    if not xs:
        return None
    k = (len(xs) - 1) * q
    lo, hi = int(np.floor(k)), int(np.ceil(k))
    return xs[lo] + (xs[hi] - xs[lo]) * (k - lo)


def main(argv=None) -> int:
    a = parse_args(argv)
    t0 = time.perf_counter()
    res = run_reference(a) if a.impl == "reference" else run_ours(a)
    if "unavailable" in res:
        emit({"impl": a.impl, "unavailable": res["unavailable"]}, a.json_out)
        return 0
    p50 = _pct(res["reload_ms"], 0.5)
    line = {"metric": "vLLM KV reload p50 (per 32k-token request, permuted block table)", "value": round(p50, 3),
            "unit": "ms", "higher_is_better": False, "n_gpus": a.gpus, "impl": a.impl,
            "via": a.via if a.impl == "ours" else "reference runtime",
            "reload_p50_ms": round(p50, 3), "reload_p99_ms": round(_pct(res["reload_ms"], 0.99), 3),
            "offload_p50_ms": round(_pct(res["offload_ms"], 0.5), 3),
            "offload_p99_ms": round(_pct(res["offload_ms"], 0.99), 3),
            "reload_gb_per_s_p50": round(res["req_bytes"] / 1e9 / (p50 / 1e3), 3),
            "samples": len(res["reload_ms"]), "verified": res["verified"], "clocks": res["clocks"],
            "config": {"model": "Llama-3-8B KV (32 layers, 8 KV heads, head_dim 128, bf16, block 16)",
                       "layers": a.layers, "requests": a.requests, "tokens_per_request": a.tokens,
                       "bytes_per_request": res["req_bytes"], "units_per_request": res["units_per_request"],
                       "chunk_bytes": a.chunk, "target_gpu": 0, "relay_gpus": list(range(1, a.gpus)),
                       "data": "synthetic bf16 N(0,1), seeded permuted block tables"},
            "wall_s": round(time.perf_counter() - t0, 1)}
    for k in ("reload_dev_ms", "offload_dev_ms"):
        if k in res:
            line[k.replace("_ms", "_p50_ms")] = round(statistics.median(res[k]), 3)
    for k in ("lane_set", "lanes", "probe", "reference_chunks_per_request"):
        if k in res:
            line[k] = res[k]
    emit(line, a.json_out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
