"""Multi-tenant training offload under one daemon.

    python -m pcie_pool_b200.benchmarks.multi_tenant_offload --jobs 4 --gpus-per-job 2
    python -m pcie_pool_b200.benchmarks.multi_tenant_offload --jobs 4 --gpus-per-job 2 --impl reference

Four jobs of two GPUs each train a 7B decoder (32 layers, hidden 4096, MLP
11008: 6,738,415,616 parameters) with fp32 master weights and Adam m/v in
host memory.  Each GPU owns half of the parameters (data-parallel shard), so
per step every GPU offloads its bf16 gradient shard (D2H) and loads its
updated bf16 parameter shard (H2D), all jobs at once.  Every transfer is a
``TransferIntent`` submitted through ``TurboBusClient`` to one in-process
daemon that plans it, arbitrates relay leases between the jobs (a GPU whose
link is busy is not lent out; weighted fair share between jobs) and executes
it on one engine.  ``--active-jobs`` runs fewer jobs so idle GPUs can lend
their links.  Reported: step time (wall, all transfers of all active jobs),
per-job time and Jain's fairness index over per-job throughput, relay share,
and the daemon's state afterwards (no reservation or quota may leak).

``--optimizer streamed-adamw`` (ours): every step is the optimizer step
itself -- per GPU shard one AdamW round-trip intent: the fp32 master weights
and Adam moments stream host -> GPU over the direct and leased relay lanes,
the landing kernel updates them with the shard's local bf16 gradients and
writes the bf16 parameters in place, and the state streams back (12 bytes per
parameter each way; adapters/streamed_optimizer.py).  A slice of every shard
is checked against torch.optim.AdamW.

``--impl reference``: the same transfers through the reference's own
runtime, one warm ``Runtime`` per GPU with every other GPU as a relay
candidate and plans from its own planner; there is no arbitration between
the jobs.
"""

from __future__ import annotations

import argparse
import statistics
import threading
import time
from concurrent.futures import ThreadPoolExecutor

from .common import ClockSampler, emit, reference_runtime


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--jobs", type=int, default=4)
    p.add_argument("--gpus-per-job", type=int, default=2)
    p.add_argument("--active-jobs", type=int, default=0, help="jobs that move data (0 = all)")
    p.add_argument("--layers", type=int, default=32, help="decoder layers (32 = the 7B model)")
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--chunk", type=int, default=16 << 20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--optimizer", choices=["none", "streamed-adamw"], default="none",
                   help="ours: run the AdamW step on the offload path instead of plain grads/params moves")
    p.add_argument("--lend-across-groups", action="store_true",
                   help="ours: measure each GPU's rate with every link busy (topology.uplink_probe) and let the "
                        "daemon lend busy GPUs of a faster uplink group to tenants of a slower one")
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


def shard_bytes(a) -> int:
    from dataclasses import replace

    from ..models.llama import decoder_7b, weight_manifest

    cfg = replace(decoder_7b(), layers=a.layers)
    total = weight_manifest(cfg).param_count * 2
    per = total // a.gpus_per_job
    return per - per % 4096


def jain(xs) -> float:
    xs = [float(x) for x in xs if x > 0]
    return (sum(xs) ** 2) / (len(xs) * sum(x * x for x in xs)) if xs else 0.0


class _Host:
    """A page-locked host buffer (torch)."""

    def __init__(self, n: int) -> None:
        import torch

        self.t = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        self.ptr = int(self.t.data_ptr())

    def numpy(self):
        return self.t.numpy()

    def release(self) -> None:
        self.t = None


class Tenants:
    """Host and device buffers of every GPU shard."""

    def __init__(self, a):
        import torch

        # torch only (page-locked tensors, device RNG): both arms use these
        # buffers and nothing of this project's native code may run on the
        # reference's path
        self.n = shard_bytes(a)
        self.gpus = list(range(a.jobs * a.gpus_per_job))
        self.job_of = {g: g // a.gpus_per_job for g in self.gpus}
        self.host_params, self.host_grads, self.dev_params, self.dev_grads = {}, {}, {}, {}
        for g in self.gpus:
            hp = _Host(self.n)
            gen = torch.Generator(device=f"cuda:{g}").manual_seed(1000 + g)
            step = 1 << 30
            for o in range(0, self.n, step):
                k = min(step, self.n - o)
                w = (torch.randn(k // 2, device=f"cuda:{g}", generator=gen) * 0.02).to(torch.bfloat16)
                hp.t[o:o + k].copy_(w.view(torch.uint8))
            self.host_params[g] = hp
            self.host_grads[g] = _Host(self.n)
            self.dev_params[g] = torch.empty(self.n, dtype=torch.uint8, device=f"cuda:{g}")
            dg = torch.empty(self.n // 2, dtype=torch.bfloat16, device=f"cuda:{g}")
            dg.normal_(0.0, 1e-3)
            self.dev_grads[g] = dg.view(torch.uint8)

    def verify(self, g: int) -> bool:
        import torch

        n = 1 << 24
        hp = torch.from_numpy(self.host_params[g].numpy()[:n])
        hg = torch.from_numpy(self.host_grads[g].numpy()[:n])
        return bool(torch.equal(self.dev_params[g][:n].cpu(), hp)) and bool(
            torch.equal(self.dev_grads[g][:n].cpu(), hg))

    def release(self):
        for d in (self.host_params, self.host_grads):
            for h in d.values():
                h.release()


TRANSFER_TIMEOUT_S = 180.0
LINK_GIBPS = 51.6  # one Gen5 x16 link alone (measured 55.4 GB/s)


def shard_job(job: int, gpu: int) -> str:
    """Daemon job of one GPU shard: a daemon job is bound to one session and a
    session to one target GPU, so every shard is its own job; the tenant's
    weight is split between its shards."""
    return f"job{job}-gpu{gpu}"


def setup_tenants(daemon, dc, gpus, job_of, gpus_per_job: int, n: int, addrs) -> dict:
    """Profile, session, job and the four buffers of every GPU shard;
    ``addrs[g] = (host params, host grads, device params, device grads)``."""
    sessions = {}
    for g in gpus:
        relays = [r for r in gpus if r != g]
        daemon.put_profile(g, relays, {
            "target_device": g, "direct_h2d_bw_gbps": LINK_GIBPS, "direct_d2h_bw_gbps": LINK_GIBPS,
            "relays": [{"relay_device": r, "target_device": g, "h2d_bw_gbps": LINK_GIBPS, "d2h_bw_gbps": LINK_GIBPS,
                        "p2p_bw_gbps": 700.0, "effective_bw_gbps": LINK_GIBPS, "effective_d2h_bw_gbps": LINK_GIBPS,
                        "p2p_enabled": True} for r in relays]})
        r = dc.register_session(g, relays, max_inflight_chunks=1 << 16)
        if not r.ok:
            raise RuntimeError(r.error)
        sid = r.payload["session"]["session_id"]
        job = shard_job(job_of[g], g)
        r = dc.register_job(job, user_id=f"tenant{job_of[g]}", session_id=sid, weight=1.0 / gpus_per_job)
        if not r.ok:
            raise RuntimeError(r.error)
        hp, hg, dp, dg = addrs[g]
        for name, kind, dev, addr in ((f"hp{g}", "cpu_pinned", None, hp), (f"hg{g}", "cpu_pinned", None, hg),
                                      (f"dp{g}", "gpu", g, dp), (f"dg{g}", "gpu", g, dg)):
            r = dc.register_buffer(name, job, kind, n, device_index=dev, address=addr, pinned=kind == "cpu_pinned")
            if not r.ok:
                raise RuntimeError(r.error)
        sessions[g] = sid
    return sessions


def run_ours(a) -> dict:
    import torch

    from .. import TransferIntent, TransferStatusState, TurboBusClient
    from ..daemon import EngineDataPlane, InProcessDaemonClient, IntentExecutor, TurboBusDaemon
    from ..parallel.engine import PoolEngine
    from ..topology import StaticTopologyProvider, synthetic_inventory
    from ..topology.cuda_nvml import CudaNvmlTopologyProvider

    T = Tenants(a)
    gpus = T.gpus
    eng = PoolEngine(gpus, slot_bytes=a.chunk, slots=3, ctas_per_lane=4, timeout_s=60.0)
    try:
        prov = CudaNvmlTopologyProvider()
        prov.snapshot()
    except Exception:  # noqa: BLE001 - described node when NVML is absent
        prov = StaticTopologyProvider(synthetic_inventory(len(gpus), source="declared"))
    daemon = TurboBusDaemon(gpus, max_sessions_per_relay=len(gpus), max_inflight_chunks_per_relay=1 << 16,
                            topology_provider=prov,
                            executor=IntentExecutor(EngineDataPlane(engine=eng, checksum=True),
                                                    max_workers=4 * len(gpus)))
    if getattr(a, "lend_across_groups", False):
        from ..topology.uplink_probe import probe_rates

        daemon.set_uplink_rates(probe_rates(gpus)["concurrent"])
    dc = InProcessDaemonClient(daemon)
    sessions = setup_tenants(daemon, dc, gpus, T.job_of, a.gpus_per_job, T.n,
                             {g: (T.host_params[g].ptr, T.host_grads[g].ptr, T.dev_params[g].data_ptr(),
                                  T.dev_grads[g].data_ptr()) for g in gpus})
    client = TurboBusClient(daemon=dc)
    active = gpus[:(a.active_jobs or a.jobs) * a.gpus_per_job]
    rng = ({"src_offset": 0, "dst_offset": 0, "bytes": T.n},)
    if a.optimizer == "streamed-adamw":
        return _run_streamed_adamw(a, T, dc, client, sessions, active, gpus)
    counter = iter(range(1 << 30))
    pool = ThreadPoolExecutor(max_workers=2 * len(active))

    def one(g, kind):
        job = shard_job(T.job_of[g], g)
        i = next(counter)
        if kind == "grads":
            it = TransferIntent(f"{job}-g{g}-grads-{i}", job, sessions[g], f"dg{g}", f"hg{g}", "d2h", T.n, rng,
                                workload_kind="training_state", metadata={"chunk_bytes": a.chunk})
        else:
            it = TransferIntent(f"{job}-g{g}-params-{i}", job, sessions[g], f"hp{g}", f"dp{g}", "h2d", T.n, rng,
                                workload_kind="training_state", metadata={"chunk_bytes": a.chunk})
        t0 = time.perf_counter()
        r = client.transfer(it, timeout_seconds=TRANSFER_TIMEOUT_S)
        if r.state is not TransferStatusState.COMPLETE:
            raise RuntimeError(f"{it.intent_id}: {r.error}")
        return g, kind, time.perf_counter() - t0, r

    def step():
        t0 = time.perf_counter()
        futs = [pool.submit(one, g, k) for g in active for k in ("grads", "params")]
        try:
            res = [f.result() for f in futs]
        except Exception:
            for f in futs:
                f.cancel()
            pool.shutdown(wait=False, cancel_futures=True)
            raise
        return time.perf_counter() - t0, res

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(len(gpus)).start()
    steps = [step() for _ in range(a.steps)]
    clk = clocks.stop()
    pool.shutdown()
    desc = dc.describe().payload
    leaked = {k: q["active_chunks"] for k, q in desc["relay_quotas"].items() if q["active_chunks"]}
    per_job, relay_b, total_b = {}, 0, 0
    for _dt, res in steps:
        for g, _k, secs, r in res:
            j = T.job_of[g]
            per_job[j] = max(per_job.get(j, 0.0), secs)
            for p in r.path_stats:
                total_b += int(p.get("bytes", 0))
                relay_b += int(p.get("bytes", 0)) if p.get("kind") == "relay" else 0
    verified = all(T.verify(g) for g in active)
    out = {"step_s": [round(dt, 4) for dt, _ in steps], "per_job_s": per_job, "clocks": clk,
           "relay_share": round(relay_b / max(1, total_b), 4), "verified": verified,
           "leaked_quota_chunks": leaked, "open_reservations": len(desc["reservations"]),
           "shard_bytes": T.n, "active_gpus": active}
    T.release()
    return out


ADAM_KW = dict(lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
CHECK_PARAMS = 64 * 2048


def _run_streamed_adamw(a, T, dc, client, sessions, active, gpus) -> dict:
    import torch

    from ..adapters.streamed_optimizer import TILE_BYTES, StreamedAdamW

    opts, p0 = {}, {}
    for g in active:
        # start from the host image of the parameters (the device copy is uninitialised)
        T.dev_params[g].copy_(torch.from_numpy(T.host_params[g].numpy()))
        torch.cuda.synchronize(g)
        params = T.dev_params[g].view(torch.bfloat16)
        p0[g] = params[:CHECK_PARAMS].cpu().clone()
        opts[g] = StreamedAdamW(params, client=client, daemon_client=dc, session_id=sessions[g],
                                job_id=shard_job(T.job_of[g], g), chunk_bytes=max(TILE_BYTES, a.chunk // TILE_BYTES
                                                                                   * TILE_BYTES),
                                prefix=f"opt{g}", **ADAM_KW)
    pool = ThreadPoolExecutor(max_workers=len(active))
    grads = {g: T.dev_grads[g].view(torch.bfloat16) for g in active}

    def one(g):
        t0 = time.perf_counter()
        st = opts[g].step(grads[g])
        return g, time.perf_counter() - t0, st

    def step():
        t0 = time.perf_counter()
        res = [f.result() for f in [pool.submit(one, g) for g in active]]
        return time.perf_counter() - t0, res

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(len(gpus)).start()
    steps = [step() for _ in range(a.steps)]
    clk = clocks.stop()
    pool.shutdown()
    desc = dc.describe().payload
    leaked = {k: q["active_chunks"] for k, q in desc["relay_quotas"].items() if q["active_chunks"]}
    per_job, relay_b, total_b, dev_ms = {}, 0, 0, []
    for _dt, res in steps:
        for g, secs, st in res:
            j = T.job_of[g]
            per_job[j] = max(per_job.get(j, 0.0), secs)
            dev_ms.append(st.cuda_ms)
            for dev, nb, _ms in st.lanes:
                total_b += int(nb or 0)
                relay_b += int(nb or 0) if dev not in (-1, None) else 0
    # a slice of every shard against torch.optim.AdamW (same gradient every step)
    verified = True
    nsteps = a.warmup + a.steps
    for g in active:
        ref = torch.nn.Parameter(p0[g].float())
        o = torch.optim.AdamW([ref], **ADAM_KW)
        gr = grads[g][:CHECK_PARAMS].float().cpu()
        for _ in range(nsteps):
            ref.grad = gr
            o.step()
        got = opts[g].state()["master"][:CHECK_PARAMS]
        verified &= bool(torch.allclose(got, ref.detach(), rtol=1e-5, atol=1e-7))
    out = {"step_s": [round(dt, 4) for dt, _ in steps], "per_job_s": per_job, "clocks": clk,
           "relay_share": round(relay_b / max(1, total_b), 4), "verified": verified,
           "leaked_quota_chunks": leaked, "open_reservations": len(desc["reservations"]),
           "shard_bytes": opts[active[0]].tiles * TILE_BYTES, "active_gpus": active,
           "optimizer": "streamed-adamw", "params_per_gpu": opts[active[0]].nparams,
           "step_device_ms_median": round(statistics.median(dev_ms), 3)}
    T.release()
    return out


def run_reference(a) -> dict:
    import torch

    rt0, why = reference_runtime(1, a.chunk)
    if rt0 is None:
        return {"unavailable": why}
    del rt0
    from turbobus import runtime_engine
    from turbobus.planner_engine import PlannerEngine

    T = Tenants(a)
    gpus = T.gpus
    native = runtime_engine._turbobus
    from turbobus.runtime_engine import RuntimeOptions

    rts, plans = {}, {}
    active = gpus[:(a.active_jobs or a.jobs) * a.gpus_per_job]
    for g in active:
        torch.cuda.set_device(g)
        rt = native.Runtime(RuntimeOptions(chunk_bytes=a.chunk).to_native())
        rt.init(g, [r for r in gpus if r != g])
        prof = rt.profile(256 << 20, False)
        for d in ("h2d", "d2h"):
            plans[(g, d)] = runtime_engine._native_transfer_plan(PlannerEngine().plan(T.n, a.chunk, prof, "pool",
                                                                                     direction=d))
        rts[g] = rt
    lock = threading.Lock()

    def one(g, kind):
        rt = rts[g]
        t0 = time.perf_counter()
        with lock:  # the reference runtime is driven from one thread at a time per process
            torch.cuda.set_device(g)
            if kind == "grads":
                h = rt.offload_plan_to_cpu(T.dev_grads[g].data_ptr(), T.n, T.host_grads[g].ptr, T.n,
                                           plans[(g, "d2h")])
            else:
                h = rt.fetch_plan_to_gpu(T.host_params[g].ptr, T.n, T.dev_params[g].data_ptr(), T.n,
                                         plans[(g, "h2d")])
        rt.wait(h)
        return g, kind, time.perf_counter() - t0

    pool = ThreadPoolExecutor(max_workers=2 * len(active))

    def step():
        t0 = time.perf_counter()
        res = [f.result() for f in [pool.submit(one, g, k) for g in active for k in ("grads", "params")]]
        return time.perf_counter() - t0, res

    for _ in range(a.warmup):
        step()
    clocks = ClockSampler(len(gpus)).start()
    steps = [step() for _ in range(a.steps)]
    clk = clocks.stop()
    pool.shutdown()
    per_job = {}
    for _dt, res in steps:
        for g, _k, secs in res:
            per_job[T.job_of[g]] = max(per_job.get(T.job_of[g], 0.0), secs)
    verified = all(T.verify(g) for g in active)
    del rts
    out = {"step_s": [round(dt, 4) for dt, _ in steps], "per_job_s": per_job, "clocks": clk, "verified": verified,
           "shard_bytes": T.n, "active_gpus": active, "relay_share": None}
    T.release()
    return out


def main(argv=None) -> int:
    a = parse_args(argv)
    try:
        res = run_reference(a) if a.impl == "reference" else run_ours(a)
    except Exception as exc:  # noqa: BLE001 - report and leave without waiting on worker threads
        import os
        import traceback

        traceback.print_exc()
        emit({"impl": a.impl, "error": f"{type(exc).__name__}: {exc}"}, a.json_out)
        os._exit(1)
    if "unavailable" in res:
        emit({"impl": a.impl, "unavailable": res["unavailable"]}, a.json_out)
        return 0
    step = statistics.median(res["step_s"])
    nbytes = 2 * res["shard_bytes"] * len(res["active_gpus"])
    per_job = res["per_job_s"]
    metric = ("multi-tenant training offload step (bf16 grads D2H + params H2D, all jobs)"
              if res.get("optimizer") is None else
              "multi-tenant streamed AdamW step (fp32 state H2D + D2H, fused update, all jobs)")
    line = {"metric": metric,
            "value": round(step * 1e3, 2), "unit": "ms", "higher_is_better": False, "impl": a.impl,
            "n_gpus": len(res["active_gpus"]), "steps": a.steps, "warmup": a.warmup,
            "aggregate_gb_per_s": round(nbytes / 1e9 / step, 2), "per_job_ms": {f"job{k}": round(v * 1e3, 1)
                                                                                for k, v in per_job.items()},
            "jain_fairness": round(jain([1.0 / v for v in per_job.values()]), 4),
            "relay_share": res.get("relay_share"), "verified": res["verified"], "clocks": res["clocks"],
            "optimizer": res.get("optimizer", "none"), "params_per_gpu": res.get("params_per_gpu"),
            "step_device_ms_median": res.get("step_device_ms_median"),
            "leaked_quota_chunks": res.get("leaked_quota_chunks"), "open_reservations": res.get("open_reservations"),
            "config": {"model": f"decoder-7b ({a.layers} layers) data-parallel x{a.gpus_per_job}",
                       "jobs": a.jobs, "gpus_per_job": a.gpus_per_job, "active_jobs": a.active_jobs or a.jobs,
                       "lend_across_groups": bool(getattr(a, "lend_across_groups", False)),
                       "shard_bytes_per_gpu": res["shard_bytes"], "bytes_per_step": nbytes, "chunk_bytes": a.chunk,
                       "data": "synthetic bf16 (params N(0,0.02), grads N(0,1e-3)), seeded"}}
    emit(line, a.json_out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
