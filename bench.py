#!/usr/bin/env python
"""Headline benchmark: pooled host->GPU bandwidth into GPU0.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

One step moves ``--bytes`` (default 4 GiB, far larger than the 126 MB L2)
of uniform-random bytes from a page-locked host buffer into GPU0 over the
direct PCIe lane plus N-1 relay lanes.  The total work is
fixed as N grows (strong scaling).  Every step is submitted and waited through
the data plane; the K timed steps are bracketed by a barrier and a device
synchronisation on both sides and timed with CUDA events on GPU0; the
reported time is the max over ranks.  Under torchrun every rank joins the
barriers, rank 0 drives the data plane, which holds contexts on all N GPUs
(one data-plane process per node, as in the reference's worker).

``--impl reference`` runs the unmodified reference (installed under
baseline/_ref) through its own public runtime API: one persistent
``_turbobus.Runtime``, its own profiler and planner, ``fetch_plan_to_gpu`` +
``wait`` per step.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = "pooled host->GPU GB/s into one GPU"


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--bytes", type=int, default=4 << 30)
    p.add_argument("--chunk", type=int, default=16 << 20)
    p.add_argument("--slots", type=int, default=3)
    p.add_argument("--ctas", type=int, default=4, help="lane-kernel CTAs per lane")
    p.add_argument("--coalesce", type=int, default=64 << 20,
                   help="largest merged copy-engine transfer on the direct lane (bytes)")
    p.add_argument("--direction", choices=["h2d", "d2h"], default="h2d")
    p.add_argument("--lane-order", choices=["spread", "index"], default="spread",
                   help="ours: GPU0 plus N-1 relays spread over measured contention groups and PCIe uplinks "
                        "(socket, root complex, switch) among the visible GPUs, or simply GPUs 0..N-1")
    p.add_argument("--no-checksum", action="store_true", help="skip the fused per-chunk checksum")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-extra", action="store_true",
                   help="skip the other two BASELINE metrics (8B-shape load s, KV reload p50)")
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


# ---- distributed plumbing -------------------------------------------------------------

class Dist:
    """One rank per GPU of the lane set: rank r runs on ``lane_set[r]`` (the
    lane set is computed identically on every rank from the topology), so
    exactly the N GPUs that carry lanes are active."""

    def __init__(self, lane_set=None):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.device = int(lane_set[self.local_rank]) if lane_set and self.local_rank < len(lane_set) \
            else self.local_rank
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            torch.cuda.set_device(self.device)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", self.device))
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            import torch

            self.pg.barrier(device_ids=[self.device])
            torch.cuda.synchronize()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64, device=f"cuda:{self.device}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


# ---- clocks and host data ---------------------------------------------------------------

from pcie_pool_b200.benchmarks.common import ClockSampler, fill_random, fill_random_torch  # noqa: E402


# ---- the other two BASELINE metrics ---------------------------------------------------------

def extra_metrics(args, impl: str, devices) -> dict:
    """Llama-3-8B-shape bf16 load time (BASELINE config 3a, 16.06 GB into
    GPU0 over the lane set) and the vLLM KV reload p50 (config 4: 32k-token
    requests of a Llama-3-8B KV cache restored into permuted block tables),
    on the same GPUs as the headline.  Ours goes through the daemon (intents
    under relay leases); the reference through its own runtime.  Measured
    after the headline's timed region; each failure is reported in place of
    its figure."""
    from types import SimpleNamespace

    from pcie_pool_b200.benchmarks import kv_offload, llama_load

    if impl == "reference":
        return reference_extra_metrics(args, len(devices))
    out: dict = {}
    common = dict(gpus=len(devices), devices=list(devices), impl=impl, via="daemon", json_out="")
    try:
        a = SimpleNamespace(**common, steps=3, warmup=1, variant="bf16", chunk=16 << 20, api=False, layers=0)
        r = llama_load.run_reference(a) if impl == "reference" else llama_load.run_ours(a)
        out["load_s"] = (r["unavailable"] if "unavailable" in r else round(r["ms"] / 1e3, 4))
        out["load_verified"] = r.get("verified")
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        out["load_s"] = f"error: {type(exc).__name__}: {exc}"
    try:
        import statistics

        a = SimpleNamespace(**common, requests=4, tokens=32768, layers=32, steps=2, warmup=1, chunk=4 << 20, seed=0)
        r = kv_offload.run_reference(a) if impl == "reference" else kv_offload.run_ours(a)
        if "unavailable" in r:
            out["kv_reload_p50_ms"] = r["unavailable"]
        else:
            out["kv_reload_p50_ms"] = round(statistics.median(r["reload_ms"]), 3)
            out["kv_offload_p50_ms"] = round(statistics.median(r["offload_ms"]), 3)
            out["kv_verified"] = r.get("verified")
            out["kv_config"] = "Llama-3-8B KV, 4 requests x 32k tokens (4 GiB each), permuted block tables"
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        out["kv_reload_p50_ms"] = f"error: {type(exc).__name__}: {exc}"
    return out


def _child_json(argv: list[str], timeout_s: float) -> dict:
    """Run ``python -m <argv>`` in its own process group and return the JSON
    object it wrote to ``--json-out``; a crash or a run past ``timeout_s``
    (the whole group is killed) comes back as ``{"error": ...}``."""
    import signal
    import subprocess
    import tempfile

    with tempfile.NamedTemporaryFile(suffix=".json", delete=False) as fh:
        path = fh.name
    try:
        proc = subprocess.Popen([sys.executable, "-m", *argv, "--json-out", path], cwd=str(ROOT),
                                stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, start_new_session=True)
        try:
            _, err = proc.communicate(timeout=timeout_s)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)
            proc.communicate()
            return {"error": f"no result within {timeout_s:.0f} s (process group killed)"}
        if proc.returncode != 0:
            tail = (err or b"").decode(errors="replace").strip().splitlines()[-1:] or [""]
            return {"error": f"exit code {proc.returncode}: {tail[0][:200]}"}
        with open(path) as fh:
            return json.load(fh)
    except (OSError, ValueError) as exc:
        return {"error": f"{type(exc).__name__}: {exc}"}
    finally:
        try:
            os.unlink(path)
        except OSError:
            pass


def reference_extra_metrics(args, n_gpus: int) -> dict:
    """The reference arm's load time and KV reload p50, each in a child
    process with a time limit, so that a crash or a stall inside the
    reference's code costs that one figure and not the bench line."""
    out: dict = {}
    g = str(n_gpus)
    r = _child_json(["pcie_pool_b200.benchmarks.llama_load", "--impl", "reference", "--gpus", g, "--variant", "bf16",
                     "--steps", "3", "--warmup", "1"], 300)
    if "error" in r or "unavailable" in r:
        out["load_s"] = r.get("unavailable") or f"error: {r['error']}"
    else:
        out["load_s"] = round(r["value"], 4) if r.get("unit") == "s" else r.get("load_s", r.get("value"))
        out["load_verified"] = r.get("verified")
    # The reference plans a paged-KV request as 131,072 separate 32 KiB ranges
    # and moves them one by one: 4 requests x 3 passes x 2 directions ran past
    # 300 s on one GPU, so its arm takes 2 requests x 2 passes (same request
    # shape, fewer samples of the p50).
    r = _child_json(["pcie_pool_b200.benchmarks.kv_offload", "--impl", "reference", "--gpus", g, "--requests", "2",
                     "--tokens", "32768", "--steps", "1", "--warmup", "1"], 300)
    if "error" in r or "unavailable" in r:
        out["kv_reload_p50_ms"] = r.get("unavailable") or f"error: {r['error']}"
    else:
        out["kv_reload_p50_ms"] = r["reload_p50_ms"]
        out["kv_offload_p50_ms"] = r["offload_p50_ms"]
        out["kv_verified"] = r.get("verified")
        out["kv_config"] = "Llama-3-8B KV, 2 requests x 32k tokens (4 GiB each), permuted block tables"
    return out


# ---- our implementation ---------------------------------------------------------------

def run_ours(args, dist: Dist) -> dict:
    import numpy as np
    import torch

    from pcie_pool_b200.parallel.engine import D2H, H2D, PoolEngine
    from pcie_pool_b200.parallel.planning import plan_lanes
    from pcie_pool_b200.utils.checksum import combine, rebase_chunk_sums
    from pcie_pool_b200.utils.host_memory import PinnedHostBuffer

    N = args.gpus
    devices = list(args.lane_set)
    n = args.bytes
    out: dict = {}
    if dist.rank == 0:
        torch.cuda.set_device(0)
        host = PinnedHostBuffer(n, fill=None)
        fill_random(host.numpy(), seed=1234)
        dev = torch.empty(n, dtype=torch.uint8, device="cuda:0")
        if args.direction == "d2h":
            dev.copy_(torch.from_numpy(host.numpy()).to("cuda:0"))
        eng = PoolEngine(devices, slot_bytes=max(args.chunk, 1 << 20), slots=args.slots,
                         ctas_per_lane=args.ctas, timeout_s=20.0, coalesce_bytes=args.coalesce)
        direction = H2D if args.direction == "h2d" else D2H
        dname = args.direction
        checksum = not args.no_checksum
        kernel_per_step = 1 if (checksum or N > 1) else 0
        # Calibration (outside the timed region): the link probe measures the
        # lanes solo and together and picks the lane set with the highest
        # aggregate; warm-up steps then refine the per-lane weights.
        profile = None
        lane_set, weights = devices, None
        if N > 1:
            from pcie_pool_b200.parallel.linkprobe import concurrent_lane_plan, probe_profile

            profile = probe_profile(eng, 0, devices[1:], nbytes=min(n, 1 << 30), chunk=args.chunk)
            picked = concurrent_lane_plan(profile, dname)
            if picked is not None:
                lane_set, weights = picked
        from pcie_pool_b200.parallel.balance import LaneBalancer

        balancer = LaneBalancer(alpha=0.5)
        if weights is not None:
            balancer.seed(0, dname, dict(zip(lane_set, weights)))
        state = {"lanes": plan_lanes(n, args.chunk, lane_set, target=0, bw_gibps=weights)}

        def step(adapt: bool = False):
            r = eng.run(direction, 0, host.ptr, n, dev.data_ptr(), n, state["lanes"], checksum=checksum)
            if not r.ok:
                raise RuntimeError(r.error)
            if adapt and len(lane_set) > 1:
                balancer.observe(0, dname, r)
                w = balancer.weights(0, dname, lane_set)
                state["lanes"] = plan_lanes(n, args.chunk, lane_set, target=0, bw_gibps=w)
            return r

        for _ in range(args.warmup):
            step(adapt=True)
    dist.barrier()
    res = None
    elapsed_ms = 0.0
    clocks = ClockSampler(devices)
    if dist.rank == 0:
        torch.cuda.synchronize()
        clocks.start()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            res = step()
        e1.record()
        torch.cuda.synchronize()
        elapsed_ms = e0.elapsed_time(e1)
        clk = clocks.stop()
    dist.barrier()
    elapsed_ms = dist.max(elapsed_ms)
    if dist.rank == 0:
        verified = None
        lanes = state["lanes"]
        if checksum and direction == H2D:
            C = __import__("pcie_pool_b200._C", fromlist=["x"])
            host_sum = C.checksum_host(host.ptr, n)
            got = combine(rebase_chunk_sums(res.checksums, lanes))
            verified = (tuple(int(x) for x in host_sum) == got)
        out = {
            "elapsed_ms": elapsed_ms,
            "clocks": clk,
            "lane_ms": [(l.device, round(l.cuda_ms, 3), l.bytes) for l in res.lanes],
            "verified": verified,
            "gpu_launches": kernel_per_step * args.steps,
            "transfer_cuda_ms": res.cuda_ms,
            "lane_set": list(lane_set),
            "gpus_bound": list(devices),
            "lane_choice": args.lane_info,
            "probe": None if profile is None else profile.get("concurrent"),
        }
        if not args.no_e2e and direction == H2D:
            from pcie_pool_b200.e2e import public_api_pooled_load, socket_daemon_pooled_load

            try:
                out["e2e"] = socket_daemon_pooled_load(args, host.numpy(), dev, profile, lane_set)
            except Exception as exc:  # pragma: no cover - reported in the JSON line
                out["e2e"] = {"error": f"{type(exc).__name__}: {exc}"}
            try:
                out["e2e_inprocess"] = public_api_pooled_load(args, eng, host, dev, profile)
            except Exception as exc:  # pragma: no cover - reported in the JSON line
                out["e2e_inprocess"] = {"error": f"{type(exc).__name__}: {exc}"}
        del eng, dev
        host.release()
        torch.cuda.empty_cache()
        if not args.no_extra and direction == H2D:
            out["extra"] = extra_metrics(args, "ours", devices)
    return out


# ---- reference implementation -----------------------------------------------------------

def reference_runtime_e2e(args, rt, host_t, dev, profile, relays) -> dict:
    """The reference end to end through its runtime API, as an application
    that drives it directly: every step its planner plans the transfer on its
    profile (``PlannerEngine.plan`` + ``_native_transfer_plan``), its runtime
    moves the bytes (``fetch_plan_to_gpu`` + ``wait``), and 4 KiB of the
    landed bytes are read back to the host; wall clock with the device
    synchronised on both sides.  Its other byte-moving public path, the
    worker-managed client (daemon + worker-helper processes), is not run: on
    this pool it crashed (SIGSEGV) in one call and hung past 900 s in the
    next, at N=1 and N=2."""
    import time

    import torch
    from turbobus import runtime_engine
    from turbobus.planner_engine import PlannerEngine

    n = args.bytes
    probe = torch.empty(4096, dtype=torch.uint8)

    def step():
        plan = PlannerEngine().plan(n, args.chunk, profile, "pool" if relays else "direct", direction="h2d")
        h = rt.fetch_plan_to_gpu(host_t.data_ptr(), n, dev.data_ptr(), n, runtime_engine._native_transfer_plan(plan))
        rt.wait(h)
        probe.copy_(dev[n - 4096:])

    for _ in range(max(1, min(args.warmup, 3))):
        step()
    steps = max(1, args.steps)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3
    return {"value": round(n * steps / 1e9 / (ms / 1e3), 3), "unit": "GB/s", "ms_per_step": round(ms / steps, 3),
            "steps": steps, "h2d_bytes_per_step": n, "d2h_bytes_per_step": 4096,
            "verified_tail": bool(torch.equal(probe, host_t[n - 4096:])),
            "path": "turbobus PlannerEngine.plan -> _turbobus.Runtime.fetch_plan_to_gpu -> wait, per step "
                    "(runtime API; the worker-managed client path crashed and hung on this pool and is not run)"}


def run_reference(args, dist: Dist) -> dict:
    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "turbobus").exists() and dist.rank == 0:
        # A fresh box gets the install only when it was made before the
        # snapshot; build it here from the reference source if that exists.
        from __graft_entry__ import install_reference

        outcome = install_reference(str(ref_root))
        print(f"reference arm: {outcome}", file=sys.stderr, flush=True)
    dist.barrier()
    if not (ref_root / "turbobus").exists():
        return {"unavailable": "reference not installed under baseline/_ref and its source is not on this box"}
    sys.path.insert(0, str(ref_root))
    import torch

    out: dict = {}
    N = args.gpus
    n = args.bytes
    if dist.rank == 0:
        from turbobus import runtime_engine
        from turbobus.planner_engine import PlannerEngine
        from turbobus.runtime_engine import RuntimeOptions

        native = runtime_engine._turbobus
        if native is None:
            return {"unavailable": "reference native extension failed to import"}
        torch.cuda.set_device(0)
        host_t = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        fill_random_torch(host_t, seed=1234)
        dev = torch.empty(n, dtype=torch.uint8, device="cuda:0")
        opts = RuntimeOptions(chunk_bytes=args.chunk)
        rt = native.Runtime(opts.to_native())
        relays = list(range(1, N))
        rt.init(0, relays)
        profile = rt.profile(256 << 20, False)
        plan = PlannerEngine().plan(n, args.chunk, profile, "pool", direction=args.direction)
        nplan = runtime_engine._native_transfer_plan(plan)

        def step():
            if args.direction == "h2d":
                h = rt.fetch_plan_to_gpu(host_t.data_ptr(), n, dev.data_ptr(), n, nplan)
            else:
                h = rt.offload_plan_to_cpu(dev.data_ptr(), n, host_t.data_ptr(), n, nplan)
            rt.wait(h)
            return rt.stats(h)

        for _ in range(args.warmup):
            step()
    dist.barrier()
    elapsed_ms = 0.0
    clocks = ClockSampler(N)
    if dist.rank == 0:
        torch.cuda.synchronize()
        clocks.start()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            st = step()
        e1.record()
        torch.cuda.synchronize()
        elapsed_ms = e0.elapsed_time(e1)
        clk = clocks.stop()
    dist.barrier()
    elapsed_ms = dist.max(elapsed_ms)
    if dist.rank == 0:
        verified = bool(torch.equal(dev.cpu(), host_t)) if args.direction == "h2d" else None
        out = {
            "elapsed_ms": elapsed_ms,
            "clocks": clk,
            "verified": verified,
            "gpu_launches": 0,
            "transfer_cuda_ms": st.cuda_elapsed_ms,
            "lane_ms": [(p.relay_device, round(p.cuda_elapsed_ms, 3), p.bytes) for p in st.path_stats],
            "profile": {
                "direct_h2d_gibps": profile.direct_h2d_bw_gbps,
                "relays": [(r.relay_device, r.h2d_bw_gbps, r.p2p_bw_gbps, r.effective_bw_gbps)
                           for r in profile.relays],
            },
        }
        if not args.no_e2e and args.direction == "h2d":
            try:
                out["e2e"] = reference_runtime_e2e(args, rt, host_t, dev, profile, relays)
            except Exception as exc:  # noqa: BLE001 - reported in the JSON line
                out["e2e"] = {"error": f"{type(exc).__name__}: {exc}"}
        del rt, host_t, dev
        torch.cuda.empty_cache()
        if not args.no_extra and args.direction == "h2d":
            out["extra"] = extra_metrics(args, "reference", list(range(N)))
    return out


def _measured_lane_set(n: int) -> tuple[list[int], dict]:
    """GPU0 plus n-1 relays among the visible GPUs: spread over contention
    groups measured by a short engine-free copy probe
    (``topology.uplink_probe``), then over the PCIe topology.  With every
    visible GPU in the set the order is the topology's."""
    import torch

    from pcie_pool_b200.topology.cuda_nvml import cuda_lane_set
    from pcie_pool_b200.topology.uplink_probe import contention_groups, probe_rates

    visible = torch.cuda.device_count()
    if n <= 1 or n >= visible:
        return cuda_lane_set(n)
    try:
        rates = probe_rates(list(range(visible)))
        groups = contention_groups(rates["solo"], rates["concurrent"])
    except Exception as exc:  # noqa: BLE001 - a failed probe keeps the topology rule
        lane_set, info = cuda_lane_set(n)
        return lane_set, {**info, "probe": f"failed: {type(exc).__name__}: {exc}"}
    lane_set, info = cuda_lane_set(n, groups=groups)
    info["probe_gb_per_s"] = {k: {str(d): round(v, 2) for d, v in sorted(r.items())} for k, r in rates.items()}
    return lane_set, info


def choose_lane_set(n: int) -> tuple[list[int], dict]:
    """The lane set, identical on every rank: the local rank 0 measures and
    chooses before any process group exists and hands the choice to the other
    ranks of this launch through a file named for the launcher's process and
    port (every rank of one torchrun launch shares both); they wait for it
    with a time limit."""
    import tempfile
    import time

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return _measured_lane_set(n)
    path = Path(tempfile.gettempdir()) / (f"ppb_lane_set_{os.getppid()}_"
                                          f"{os.environ.get('MASTER_PORT', '0')}.json")
    if int(os.environ.get("LOCAL_RANK", "0")) == 0:
        try:
            lane_set, info = _measured_lane_set(n)
        except Exception as exc:  # noqa: BLE001 - every rank must still get a lane set
            lane_set, info = list(range(n)), {"rule": "GPUs 0..N-1", "fallback": f"{type(exc).__name__}: {exc}"}
        tmp = path.with_suffix(".tmp")
        tmp.write_text(json.dumps({"lane_set": lane_set, "info": info}))
        os.replace(tmp, path)
        return lane_set, info
    deadline = time.monotonic() + 300.0
    while not path.exists():
        if time.monotonic() > deadline:
            raise RuntimeError(f"local rank 0 did not publish the lane set ({path}) within 300 s")
        time.sleep(0.05)
    d = json.loads(path.read_text())
    return [int(x) for x in d["lane_set"]], d["info"]


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "ours" and args.lane_order == "spread":
        args.lane_set, args.lane_info = choose_lane_set(args.gpus)
    else:
        args.lane_set, args.lane_info = list(range(args.gpus)), {"rule": "GPUs 0..N-1"}
    dist = Dist(args.lane_set)
    if args.impl == "reference":
        res = run_reference(args, dist)
    else:
        res = run_ours(args, dist)
    if dist.rank == 0:
        if "unavailable" in res:
            line = {"impl": "reference", "unavailable": res["unavailable"]}
        else:
            total = args.bytes * args.steps
            ms = res["elapsed_ms"]
            value = total / 1e9 / (ms / 1e3)
            N = args.gpus
            line = {
                "metric": METRIC,
                "value": round(value, 3),
                "unit": "GB/s",
                "n_gpus": N,
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": round(ms / args.steps, 3),
                "higher_is_better": True,
                "scaling": "strong",
                "vs_baseline": None,
                "dtype": "uint8 (raw bytes)",
                "data": "synthetic (uniform-random bytes, seeded)",
                "config": {
                    "model": "pooled-transfer sweep point (BASELINE config 2)",
                    "direction": args.direction,
                    "transfer_bytes": args.bytes,
                    "chunk_bytes": args.chunk, "coalesce_bytes": args.coalesce,
                    "target_gpu": 0,
                    "relay_gpus": list(args.lane_set[1:]),
                    "parallelism": f"direct+{N - 1}relay",
                    "l2": "inputs larger than L2 (each step moves a fresh 4 GiB stream)",
                },
                "clocks": res.get("clocks"),
                "gpu_launches": res.get("gpu_launches"),
                **{k: v for k, v in (res.get("extra") or {}).items()},
                "verified": res.get("verified"),
                "lane_ms": res.get("lane_ms"),
            }
            if args.impl == "reference":
                line["impl"] = "reference"
                line["profile"] = res.get("profile")
                if "e2e" in res:
                    line["e2e"] = res["e2e"]
            else:
                line["impl"] = "ours"
                line["lane_set"] = res.get("lane_set")
                line["gpus_bound"] = res.get("gpus_bound")
                line["lane_choice"] = res.get("lane_choice")
                line["probe"] = res.get("probe")
                if "e2e" in res:
                    line["e2e"] = res["e2e"]
                if "e2e_inprocess" in res:
                    line["e2e_inprocess"] = res["e2e_inprocess"]
        s = json.dumps(line)
        print(s, flush=True)
        if args.json_out:
            Path(args.json_out).write_text(s + "\n")
    if dist.world > 1 and dist.local_rank == 0:
        import tempfile

        # every rank read the lane set before the process group formed
        (Path(tempfile.gettempdir()) / (f"ppb_lane_set_{os.getppid()}_"
                                        f"{os.environ.get('MASTER_PORT', '0')}.json")).unlink(missing_ok=True)
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
