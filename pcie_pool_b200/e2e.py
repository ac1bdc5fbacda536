"""End-to-end measurement through the public API.

``socket_daemon_pooled_load`` is the headline: the daemon is its own process
on an AF_UNIX socket.  ``public_api_pooled_load`` runs the same intents on an
in-process daemon whose executor drives the bench's engine.

One step = one intent through ``TurboBusClient``.  Inside the step:
the daemon plans (scheduler + planner on the probed profile), leases relays,
issues the ticket, the executor runs the pooled H2D copy of the step's input
from page-locked host memory into GPU0 (fused landing kernel with per-chunk
checksums), and the per-chunk checksums are read back to the host and
returned in the receipt -- that device->host read is the step's result.
"""

from __future__ import annotations

import time
from typing import Any


def build_inprocess_node(engine, devices, target: int = 0, profile: dict | None = None,
                         max_chunks: int = 1 << 16, workers: int = 2):
    """A daemon in this process whose executor drives ``engine``.  Discovery
    only looks at ``devices``; ``workers`` executor threads let a session's
    next intent reach the engine while its current one runs."""
    from .daemon import EngineDataPlane, InProcessDaemonClient, IntentExecutor, TurboBusDaemon
    from .topology import synthetic_inventory
    from .topology.cuda_nvml import CudaNvmlTopologyProvider, TopologyDiscoveryError

    try:
        provider = CudaNvmlTopologyProvider(devices=devices)
        provider.snapshot()
    except (TopologyDiscoveryError, Exception):  # noqa: BLE001 - fall back to a described node
        from .topology import StaticTopologyProvider

        provider = StaticTopologyProvider(synthetic_inventory(max(devices) + 1, source="declared"))
    relays = [d for d in devices if d != target]
    plane = EngineDataPlane(engine=engine, checksum=True)
    daemon = TurboBusDaemon(relays, max_inflight_chunks_per_relay=max_chunks, topology_provider=provider,
                            executor=IntentExecutor(plane, max_workers=int(workers)))
    if profile is not None and relays:
        daemon.put_profile(target, relays, profile)
    return daemon, InProcessDaemonClient(daemon)


def nominal_profile(target: int, relays, lane_gibps: float = 50.0, p2p_gibps: float = 700.0) -> dict:
    """An even profile (every lane the same rate) for a daemon that has not
    probed its links yet: the planner then splits evenly across the direct
    lane and the relays; a probed profile replaces it."""
    return {"target_device": int(target), "direct_h2d_bw_gbps": lane_gibps, "direct_d2h_bw_gbps": lane_gibps,
            "relays": [{"relay_device": int(r), "target_device": int(target), "h2d_bw_gbps": lane_gibps,
                        "d2h_bw_gbps": lane_gibps, "p2p_bw_gbps": p2p_gibps, "effective_bw_gbps": lane_gibps,
                        "effective_d2h_bw_gbps": lane_gibps, "p2p_enabled": True} for r in relays]}


def public_api_pooled_load(args, eng, host, dev, profile: dict | None = None, depth: int = 2) -> dict[str, Any]:
    import torch

    from . import TransferIntent, TransferStatusState, TurboBusClient

    n = int(args.bytes)
    devices = list(range(args.gpus))
    daemon, dc = build_inprocess_node(eng, devices, 0, profile, workers=max(2, depth))
    sess = dc.register_session(0, devices[1:], max_inflight_chunks=1 << 16)
    if not sess.ok:
        raise RuntimeError(sess.error)
    sid = sess.payload["session"]["session_id"]
    dc.register_job("bench-e2e", session_id=sid)
    dc.register_buffer("host-src", "bench-e2e", "cpu_pinned", n, address=host.ptr, pinned=True)
    dc.register_buffer("gpu0-dst", "bench-e2e", "gpu", n, device_index=0, address=dev.data_ptr())
    client = TurboBusClient(daemon=dc)
    hint = {"chunk_bytes": int(args.chunk)}

    def intent(i: int):
        return TransferIntent(f"e2e-{i}", "bench-e2e", sid, "host-src", "gpu0-dst", "h2d", n,
                              ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                              workload_kind="model_weights", metadata=hint)

    def run(first: int, count: int):
        # ``depth`` intents in flight: submit the next, then wait the oldest
        inflight, last = [], None
        for i in range(first, first + count):
            client.submit_transfer_intent(intent(i))
            inflight.append(f"e2e-{i}")
            if len(inflight) >= depth:
                last = client.wait(inflight.pop(0), timeout_seconds=120)
                if last.state is not TransferStatusState.COMPLETE:
                    raise RuntimeError(f"e2e step failed: {last.error}")
        for iid in inflight:
            last = client.wait(iid, timeout_seconds=120)
            if last.state is not TransferStatusState.COMPLETE:
                raise RuntimeError(f"e2e step failed: {last.error}")
        return last

    run(0, max(1, args.warmup))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    last = run(max(1, args.warmup), args.steps)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    wall = (time.perf_counter() - t0) * 1e3
    meas = (last.metadata or {}).get("measured", {}) if last else {}
    nchunks = len(meas.get("chunk_checksums", [])) if meas else 0
    # the engine reads back the per-chunk checksum table (256-byte aligned)
    # plus one 256-byte status block after every transfer
    d2h = ((16 * max(nchunks, 1) + 255) // 256) * 256 + 256
    return {"value": round(n * args.steps / 1e9 / (ms / 1e3), 3), "unit": "GB/s",
            "ms_per_step": round(ms / args.steps, 3), "wall_ms_per_step": round(wall / args.steps, 3),
            "h2d_bytes_per_step": n, "d2h_bytes_per_step": d2h,
            "intents_in_flight": depth,
            "path": "TurboBusClient -> in-process daemon (scheduler, leases, ticket) -> executor -> PoolEngine",
            "lanes": [(p.get("relay_device"), p.get("bytes")) for p in last.path_stats] if last else []}


def socket_daemon_pooled_load(args, host_np, dev, profile: dict | None, lane_set, *, depth: int = 2,
                              steps: int | None = None, warmup: int | None = None) -> dict[str, Any]:
    """End to end as an application on the node sees it: the daemon runs as
    its own process (``python -m pcie_pool_b200.daemon --execute``) on an
    AF_UNIX socket and owns the data plane for the lane-set GPUs only; this
    process is the client.  The step's input sits in a shared page-locked
    host buffer (``SharedPinnedCpuBuffer``), the destination is GPU0 memory
    exported by CUDA IPC (``CudaIpcDeviceBuffer``), and each step is one
    ``TurboBusClient`` intent.  The client keeps ``depth`` intents in
    flight (submit the next, then wait for the oldest): the daemon admits a
    session's next intent behind its running one, so planning and the
    socket round trips overlap the data movement.  The daemon's data plane
    reads the per-chunk checksums back from the device (the step's result)
    and returns them in the receipt.  Timed by wall clock with the device
    synchronised on both sides: the work runs in the daemon process."""
    import os
    import shutil
    import subprocess
    import sys
    import tempfile

    import torch

    from . import TransferIntent, TransferStatusState, TurboBusClient
    from .client import CudaIpcDeviceBuffer, SharedPinnedCpuBuffer
    from .daemon import TurboBusDaemonClient

    n = int(args.bytes)
    lane_set = [int(d) for d in lane_set]
    target = lane_set[0]
    relays = lane_set[1:]
    steps = int(args.steps if steps is None else steps)
    warmup = int(args.warmup if warmup is None else warmup)
    tmp = tempfile.mkdtemp(prefix="ppb-e2e-")
    sock = os.path.join(tmp, "daemon.sock")
    cmd = [sys.executable, "-m", "pcie_pool_b200.daemon", "--target-gpu", str(target), "--execute",
           "--gpus", ",".join(str(d) for d in lane_set), "--min-relays", "0",
           "--max-inflight-chunks-per-relay", str(1 << 16), "--executor-workers", str(max(2, depth)),
           "--socket-path", sock]
    if not relays:
        cmd.append("--allow-missing-fabric")
    proc = subprocess.Popen(cmd, cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    cpu = None
    dc = None
    try:
        t_end = time.monotonic() + 120
        while not os.path.exists(sock):
            if proc.poll() is not None:
                raise RuntimeError(f"daemon process exited with code {proc.returncode}")
            if time.monotonic() > t_end:
                raise RuntimeError("daemon process did not open its socket")
            time.sleep(0.05)
        dc = TurboBusDaemonClient(sock, persistent=True, timeout=600)
        if profile is not None and relays:
            r = dc.put_profile(target, relays, profile)
            if not r.ok:
                raise RuntimeError(f"daemon rejected the profile: {r.error}")
        sess = dc.register_session(target, relays, max_inflight_chunks=1 << 16)
        if not sess.ok:
            raise RuntimeError(sess.error)
        sid = sess.payload["session"]["session_id"]
        job = f"bench-e2e-{os.getpid()}"
        r = dc.register_job(job, session_id=sid)
        if not r.ok:
            raise RuntimeError(r.error)
        cpu = SharedPinnedCpuBuffer.allocate("e2e-src", job, n)
        cpu.numpy()[:] = host_np[:n]  # the daemon page-locks its mapping on first use
        gpu = CudaIpcDeviceBuffer.from_tensor("e2e-dst", job, dev)
        for b in (cpu, gpu):
            r = b.register_with_daemon(dc)
            if not r.ok:
                raise RuntimeError(r.error)
        client = TurboBusClient(daemon=dc)
        hint = {"chunk_bytes": int(args.chunk)}

        def intent(i: int):
            return TransferIntent(f"e2e-{i}", job, sid, "e2e-src", "e2e-dst", "h2d", n,
                                  ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                                  workload_kind="model_weights", metadata=hint)

        def run(first: int, count: int):
            inflight, last = [], None
            for i in range(first, first + count):
                client.submit_transfer_intent(intent(i))
                inflight.append(f"e2e-{i}")
                if len(inflight) >= depth:
                    last = client.wait(inflight.pop(0), timeout_seconds=600)
                    if last.state is not TransferStatusState.COMPLETE:
                        raise RuntimeError(f"e2e step failed: {last.error}")
            for iid in inflight:
                last = client.wait(iid, timeout_seconds=600)
                if last.state is not TransferStatusState.COMPLETE:
                    raise RuntimeError(f"e2e step failed: {last.error}")
            return last

        run(0, max(1, warmup))
        torch.cuda.synchronize(target)
        t0 = time.perf_counter()
        last = run(max(1, warmup), steps)
        torch.cuda.synchronize(target)
        ms = (time.perf_counter() - t0) * 1e3
        meas = (last.metadata or {}).get("measured", {}) if last else {}
        nchunks = len(meas.get("chunk_checksums", [])) if meas else 0
        d2h = ((16 * max(nchunks, 1) + 255) // 256) * 256 + 256
        tail = torch.equal(dev[n - 4096:].cpu(), torch.from_numpy(host_np[n - 4096:n].copy()))
        return {"value": round(n * steps / 1e9 / (ms / 1e3), 3), "unit": "GB/s",
                "ms_per_step": round(ms / steps, 3), "steps": steps, "intents_in_flight": depth,
                "h2d_bytes_per_step": n, "d2h_bytes_per_step": d2h, "verified_tail": bool(tail),
                "path": "TurboBusClient -> AF_UNIX -> daemon process (scheduler, leases, ticket, executor) -> "
                        "PoolEngine; shared pinned host buffer, CUDA IPC device buffer",
                "lanes": [(p.get("relay_device"), p.get("bytes")) for p in last.path_stats] if last else []}
    finally:
        if dc is not None:
            try:
                dc.close()
            except Exception:  # noqa: BLE001 - best-effort cleanup
                pass
        proc.terminate()
        try:
            proc.wait(timeout=30)
        except subprocess.TimeoutExpired:
            proc.kill()
        if cpu is not None:
            try:
                cpu.release()
            except Exception:  # noqa: BLE001 - best-effort cleanup
                pass
        shutil.rmtree(tmp, ignore_errors=True)
