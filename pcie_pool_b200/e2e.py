"""End-to-end measurement through the public API.

One step = the user's call: ``TurboBusClient.transfer(intent)`` on an
in-process daemon whose executor drives the same engine.  Inside the step:
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
                         max_chunks: int = 1 << 16):
    from .daemon import EngineDataPlane, InProcessDaemonClient, IntentExecutor, TurboBusDaemon
    from .topology import synthetic_inventory
    from .topology.cuda_nvml import CudaNvmlTopologyProvider, TopologyDiscoveryError

    try:
        provider = CudaNvmlTopologyProvider()
        provider.snapshot()
    except (TopologyDiscoveryError, Exception):  # noqa: BLE001 - fall back to a described node
        from .topology import StaticTopologyProvider

        provider = StaticTopologyProvider(synthetic_inventory(max(devices) + 1, source="declared"))
    relays = [d for d in devices if d != target]
    plane = EngineDataPlane(engine=engine, checksum=True)
    daemon = TurboBusDaemon(relays, max_inflight_chunks_per_relay=max_chunks, topology_provider=provider,
                            executor=IntentExecutor(plane, max_workers=1))
    if profile is not None and relays:
        daemon.put_profile(target, relays, profile)
    return daemon, InProcessDaemonClient(daemon)


def public_api_pooled_load(args, eng, host, dev, profile: dict | None = None) -> dict[str, Any]:
    import torch

    from . import TransferIntent, TransferStatusState, TurboBusClient

    n = int(args.bytes)
    devices = list(range(args.gpus))
    daemon, dc = build_inprocess_node(eng, devices, 0, profile)
    sess = dc.register_session(0, devices[1:], max_inflight_chunks=1 << 16)
    if not sess.ok:
        raise RuntimeError(sess.error)
    sid = sess.payload["session"]["session_id"]
    dc.register_job("bench-e2e", session_id=sid)
    dc.register_buffer("host-src", "bench-e2e", "cpu_pinned", n, address=host.ptr, pinned=True)
    dc.register_buffer("gpu0-dst", "bench-e2e", "gpu", n, device_index=0, address=dev.data_ptr())
    client = TurboBusClient(daemon=dc)
    hint = {"chunk_bytes": int(args.chunk)}

    def step(i: int):
        it = TransferIntent(f"e2e-{i}", "bench-e2e", sid, "host-src", "gpu0-dst", "h2d", n,
                            ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                            workload_kind="model_weights", metadata=hint)
        r = client.transfer(it, timeout_seconds=120)
        if r.state is not TransferStatusState.COMPLETE:
            raise RuntimeError(f"e2e step failed: {r.error}")
        return r

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    last = None
    for i in range(args.steps):
        last = step(args.warmup + i)
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
            "path": "TurboBusClient.transfer -> daemon (scheduler, leases, ticket) -> executor -> PoolEngine",
            "lanes": [(p.get("relay_device"), p.get("bytes")) for p in last.path_stats] if last else []}
