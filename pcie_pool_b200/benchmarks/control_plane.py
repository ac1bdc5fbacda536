"""Control-plane cost of one intent, without a data plane.

    python -m pcie_pool_b200.benchmarks.control_plane --lanes 8 --bytes 4G --chunk 16M --intents 200

Runs ``TurboBusClient.transfer`` against an in-process daemon whose
executor drives a stand-in engine that completes instantly, so the time per
intent is the daemon's own work: planning on the profile, leases, ticket,
dispatch to the executor thread, completion and the receipt.  The timing is
repeated after ``--history`` earlier intents to show that the per-intent
cost does not grow with the daemon's history.  Prints one JSON line.

``--landing kv`` times a fused paged-KV restore intent instead
(``DaemonKVOffloader.restore``: a Llama-3-8B-shape cache of 32 layers, a
32k-token request = 131,072 units of 32 KiB through a permuted block table,
``units_per_chunk`` 128); the cache and host tensors are allocated but never
touched, so no memory is moved.

``--protocol daemon`` times the daemon protocol alone, the same way on this
package's daemon and, with ``--impl reference``, on the unmodified reference
daemon installed under ``baseline/_ref``: per intent ``submit_transfer_intent``
(planning, leases, ticket), ``transfer_status`` complete and
``release_transfer`` of every lease, in process, with the same synthetic
8-GPU inventory and profile and no data plane.
"""

from __future__ import annotations

import argparse
import json
import statistics
import time

UNITS = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}


def parse_size(s: str) -> int:
    s = str(s).strip().upper()
    return int(float(s[:-1]) * UNITS[s[-1]]) if s and s[-1] in UNITS else int(s)


class InstantEngine:
    """Stand-in for ``PoolEngine``: every transfer completes at once with
    per-lane statistics shaped like the real ones."""

    def run(self, direction, target, host_ptr, host_bytes, dev_ptr, dev_bytes, lanes, checksum=False, **kw):
        import numpy as np

        from ..parallel.engine import LaneResult, TransferResult

        stats = [LaneResult(device=l.device, direct=l.device == target, bytes=int(l.bytes.sum()),
                            chunks=int(l.bytes.size), cuda_ms=1.0) for l in lanes]
        nch = sum(s.chunks for s in stats)
        return TransferResult(id=1, ok=True, status_code=0, error="", bytes=sum(s.bytes for s in stats),
                              cuda_ms=1.0, submit_to_complete_ms=1.0, gib_per_s=1.0, lanes=stats,
                              checksums=np.zeros((nch, 2), dtype=np.uint64))


def build(lanes: int, nbytes: int, history_limit: int = 10000):
    from .. import TurboBusClient
    from ..e2e import build_inprocess_node

    prof = {"target_device": 0, "direct_h2d_bw_gbps": 34.0, "direct_d2h_bw_gbps": 34.0,
            "relays": [{"relay_device": r, "target_device": 0, "h2d_bw_gbps": 26.0, "d2h_bw_gbps": 26.0,
                        "p2p_bw_gbps": 700.0, "effective_bw_gbps": 26.0, "effective_d2h_bw_gbps": 26.0,
                        "p2p_enabled": True} for r in range(1, lanes)]}
    daemon, dc = build_inprocess_node(InstantEngine(), list(range(lanes)), 0, prof if lanes > 1 else None)
    daemon._history_limit = max(1, int(history_limit))
    sid = dc.register_session(0, list(range(1, lanes)), max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    dc.register_job("cp", session_id=sid)
    dc.register_buffer("h", "cp", "cpu_pinned", nbytes, address=4096, pinned=True)
    dc.register_buffer("g", "cp", "gpu", nbytes, device_index=0, address=8192)
    return daemon, TurboBusClient(daemon=dc), sid


PROFILE_BW = {"direct": 34.0, "relay": 26.0, "p2p": 700.0}


def profile_dict(lanes: int) -> dict:
    return {"target_device": 0, "direct_h2d_bw_gbps": PROFILE_BW["direct"],
            "direct_d2h_bw_gbps": PROFILE_BW["direct"],
            "relays": [{"relay_device": r, "target_device": 0, "h2d_bw_gbps": PROFILE_BW["relay"],
                        "d2h_bw_gbps": PROFILE_BW["relay"], "p2p_bw_gbps": PROFILE_BW["p2p"],
                        "effective_bw_gbps": PROFILE_BW["relay"], "effective_d2h_bw_gbps": PROFILE_BW["relay"],
                        "p2p_enabled": True} for r in range(1, lanes)]}


def daemon_protocol_node(impl: str, lanes: int, nbytes: int):
    """(daemon, TransferIntent class, session id) for the bare daemon protocol
    on this package's daemon or the reference's (its own public classes: a
    topology provider over its inventory records, then the same calls)."""
    relays = list(range(1, lanes))
    if impl == "reference":
        import pathlib
        import sys

        ref = pathlib.Path(__file__).resolve().parents[2] / "baseline" / "_ref"
        if not (ref / "turbobus").is_dir():
            raise RuntimeError("reference not installed under baseline/_ref")
        sys.path.insert(0, str(ref))
        from turbobus.daemon.server import TurboBusDaemon as RefDaemon
        from turbobus.schema import TransferIntent as RefIntent
        from turbobus.topology import (DaemonResourceInventory, FabricLinkRecord, GpuInventoryRecord,
                                       PciePathRecord, TopologyProvider)

        inv = DaemonResourceInventory(
            gpus=tuple(GpuInventoryRecord(device_id=g, role="relay" if g else "target") for g in range(lanes)),
            pcie_paths=tuple(PciePathRecord(device_id=g) for g in range(lanes)),
            fabric_links=tuple(FabricLinkRecord(src_device_id=r, dst_device_id=0, fabric="nvlink", enabled=True)
                               for r in relays),
            source="control_plane_benchmark", discovered_at=time.time())

        class Provider(TopologyProvider):
            def snapshot(self):
                return inv

            def invalidate(self):
                return None

        d = RefDaemon(relay_gpus=relays, max_inflight_chunks_per_relay=1 << 20, topology_provider=Provider())
        intent_cls = RefIntent
    else:
        from ..daemon import TurboBusDaemon
        from ..schema import TransferIntent
        from ..topology import StaticTopologyProvider

        d = TurboBusDaemon(relay_gpus=relays, max_inflight_chunks_per_relay=1 << 20,
                           topology_provider=StaticTopologyProvider(gpu_count=lanes), link_hold_seconds=0.0)
        intent_cls = TransferIntent
    assert d.put_profile(target_gpu=0, relay_gpus=relays, profile=profile_dict(lanes)).ok
    sid = d.register_session(target_gpu=0, requested_relays=relays,
                             max_inflight_chunks=1 << 20).payload["session"]["session_id"]
    assert d.register_job(job_id="cp", session_id=sid).ok
    assert d.register_buffer(buffer_id="h", job_id="cp", kind="cpu_pinned", size_bytes=nbytes, address=4096,
                             pinned=True).ok
    assert d.register_buffer(buffer_id="g", job_id="cp", kind="gpu", size_bytes=nbytes, device_index=0,
                             address=8192).ok
    return d, intent_cls, sid


def daemon_protocol_step(d, intent_cls, sid: str, i: int, n: int, chunk: int) -> int:
    """One intent through the bare protocol; returns its relay lease count."""
    it = intent_cls(intent_id=f"cp-{i}", job_id="cp", session_id=sid, source_buffer_id="h",
                    destination_buffer_id="g", direction="h2d", total_bytes=n,
                    ranges=({"src_offset": 0, "dst_offset": 0, "bytes": n},), workload_kind="model_weights",
                    metadata={"chunk_bytes": chunk})
    r = d.submit_transfer_intent(it)
    if not r.ok:
        raise RuntimeError(r.error)
    tid = r.payload["transfer_id"]
    ticket = r.payload.get("ticket") or {}
    leases = list(ticket.get("lease_ids") or ())
    st = d.transfer_status(tid, state="complete", bytes_completed=n)
    if not st.ok:
        raise RuntimeError(st.error)
    for lid in leases:
        d.release_transfer(lid)
    return len(leases)


def main(argv=None) -> int:
    from .. import TransferIntent

    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--lanes", type=int, default=8)
    p.add_argument("--bytes", default="4G")
    p.add_argument("--chunk", default="16M")
    p.add_argument("--intents", type=int, default=200)
    p.add_argument("--history", type=int, default=2000, help="intents run before the second timing")
    p.add_argument("--protocol", choices=["client", "daemon"], default="client",
                   help="client: TurboBusClient.transfer over an instant engine; daemon: bare daemon protocol")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours",
                   help="daemon implementation for --protocol daemon")
    p.add_argument("--landing", choices=["copy", "kv"], default="copy",
                   help="kv: fused paged-KV restore intents (Llama-3-8B shape, 32k tokens)")
    a = p.parse_args(argv)
    n, chunk = parse_size(a.bytes), parse_size(a.chunk)
    if a.protocol == "daemon":
        return _daemon_protocol(a, n, chunk)
    if a.landing == "kv":
        return _kv_intents(a)
    daemon, client, sid = build(a.lanes, n)
    counter = iter(range(1 << 40))

    def step():
        it = TransferIntent(f"cp-{next(counter)}", "cp", sid, "h", "g", "h2d", n,
                            ({"src_offset": 0, "dst_offset": 0, "bytes": n},), workload_kind="model_weights",
                            metadata={"chunk_bytes": chunk})
        r = client.transfer(it, timeout_seconds=60)
        if r.state.value != "complete":
            raise RuntimeError(r.error)

    cpu = []

    def timed(k):
        out = []
        for _ in range(5):
            t0, c0 = time.perf_counter(), time.process_time()
            for _ in range(max(1, k // 5)):
                step()
            out.append((time.perf_counter() - t0) * 1e3 / max(1, k // 5))
            cpu.append((time.process_time() - c0) * 1e3 / max(1, k // 5))
        return statistics.median(out)

    for _ in range(10):
        step()
    first = timed(a.intents)
    cpu_first = statistics.median(cpu)
    for _ in range(a.history):
        step()
    later = timed(a.intents)
    print(json.dumps({"metric": "control-plane ms per intent (instant data plane)", "lanes": a.lanes, "bytes": n,
                      "chunk_bytes": chunk, "chunks": -(-n // chunk), "ms_per_intent": round(first, 3),
                      "cpu_ms_per_intent": round(cpu_first, 3),
                      "ms_per_intent_after_history": round(later, 3), "history": a.history,
                      "retained_transfers": len(daemon.describe().payload["transfer_queue"])}), flush=True)
    return 0


def _kv_intents(a) -> int:
    import numpy as np
    import torch

    from .. import TurboBusClient
    from ..adapters.kv_offload import DaemonKVOffloader
    from ..e2e import build_inprocess_node

    layers, blocks, req_blocks = 32, 4096, 2048
    kvs = [torch.empty(2, blocks, 16, 8, 128, dtype=torch.bfloat16) for _ in range(layers)]
    devs = list(range(a.lanes))
    daemon, dc = build_inprocess_node(InstantEngine(), devs, 0, profile_dict(a.lanes) if a.lanes > 1 else None)
    sid = dc.register_session(0, devs[1:], max_inflight_chunks=1 << 20).payload["session"]["session_id"]
    dc.register_job("kv", session_id=sid)
    off = DaemonKVOffloader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="kv", kv_caches=kvs,
                            units_per_chunk=128, sync_stream=False)
    host = torch.empty(off.prefix_bytes(req_blocks), dtype=torch.uint8)
    rng = np.random.default_rng(0)
    tables = [[int(x) for x in rng.permutation(blocks)[:req_blocks]] for _ in range(4)]
    for i in range(5):
        off.restore(tables[i % 4], host)
    wall, cpu = [], []
    for _ in range(5):
        t0, c0 = time.perf_counter(), time.process_time()
        k = max(1, a.intents // 5)
        for i in range(k):
            off.restore(tables[i % 4], host)
        wall.append((time.perf_counter() - t0) * 1e3 / k)
        cpu.append((time.process_time() - c0) * 1e3 / k)
    print(json.dumps({"metric": "control-plane ms per fused KV restore intent (instant data plane)",
                      "lanes": a.lanes, "units_per_intent": off.units_per_block * req_blocks,
                      "bytes_per_intent": off.prefix_bytes(req_blocks), "ms_per_intent": round(statistics.median(wall), 3),
                      "cpu_ms_per_intent": round(statistics.median(cpu), 3)}), flush=True)
    return 0


def _daemon_protocol(a, n: int, chunk: int) -> int:
    d, intent_cls, sid = daemon_protocol_node(a.impl, a.lanes, n)
    counter = iter(range(1 << 40))
    leases = []

    def timed(k):
        out = []
        for _ in range(5):
            t0 = time.perf_counter()
            for _ in range(max(1, k // 5)):
                leases.append(daemon_protocol_step(d, intent_cls, sid, next(counter), n, chunk))
            out.append((time.perf_counter() - t0) * 1e3 / max(1, k // 5))
        return statistics.median(out)

    for _ in range(10):
        daemon_protocol_step(d, intent_cls, sid, next(counter), n, chunk)
    first = timed(a.intents)
    for _ in range(a.history):
        daemon_protocol_step(d, intent_cls, sid, next(counter), n, chunk)
    later = timed(a.intents)
    print(json.dumps({"metric": "daemon protocol ms per intent (submit, complete, release)", "impl": a.impl,
                      "lanes": a.lanes, "bytes": n, "chunk_bytes": chunk, "chunks": -(-n // chunk),
                      "relay_leases_per_intent": statistics.median(leases) if leases else 0,
                      "ms_per_intent": round(first, 3), "ms_per_intent_after_history": round(later, 3),
                      "history": a.history}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
