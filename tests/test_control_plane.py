"""Control plane on the CPU: planner parity with the reference's pinned
expectations, plan JSON, schema rules, fair-share scheduling, topology
parsing with fake probes / sysfs, and the daemon's state machine (leases,
status mismatch, cleanup cascade, reaping, reschedule generations, audit,
profiles, socket wire).  Mirrors test/cpp/test_planner.cpp,
test_planner_engine, test_schema, test_contract_schema, test_daemon_scheduler,
test_topology_provider, test_daemon_state and test_daemon_socket of the
reference with independent fixtures."""

import os
import tempfile
import threading
from dataclasses import asdict

import pytest

from pcie_pool_b200.daemon import InProcessDaemonClient, TurboBusDaemon
from pcie_pool_b200.plan_trace import plan_from_dict, transfer_plan_to_dict, validate_plan_dict
from pcie_pool_b200.planner_engine import PlannerEngine, PlannerEngineOptions
from pcie_pool_b200.scheduler.fairness import FAIRNESS_FALLBACK, charge_bytes
from pcie_pool_b200.schema import TransferIntent, TransferStatusState
from pcie_pool_b200.topology import (DaemonResourceInventory, FabricLinkRecord, GpuInventoryRecord, PciePathRecord,
                                    StaticTopologyProvider)
from pcie_pool_b200.topology.cuda_nvml import CudaNvmlTopologyProvider, fabric_links_from_matrix, pcie_tree

MiB = 1 << 20


def profile(direct, relays, d2h=None, rd2h=None):
    return {"target_device": 0, "direct_h2d_bw_gbps": direct, "direct_d2h_bw_gbps": d2h if d2h else direct,
            "relays": [{"relay_device": i + 1, "target_device": 0, "h2d_bw_gbps": bw,
                        "d2h_bw_gbps": (rd2h or relays)[i], "p2p_bw_gbps": 400.0, "effective_bw_gbps": bw,
                        "effective_d2h_bw_gbps": (rd2h or relays)[i], "p2p_enabled": True}
                       for i, bw in enumerate(relays)]}


def lane_chunks(plan):
    out = {}
    for a in plan.assignments:
        key = "direct" if a.path.kind == "direct" else a.path.relay_device
        out[key] = len(a.chunks)
    return out


# ---- planner ------------------------------------------------------------------------------------

def test_legacy_planner_reproduces_reference_splits():
    eng = PlannerEngine(PlannerEngineOptions(policy="legacy", use_concurrent_profile=False))
    plan = eng.plan(224 * MiB, 16 * MiB, profile(20.0, [40.0, 10.0]))
    assert lane_chunks(plan) == {"direct": 4, 1: 8, 2: 2}
    d2h = eng.plan(192 * MiB, 16 * MiB, profile(10.0, [20.0, 30.0], d2h=10.0, rd2h=[20.0, 30.0]), direction="d2h")
    assert lane_chunks(d2h) == {"direct": 2, 1: 4, 2: 6}


def test_planner_filters_and_min_chunks():
    eng = PlannerEngine(PlannerEngineOptions(policy="legacy", min_chunks_for_relay=4, use_concurrent_profile=False))
    small = eng.plan(48 * MiB, 16 * MiB, profile(20.0, [40.0]))  # 3 chunks < 4
    assert lane_chunks(small) == {"direct": 3}
    ratio = PlannerEngine(PlannerEngineOptions(policy="legacy", relay_min_direct_ratio=0.5,
                                               use_concurrent_profile=False))
    p = ratio.plan(160 * MiB, 16 * MiB, profile(20.0, [40.0, 5.0]))  # relay 2 below 0.5x direct
    assert set(lane_chunks(p)) == {"direct", 1}
    relay_only = ratio.plan(64 * MiB, 16 * MiB, profile(20.0, [40.0]), mode="relay")
    assert set(lane_chunks(relay_only)) == {1}


def test_planner_ranges_split_at_chunk_bytes():
    eng = PlannerEngine(PlannerEngineOptions(policy="legacy", use_concurrent_profile=False))
    plan = eng.plan_ranges([(0, 4096, 40 * MiB), (64 * MiB, 0, 8 * MiB)], 16 * MiB, profile(10.0, [10.0]))
    chunks = sorted((c.src_offset, c.dst_offset, c.bytes) for a in plan.assignments for c in a.chunks)
    assert chunks == [(0, 4096, 16 * MiB), (16 * MiB, 4096 + 16 * MiB, 16 * MiB),
                      (32 * MiB, 4096 + 32 * MiB, 8 * MiB), (64 * MiB, 0, 8 * MiB)]
    assert plan.total_bytes == 48 * MiB


def test_earliest_finish_balances_finish_times():
    eng = PlannerEngine(PlannerEngineOptions(policy="earliest_finish", use_concurrent_profile=False))
    plan = eng.plan(1024 * MiB, 16 * MiB, profile(50.0, [25.0, 25.0, 12.5]))
    n = lane_chunks(plan)
    t = {k: v * 16 / bw for k, v, bw in ((k, n[k], {"direct": 50.0, 1: 25.0, 2: 25.0, 3: 12.5}[k]) for k in n)}
    assert max(t.values()) - min(t.values()) <= 16 / 12.5 + 1e-9


def test_plan_json_roundtrip():
    eng = PlannerEngine(PlannerEngineOptions(policy="legacy", use_concurrent_profile=False))
    plan = eng.plan(100 * MiB, 16 * MiB, profile(20.0, [40.0, 10.0]))
    d = transfer_plan_to_dict(plan)
    validate_plan_dict(d)
    assert d["total_bytes"] == 100 * MiB and sum(a["bytes"] for a in d["assignments"]) == 100 * MiB
    assert transfer_plan_to_dict(plan_from_dict(d)) == d
    bad = dict(d, total_bytes=1)
    with pytest.raises(ValueError):
        validate_plan_dict(bad)


# ---- schema ----------------------------------------------------------------------------------------

def test_intent_rejects_physical_policy_hints_and_bad_ranges():
    base = dict(intent_id="i", job_id="j", session_id="s", source_buffer_id="a", destination_buffer_id="b",
                direction="h2d", total_bytes=10, ranges=({"src_offset": 0, "dst_offset": 0, "bytes": 10},))
    TransferIntent(**base)
    with pytest.raises(ValueError):
        TransferIntent(**{**base, "policy_hints": {"relay_gpus": [1]}})
    with pytest.raises(ValueError):
        TransferIntent(**{**base, "total_bytes": 11})
    with pytest.raises(ValueError):
        TransferIntent(**{**base, "direction": "sideways"})


def test_fairness_charges():
    assert charge_bytes(1000, "kv_cache", 0) == 750
    assert charge_bytes(1000, "training_state", 0) == 1250
    assert charge_bytes(1000, "generic", 9) == pytest.approx(1000 / 1.9)
    assert charge_bytes(1000, "generic", 50) == pytest.approx(1000 / 1.9)


# ---- topology --------------------------------------------------------------------------------------

B200_TOPO = ["\x1b[4mGPU0\tGPU1\tGPU2\tCPU Affinity\tNUMA Affinity\x1b[0m",
             "GPU0\t X \tNV18\tNV18\t0-31\t0", "GPU1\tNV18\t X \tNV18\t0-31\t0",
             "GPU2\tNV18\tSYS\t X \t0-31\t0", "", "Legend:", "  X    = Self"]


def test_fabric_links_from_topology_matrix():
    links = fabric_links_from_matrix({0, 1, 2}, B200_TOPO)
    pairs = {(l.src_device_id, l.dst_device_id): l for l in links}
    assert set(pairs) == {(0, 1), (0, 2), (1, 2)}
    assert all(l.fabric == "nvlink" and l.link_count == 18 and l.enabled for l in links)


class FakeProbe:
    def __init__(self, rows, matrix):
        self.rows, self.matrix = rows, matrix

    def query_gpu_inventory(self):
        return self.rows

    def query_topology_matrix(self):
        return self.matrix


def test_provider_with_fake_probe_and_sysfs(tmp_path):
    # sysfs: root port 0000:00:01.0 -> switch -> GPU 0000:1b:00.0
    real = tmp_path / "devices" / "pci0000:00" / "0000:00:01.0" / "0000:01:00.0" / "0000:1b:00.0"
    real.mkdir(parents=True)
    (real / "numa_node").write_text("1\n")
    (real / "current_link_speed").write_text("32.0 GT/s PCIe\n")
    (real / "current_link_width").write_text("16\n")
    link = tmp_path / "bus" / "pci" / "devices"
    link.mkdir(parents=True)
    os.symlink(real, link / "0000:1b:00.0")
    tree = pcie_tree("00000000:1B:00.0", tmp_path)
    assert tree["numa_node"] == 1 and tree["link_width"] == 16 and tree["negotiated_speed_gtps"] == 32.0
    assert tree["switch_hierarchy"] == ("0000:00:01.0", "0000:01:00.0")
    rows = [{"device_id": 0, "pci_bus_id": "00000000:1B:00.0", "pcie_link_gen_current": 5,
             "pcie_link_width_current": 16},
            {"device_id": 1, "pci_bus_id": "00000000:2B:00.0", "pcie_link_gen_current": 5,
             "pcie_link_width_current": 16}]
    now = [100.0]
    prov = CudaNvmlTopologyProvider(FakeProbe(rows, B200_TOPO[:3]), sysfs_root=str(tmp_path), now=lambda: now[0])
    inv = prov.snapshot()
    assert [g.device_id for g in inv.gpus] == [0, 1]
    p0 = next(p for p in inv.pcie_paths if p.device_id == 0)
    assert p0.numa_node == 1 and p0.bandwidth_gbps == pytest.approx(63.0, rel=0.01)
    assert inv.snapshot_id == prov.snapshot().snapshot_id  # cached within 30 s
    now[0] += 31
    assert prov.snapshot().version == 2


def test_relay_eligibility_reasons():
    inv = DaemonResourceInventory(
        gpus=(GpuInventoryRecord(0), GpuInventoryRecord(1), GpuInventoryRecord(2), GpuInventoryRecord(3)),
        pcie_paths=(PciePathRecord(0, bandwidth_gbps=63.0), PciePathRecord(1, bandwidth_gbps=63.0),
                    PciePathRecord(3, bandwidth_gbps=63.0)),
        fabric_links=(FabricLinkRecord(1, 0, fabric="nvswitch", bandwidth_gbps=900.0, enabled=True),
                      FabricLinkRecord(2, 0, fabric="nvswitch", bandwidth_gbps=900.0, enabled=True)),
        source="unit")
    el = inv.relay_eligibility(0, [0, 1, 2, 3, 9])
    assert [e["relay_gpu"] for e in el["eligible_relays"]] == [1]
    reasons = {r["relay_gpu"]: r["reason"] for r in el["filtered_relays"]}
    assert reasons == {0: "target gpu cannot relay", 9: "unknown gpu", 2: "missing pcie path",
                       3: "missing enabled fabric link"}


# ---- daemon state machine ----------------------------------------------------------------------------

class Clock:
    def __init__(self, t=1000.0):
        self.t = t

    def __call__(self):
        return self.t


def make_daemon(clock=None, relays=(1, 2, 3), inflight=64):
    d = TurboBusDaemon(relay_gpus=relays, max_inflight_chunks_per_relay=inflight,
                       topology_provider=StaticTopologyProvider(gpu_count=4), clock=clock or Clock())
    d.put_profile(0, list(relays), profile(20.0, [20.0] * len(relays)))
    return d


def planned(dc, job="job", total=64 * MiB, chunk=16 * MiB, mode="pool", direction="h2d", workload="generic",
            relays=(1, 2, 3)):
    s = dc.register_session(0, list(relays), max_inflight_chunks=64)
    assert s.ok, s.error
    sid = s.payload["session"]["session_id"]
    assert dc.register_job(job, session_id=sid).ok
    for name, kind, dev in (("src-" + job, "cpu_pinned", None), ("dst-" + job, "gpu", 0)):
        assert dc.register_buffer(name, job, kind, total, device_index=dev, address=4096,
                                  pinned=kind == "cpu_pinned").ok
    from pcie_pool_b200.transfer import TransferRequest

    req = TransferRequest.from_ranges([(0, 0, total)], chunk_bytes=chunk, direction=direction, mode=mode, job_id=job,
                                      metadata={"buffer_ids": ("src-" + job, "dst-" + job)})
    r = dc.plan_transfer_request(sid, req, mode=mode)
    assert r.ok, r.error
    return sid, r.payload


def test_plan_issues_leases_and_completion_releases():
    dc = InProcessDaemonClient(make_daemon())
    sid, p = planned(dc)
    assert len(p["lease_tokens"]) == 3 and p["plan_generation"] == 1
    tid = p["transfer_id"]
    desc = dc.describe().payload
    assert len(desc["reservations"]) == 3
    assert sum(q["active_chunks"] for q in desc["relay_quotas"].values()) > 0
    r = dc.transfer_status(tid, state="complete", bytes_completed=64 * MiB)
    assert r.ok
    # completion leaves the leases to their holder, which releases them
    assert len(dc.describe().payload["reservations"]) == 3
    for t in p["lease_tokens"]:
        assert dc.release_transfer(t["lease_id"]).ok
    desc = dc.describe().payload
    assert desc["reservations"] == {} and all(q["active_chunks"] == 0 for q in desc["relay_quotas"].values())
    events = [a["event_type"] for a in desc["audit_records"]]
    assert "worker_completion" in events
    assert all(len(a) >= 27 for a in desc["audit_records"])


def test_status_byte_mismatch_fails_and_releases():
    dc = InProcessDaemonClient(make_daemon())
    _sid, p = planned(dc)
    r = dc.transfer_status(p["transfer_id"], state="complete", bytes_completed=1)
    assert not r.ok
    st = dc.transfer_status(p["transfer_id"]).payload["status"]
    assert st["state"] == "failed"
    desc = dc.describe().payload
    assert desc["reservations"] == {}
    assert any(a["event_type"] == "detected_mismatch" for a in desc["audit_records"])
    # terminal statuses are immutable
    assert not dc.transfer_status(p["transfer_id"], state="complete", bytes_completed=64 * MiB).ok


def test_cleanup_cascade_by_job_cancels_transfers():
    dc = InProcessDaemonClient(make_daemon())
    _sid, p = planned(dc)
    r = dc.cleanup(target_kind="job", target_id="job", reason="test", force=True)
    assert r.ok
    st = dc.transfer_status(p["transfer_id"]).payload["status"]
    assert st["state"] == "canceled"
    desc = dc.describe().payload
    assert desc["reservations"] == {} and "job" not in desc["jobs"]


def test_expired_leases_are_reaped():
    clock = Clock()
    d = make_daemon(clock)
    dc = InProcessDaemonClient(d)
    _sid, p = planned(dc)
    tok = p["lease_tokens"][0]
    assert dc.validate_lease(tok["lease_id"], tok["token"]).ok
    assert not dc.validate_lease(tok["lease_id"], "wrong").ok
    clock.t += 31.0
    reaped = d.reap_expired_leases()
    assert len(reaped) == 3
    assert not dc.validate_lease(tok["lease_id"], tok["token"]).ok


def test_reschedule_bumps_generation():
    dc = InProcessDaemonClient(make_daemon())
    _sid, p = planned(dc)
    r = dc.reschedule_transfer(p["transfer_id"])
    assert r.ok, r.error
    assert r.payload["plan_generation"] == 2
    old = p["lease_tokens"][0]
    assert not dc.validate_lease(old["lease_id"], old["token"]).ok


def test_fairness_prefers_direct_for_a_job_over_its_share():
    dc = InProcessDaemonClient(make_daemon(inflight=4096))
    planned(dc, job="small", total=16 * MiB, relays=(1,))
    _sid, heavy1 = planned(dc, job="heavy", total=512 * MiB, relays=(2,))
    _sid, heavy2 = planned(dc, job="heavy", total=512 * MiB, relays=(3,))
    reasons = [heavy2["decision"].get("fallback_reason")] + [heavy2["stats"].get("fallback_reason")]
    assert FAIRNESS_FALLBACK in reasons or not heavy2["lease_tokens"]


def test_profile_cache_get_put_invalidate():
    d = make_daemon()
    assert d.get_profile(0, [1, 2, 3]).ok
    r = d.invalidate_profile(0, [1, 2, 3])
    assert r.ok and r.payload["removed"]
    assert d.get_profile(0, [1, 2, 3]).payload["profile"] is None


def test_socket_wire_roundtrip_with_peer_identity():
    from pcie_pool_b200.daemon.client import TurboBusDaemonClient
    from pcie_pool_b200.daemon.wire import serve_unix

    d = make_daemon()
    tmp = tempfile.mkdtemp(prefix="ppb-d-")
    sock = os.path.join(tmp, "d.sock")
    stop, ready = threading.Event(), threading.Event()
    t = threading.Thread(target=serve_unix, args=(d, sock), kwargs={"stop_event": stop, "ready_event": ready},
                         daemon=True)
    t.start()
    assert ready.wait(5)
    try:
        c = TurboBusDaemonClient(sock)
        s = c.register_session(0, [1, 2], max_inflight_chunks=8)
        assert s.ok, s.error
        assert c.register_job("wire-job", session_id=s.payload["session"]["session_id"]).ok
        peers = d.describe().payload["job_peer_identities"]
        assert peers["wire-job"]["process_id"] == os.getpid() and peers["wire-job"]["authenticated"]
        inv = c.get_inventory()
        assert inv.ok
        bad = c.send_raw(b"{not json}\n") if hasattr(c, "send_raw") else None
        assert bad is None or not bad.ok
    finally:
        stop.set()
        t.join(5)


def test_reserve_socket_refuses_a_live_socket_and_reclaims_a_stale_one(tmp_path):
    from pcie_pool_b200.daemon.server import reserve_socket

    path = str(tmp_path / "d.sock")
    live = reserve_socket(path)
    try:
        with pytest.raises(RuntimeError, match="running process"):
            reserve_socket(path)
    finally:
        live.close()
    assert os.path.exists(path)  # closed listener leaves a stale file behind
    again = reserve_socket(path)
    again.close()


def test_native_and_python_planners_agree():
    """The C++ planner and its Python twin give the same chunk assignment and
    the same chunk-size choice on random lane models."""
    import numpy as np

    from pcie_pool_b200._native import native
    from pcie_pool_b200.planner_engine import _estimate, assign_python

    C = native()
    rng = np.random.default_rng(11)
    for _ in range(40):
        lanes = int(rng.integers(1, 9))
        sizes = [int(x) for x in rng.choice([MiB, 4 * MiB, 16 * MiB], size=int(rng.integers(1, 200)))]
        bw = [float(x) for x in rng.uniform(5.0, 60.0, lanes)]
        lat = [float(x) for x in rng.uniform(0.0, 3e-5, lanes)]
        for policy, pol in (("legacy", C.POLICY_LEGACY), ("earliest_finish", C.POLICY_EARLIEST_FINISH)):
            lat_p = [] if policy == "legacy" else lat
            native_idx = [int(i) for i in C.assign_chunks(np.asarray(sizes, dtype=np.uint64), bw, lat_p, pol)]
            assert native_idx == assign_python(sizes, bw, lat_p, policy), policy
        cands = [MiB, 4 * MiB, 16 * MiB, 64 * MiB]
        total = int(rng.integers(1, 64)) * 16 * MiB
        assert int(C.choose_chunk_bytes(total, cands, bw, lat)) == min(cands, key=lambda c: _estimate(total, c, bw, lat))


def test_plan_records_convert_exactly_like_dataclasses_asdict():
    from dataclasses import asdict, fields

    from pcie_pool_b200.planner_types import PlannerChunk, PlannerPath, PlannerPathAssignment

    path = PlannerPath("relay", "h2d", 0, 3, 26.0, 25.0, 700.0, 26.0, True, "nvswitch")
    assert path.as_dict() == asdict(path) and list(path.as_dict()) == [f.name for f in fields(PlannerPath)]
    a = PlannerPathAssignment(path, (PlannerChunk(0, 0, 8, 3), PlannerChunk(8, 8, 4)))
    d = a.as_dict()
    assert d["path"] == asdict(path) and d["chunks"] == [asdict(c) for c in a.chunks]
    assert (d["bytes"], d["chunk_count"]) == (12, 2)
