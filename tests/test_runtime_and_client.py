"""The runtime facade over a stand-in engine and the public intent client
over a stand-in daemon: plan validation into lanes, handles and their
status, stats mapping, tuning / profile JSON, daemon profile conversion and
freshness, range helpers; receipts, failures and mismatches at the public
boundary.  Behaviours follow unit/test_runtime_engine.py and
unit/test_public_client_api.py of the reference with independent fakes."""

from __future__ import annotations

import json
import time
from types import SimpleNamespace

import numpy as np
import pytest

from pcie_pool_b200 import TransferIntent, TurboBusClient
from pcie_pool_b200.runtime_engine import (PoolRuntime, RuntimeOptions, TransferHandle, daemon_profile_is_fresh,
                                           plan_to_lanes, profile_from_daemon_entry, profile_to_daemon_dict,
                                           range_fields, stats_from_result, validate_ranges)
from pcie_pool_b200.schema import DaemonResponse, TransferReceipt

MiB = 1 << 20


def plan(chunks_direct=((0, 0, 4 * MiB),), chunks_relay=((4 * MiB, 4 * MiB, 4 * MiB),), total=None, relay=2):
    def asg(kind, chunks, rd):
        return {"path": {"kind": kind, "direction": "h2d", "target_device": 0, "relay_device": rd, "enabled": True},
                "chunks": [{"src_offset": s, "dst_offset": d, "bytes": n} for s, d, n in chunks]}

    a = [asg("direct", chunks_direct, -1)] + ([asg("relay", chunks_relay, relay)] if chunks_relay else [])
    n = sum(c[2] for c in chunks_direct) + sum(c[2] for c in chunks_relay or ())
    return {"total_bytes": n if total is None else total, "chunk_bytes": 4 * MiB, "assignments": a}


# ---- plans into lanes --------------------------------------------------------------------------------

def test_plan_to_lanes_keeps_the_daemon_assignment():
    lanes = plan_to_lanes(plan(), 0, source_bytes=8 * MiB, destination_bytes=8 * MiB)
    assert [(l.device, l.src_off.tolist(), l.bytes.tolist()) for l in lanes] == [
        (0, [0], [4 * MiB]), (2, [4 * MiB], [4 * MiB])]


@pytest.mark.parametrize("kw,msg", [
    ({"total": 1}, "total_bytes"),
    ({"chunks_relay": ((4 * MiB, 4 * MiB, 0),)}, "bytes positive"),
    ({"chunks_direct": ((-1, 0, 4 * MiB),)}, "non-negative"),
])
def test_plan_to_lanes_rejections(kw, msg):
    with pytest.raises(ValueError, match=msg):
        plan_to_lanes(plan(**kw), 0)


def test_plan_to_lanes_bounds_and_disabled_paths():
    with pytest.raises(ValueError, match="past source"):
        plan_to_lanes(plan(), 0, source_bytes=6 * MiB)
    with pytest.raises(ValueError, match="past destination"):
        plan_to_lanes(plan(), 0, destination_bytes=6 * MiB)
    p = plan()
    p["assignments"][1]["path"]["enabled"] = False
    with pytest.raises(ValueError, match="disabled"):
        plan_to_lanes(p, 0)


# ---- runtime over a stand-in engine ------------------------------------------------------------------

class Engine:
    def __init__(self, fail=False):
        self.fail, self.submitted = fail, []

    def submit(self, direction, target, host_ptr, host_bytes, dev_ptr, dev_bytes, lanes, checksum=False):
        self.submitted.append((direction, target, [l.device for l in lanes], checksum))
        return len(self.submitted)

    def wait(self, tid):
        lanes = [SimpleNamespace(device=0, direct=True, bytes=4 * MiB, chunks=1, cuda_ms=1.0),
                 SimpleNamespace(device=2, direct=False, bytes=4 * MiB, chunks=1, cuda_ms=2.0)]
        return SimpleNamespace(ok=not self.fail, error="lane 2 timed out" if self.fail else "", bytes=8 * MiB,
                               submit_to_complete_ms=4.0, cuda_ms=2.0, gib_per_s=4.0, checksums=np.zeros((2, 2)),
                               lanes=lanes)


def runtime(engine):
    rt = PoolRuntime(RuntimeOptions(chunk_bytes=4 * MiB))
    rt._engine, rt.target_device, rt.relay_devices = engine, 0, [1, 2]
    return rt


def test_runtime_wait_marks_complete_and_maps_stats():
    eng = Engine()
    rt = runtime(eng)
    h = TransferHandle(rt, rt.fetch_plan_to_gpu(4096, 8 * MiB, 8192, 8 * MiB, plan()))
    assert h.status == "submitted" and not h.done
    h.wait()
    assert h.done and h.status == "complete"
    st = h.stats
    assert (st.bytes, st.direct_bytes, st.relay_bytes, st.relay_devices) == (8 * MiB, 4 * MiB, 4 * MiB, [2])
    assert st.submit_gib_per_second == pytest.approx((8 * MiB / (1 << 30)) / 0.004)
    assert eng.submitted[0] == (0, 0, [0, 2], True) and rt.last_plan()["total_bytes"] == 8 * MiB
    h.wait()  # idempotent once complete


def test_runtime_wait_failure_marks_failed():
    rt = runtime(Engine(fail=True))
    h = TransferHandle(rt, rt.offload_plan_to_cpu(8192, 8 * MiB, 4096, 8 * MiB, plan()))
    with pytest.raises(RuntimeError, match="lane 2 timed out"):
        h.wait()
    assert h.status == "failed" and "lane 2" in h.error
    with pytest.raises(ValueError, match="wait first"):
        rt.stats(SimpleNamespace(id=99))


def test_stats_from_result_per_path():
    res = Engine().wait(1)
    st = stats_from_result(res, "h2d", 0)
    kinds = [(p.kind, p.relay_device, p.bytes) for p in st.path_stats]
    assert kinds == [("direct", -1, 4 * MiB), ("relay", 2, 4 * MiB)]
    assert st.path_stats[1].gib_per_second == pytest.approx((4 * MiB / (1 << 30)) / 0.002)


# ---- options, profiles, ranges ------------------------------------------------------------------------

def test_runtime_options_from_tuning_and_profile_json(tmp_path):
    t = tmp_path / "tune.json"
    t.write_text(json.dumps({"best": {"chunk_bytes": 8 * MiB, "staging_slots": 4}}))
    o = RuntimeOptions.from_tuning_json(t)
    assert (o.chunk_bytes, o.staging_slots) == (8 * MiB, 4)
    p = tmp_path / "prof.json"
    p.write_text(json.dumps({"config": {"chunk_bytes": 2 * MiB, "staging_slots": 2, "profile_bytes": 64 * MiB}}))
    o = RuntimeOptions.from_profile_json(p)
    assert (o.chunk_bytes, o.staging_slots, o.profile_bytes) == (2 * MiB, 2, 64 * MiB)
    assert o.planner_options().min_chunks_for_relay == o.min_chunks_for_relay


def test_profile_round_trip_and_freshness():
    prof = SimpleNamespace(target_device=0, direct_h2d_bw_gbps=50.0, direct_d2h_bw_gbps=52.0,
                           relays=[SimpleNamespace(relay_device=1, target_device=0, h2d_bw_gbps=48.0,
                                                   d2h_bw_gbps=49.0, p2p_bw_gbps=700.0, effective_bw_gbps=48.0,
                                                   effective_d2h_bw_gbps=49.0, p2p_enabled=True)],
                           concurrent={"h2d": {"aggregate_gb_per_s": 98.0}})
    d = profile_to_daemon_dict(prof)
    assert d["relays"][0]["p2p_enabled"] is True and d["concurrent"]["h2d"]["aggregate_gb_per_s"] == 98.0
    back = profile_from_daemon_entry({"profile": d}, 0)
    assert back.direct_h2d_bw_gbps == 50.0 and back.relays[0].effective_d2h_bw_gbps == 49.0
    with pytest.raises(ValueError, match="direct_h2d_bw_gbps"):
        profile_from_daemon_entry({"profile": {**d, "direct_h2d_bw_gbps": 0}}, 0)
    with pytest.raises(ValueError, match="no profile"):
        profile_from_daemon_entry({}, 0)
    assert daemon_profile_is_fresh({"updated_at": time.time() - 10}, 60)
    assert not daemon_profile_is_fresh({"updated_at": time.time() - 120}, 60)
    assert not daemon_profile_is_fresh({}, 60) and daemon_profile_is_fresh({}, 0)


def test_range_helpers():
    assert range_fields({"src_offset": 1, "dst_offset": 2, "bytes": 3}) == (1, 2, 3)
    assert range_fields((4, 5, 6)) == (4, 5, 6)
    assert range_fields(SimpleNamespace(src_offset=7, dst_offset=8, bytes=9)) == (7, 8, 9)
    with pytest.raises(ValueError, match="tuples"):
        range_fields((1, 2))
    assert validate_ranges([(0, 0, 4), (4, 8, 4)], 8, 12) == [(0, 0, 4), (4, 8, 4)]
    for bad, msg in (([(6, 0, 4)], "source"), ([(0, 10, 4)], "destination"), ([], "at least one")):
        with pytest.raises(ValueError, match=msg):
            validate_ranges(bad, 8, 12)


# ---- public client over a stand-in daemon ------------------------------------------------------------------

def _intent(iid="i1"):
    return TransferIntent(iid, "j", "s", "a", "b", "h2d", 16, ({"src_offset": 0, "dst_offset": 0, "bytes": 16},))


def _receipt(iid, state="complete"):
    return {"receipt_id": "r", "ticket_id": "t", "intent_id": iid, "decision_id": "d", "topology_snapshot_id": "x",
            "job_id": "j", "session_id": "s", "state": state, "bytes_total": 16,
            "bytes_completed": 16 if state == "complete" else 0}


class Daemon:
    def __init__(self, reply=None):
        self.calls, self.reply = [], reply

    def submit_transfer_intent(self, intent):
        self.calls.append(("submit", intent.intent_id))
        return self.reply or DaemonResponse(ok=True, payload={"receipt": _receipt(intent.intent_id, "running")})

    def wait_transfer_receipt(self, intent_id, timeout_seconds=None):
        self.calls.append(("wait", intent_id, timeout_seconds))
        return self.reply or DaemonResponse(ok=True, payload={"receipt": _receipt(intent_id)})


def test_client_submit_wait_and_transfer():
    d = Daemon()
    c = TurboBusClient(daemon=d)
    r = c.submit(_intent())
    assert isinstance(r, TransferReceipt) and r.state.value == "running"
    assert c.wait("i1", timeout_seconds=3).state.value == "complete"
    assert c.transfer(_intent("i2"), timeout_seconds=7).intent_id == "i2"
    assert d.calls[-1] == ("wait", "i2", 7)
    with pytest.raises(TypeError):
        c.submit({"intent_id": "x"})
    with pytest.raises(ValueError):
        TurboBusClient()
    with pytest.raises(ValueError):
        TurboBusClient(daemon=d, socket_path="/tmp/x")


def test_client_failure_and_mismatch_at_the_public_boundary():
    with pytest.raises(RuntimeError, match="no capacity"):
        TurboBusClient(daemon=Daemon(DaemonResponse(ok=False, error="no capacity"))).submit(_intent())
    wrong = Daemon(DaemonResponse(ok=True, payload={"receipt": _receipt("other")}))
    with pytest.raises(ValueError, match="does not match"):
        TurboBusClient(daemon=wrong).wait("i1")
    extra = Daemon(DaemonResponse(ok=True, payload={"receipt": {**_receipt("i1"), "surprise": 1}}))
    with pytest.raises(ValueError, match="unknown fields"):
        TurboBusClient(daemon=extra).wait("i1")
    with pytest.raises(ValueError, match="missing receipt"):
        TurboBusClient(daemon=Daemon(DaemonResponse(ok=True, payload={}))).wait("i1")
