"""The daemon's state machine in-process, one rule per test: sessions and
relay capacity, job / buffer ownership against authenticated peers, plans
and their leases, worker authorization checks, terminal statuses, manual
reservations, reaping, delayed admission and rescheduling, intents,
cleanup targets, profiles and audit records.  The behaviours are the ones
integration/test_daemon_state.py of the reference covers; the fixtures and
cases here are independent."""

from __future__ import annotations

import pytest

from pcie_pool_b200.daemon import InProcessDaemonClient, TurboBusDaemon
from pcie_pool_b200.schema import PeerIdentity, TransferIntent, WorkerTransferAuthorizationRequest
from pcie_pool_b200.topology import StaticTopologyProvider
from pcie_pool_b200.transfer import TransferRequest
from pcie_pool_b200.planner_types import assignment_chunks

MiB = 1 << 20


class Clock:
    def __init__(self, t: float = 1000.0) -> None:
        self.t = t

    def __call__(self) -> float:
        return self.t


def profile(n_relays: int = 3, bw: float = 20.0) -> dict:
    return {"target_device": 0, "direct_h2d_bw_gbps": bw, "direct_d2h_bw_gbps": bw,
            "relays": [{"relay_device": r, "target_device": 0, "h2d_bw_gbps": bw, "d2h_bw_gbps": bw,
                        "p2p_bw_gbps": 400.0, "effective_bw_gbps": bw, "effective_d2h_bw_gbps": bw,
                        "p2p_enabled": True} for r in range(1, n_relays + 1)]}


def daemon(clock=None, sessions_per_relay: int = 4, inflight: int = 4096, **kw) -> TurboBusDaemon:
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_sessions_per_relay=sessions_per_relay,
                       max_inflight_chunks_per_relay=inflight, topology_provider=StaticTopologyProvider(gpu_count=4),
                       clock=clock or Clock(), **kw)
    d.put_profile(0, [1, 2, 3], profile())
    return d


def peer(user: str, pid: int = 100) -> PeerIdentity:
    return PeerIdentity(authenticated=True, source="so_peercred", user_id=user, process_id=pid)


def setup_job(d: TurboBusDaemon, job: str = "job", relays=(1, 2, 3), total: int = 64 * MiB, who=None,
              inflight: int = 64) -> str:
    s = d.register_session(0, list(relays), max_inflight_chunks=inflight, peer_identity=who)
    assert s.ok, s.error
    sid = s.payload["session"]["session_id"]
    assert d.register_job(job, session_id=sid, peer_identity=who).ok
    for name, kind, dev in ((f"src-{job}", "cpu_pinned", None), (f"dst-{job}", "gpu", 0)):
        r = d.register_buffer(name, job, kind, total, device_index=dev, address=4096, pinned=kind == "cpu_pinned",
                              peer_identity=who)
        assert r.ok, r.error
    return sid


def plan(d: TurboBusDaemon, sid: str, job: str = "job", total: int = 64 * MiB, chunk: int = 16 * MiB,
         mode: str = "pool", direction: str = "h2d", **kw):
    return d.plan_transfer(sid, total, chunk, mode=mode, direction=direction, job_id=job,
                           buffer_ids=[f"src-{job}", f"dst-{job}"], **kw)


# ---- sessions -------------------------------------------------------------------------------------

def test_session_rejects_unknown_relays_and_bad_inflight():
    d = daemon()
    assert "unavailable" in d.register_session(0, [7]).error
    assert "positive" in d.register_session(0, [1], max_inflight_chunks=0).error


def test_relay_session_capacity_is_enforced_and_freed_on_close():
    d = daemon(sessions_per_relay=1)
    first = d.register_session(0, [1])
    assert first.ok
    assert not d.register_session(0, [1]).ok, "relay 1 already has its one session"
    assert d.register_session(0, [2]).ok, "other relays are unaffected"
    assert d.close_session(first.payload["session"]["session_id"]).ok
    assert d.register_session(0, [1]).ok


def test_close_unknown_session_fails():
    assert not daemon().close_session("nope").ok


# ---- jobs, buffers, peers ------------------------------------------------------------------------

def test_job_binds_to_authenticated_peer_and_rejects_spoofed_user():
    d = daemon()
    alice = peer("alice")
    r = d.register_job("j", user_id="alice", peer_identity=alice)
    assert r.ok and r.payload["job"]["user_id"] == "alice"
    assert "does not match" in d.register_job("j2", user_id="mallory", peer_identity=alice).error


def test_job_on_unknown_session_fails():
    assert "unknown session" in daemon().register_job("j", session_id="missing").error


def test_buffer_requires_known_job_and_owner():
    d = daemon()
    assert "unknown job" in d.register_buffer("b", "ghost", "gpu", 10, device_index=0).error
    alice, bob = peer("alice", 1), peer("bob", 2)
    assert d.register_job("j", peer_identity=alice).ok
    assert not d.register_buffer("b", "j", "gpu", 10, device_index=0, peer_identity=bob).ok
    assert d.register_buffer("b", "j", "gpu", 10, device_index=0, peer_identity=alice).ok


def test_buffer_cannot_be_replaced_while_leased():
    d = daemon()
    sid = setup_job(d)
    assert plan(d, sid).ok
    r = d.register_buffer("src-job", "job", "cpu_pinned", 64 * MiB, address=4096, pinned=True)
    assert "active lease" in r.error


def test_plan_rejects_buffers_of_another_job():
    d = daemon()
    sid = setup_job(d, "a")
    setup_job(d, "b")
    r = d.plan_transfer(sid, 64 * MiB, 16 * MiB, job_id="a", buffer_ids=["src-b", "dst-b"])
    assert not r.ok


# ---- plans and leases -----------------------------------------------------------------------------

def test_pool_plan_covers_every_byte_and_leases_each_relay():
    d = daemon()
    sid = setup_job(d)
    r = plan(d, sid)
    assert r.ok, r.error
    p = r.payload
    chunks = [c for a in p["plan"]["assignments"] for c in assignment_chunks(a)]
    assert sum(c["bytes"] for c in chunks) == 64 * MiB
    assert sorted(t["relay_gpu"] for t in p["lease_tokens"]) == [1, 2, 3]
    assert p["plan_generation"] == 1 and p["transfer_id"]


def test_direct_mode_plan_has_no_leases_and_a_ticket():
    d = daemon()
    sid = setup_job(d)
    r = plan(d, sid, mode="direct")
    assert r.ok and not r.payload["lease_tokens"]
    tid = r.payload["transfer_id"]
    assert all(a["path"]["kind"] == "direct" for a in r.payload["plan"]["assignments"])
    assert r.payload["ticket"]["metadata"]["transfer_id"] == tid


def test_session_chunk_quota_bounds_relay_chunks():
    d = daemon()
    sid = setup_job(d, inflight=2)
    r = plan(d, sid, total=256 * MiB, chunk=16 * MiB)
    assert r.ok
    relay_chunks = sum(len(assignment_chunks(a)) for a in r.payload["plan"]["assignments"] if a["path"]["kind"] == "relay")
    assert relay_chunks <= 2 or not r.payload["lease_tokens"]


def test_validate_lease_checks_every_field():
    d = daemon()
    sid = setup_job(d)
    tok = plan(d, sid).payload["lease_tokens"][0]
    lid, t = tok["lease_id"], tok["token"]
    assert d.validate_lease(lid, t, session_id=sid, relay_gpu=tok["relay_gpu"], job_id="job").ok
    assert "unknown lease" in d.validate_lease("nope", t).error
    assert "token" in d.validate_lease(lid, "bad").error
    assert "session" in d.validate_lease(lid, t, session_id="other").error
    assert "relay" in d.validate_lease(lid, t, relay_gpu=99).error
    assert "job" in d.validate_lease(lid, t, job_id="other").error
    assert "buffer" in d.validate_lease(lid, t, buffer_ids=["dst-job", "src-job"]).error


def test_lease_expires_with_the_clock():
    clock = Clock()
    d = daemon(clock)
    sid = setup_job(d)
    tok = plan(d, sid).payload["lease_tokens"][0]
    clock.t += 3600.0
    r = d.validate_lease(tok["lease_id"], tok["token"])
    assert not r.ok and "expired" in r.error


# ---- worker authorization -------------------------------------------------------------------------

def _auth_request(p: dict, sid: str, **over) -> WorkerTransferAuthorizationRequest:
    tok = p["lease_tokens"][0]
    kw = dict(transfer_id=p["transfer_id"], lease_id=tok["lease_id"], token=tok["token"], session_id=sid,
              job_id="job", src_buffer_id="src-job", dst_buffer_id="dst-job", direction="h2d")
    kw.update(over)
    return WorkerTransferAuthorizationRequest(**kw)


def test_worker_authorization_issues_ticket_and_staging_records():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    r = d.authorize_worker_transfer(_auth_request(p, sid))
    assert r.ok, r.error
    assert r.payload["ticket"]["metadata"]["issuer"] == "turbobus-daemon"
    assert len(r.payload["staging_records"]) == len(p["lease_tokens"])
    events = [a["event_type"] for a in d.describe().payload["audit_records"]]
    assert events.count("relay_authorized") == len(p["lease_tokens"])


@pytest.mark.parametrize("field,value,msg", [("token", "forged", "token"), ("session_id", "other", "session"),
                                             ("job_id", "other", "job"), ("direction", "d2h", "direction"),
                                             ("src_buffer_id", "dst-job", "buffer")])
def test_worker_authorization_rejects_mismatches(field, value, msg):
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    r = d.authorize_worker_transfer(_auth_request(p, sid, **{field: value}))
    assert not r.ok and msg in r.error, r.error


def test_worker_authorization_rejects_terminal_transfer():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    assert d.transfer_status(p["transfer_id"], state="canceled").ok
    assert not d.authorize_worker_transfer(_auth_request(p, sid)).ok


def test_worker_authorization_rejects_another_peer():
    d = daemon()
    alice = peer("alice", 1)
    sid = setup_job(d, who=alice)
    p = plan(d, sid, peer_identity=alice).payload
    assert not d.authorize_worker_transfer(_auth_request(p, sid), peer_identity=peer("bob", 2)).ok
    assert d.authorize_worker_transfer(_auth_request(p, sid), peer_identity=alice).ok


# ---- statuses -------------------------------------------------------------------------------------

def test_status_moves_forward_and_terminal_is_final():
    d = daemon()
    sid = setup_job(d)
    tid = plan(d, sid).payload["transfer_id"]
    assert d.transfer_status(tid).payload["status"]["state"] == "submitted"
    assert d.transfer_status(tid, state="running", bytes_completed=MiB).ok
    assert d.transfer_status(tid, state="complete", bytes_completed=64 * MiB).ok
    # repeating the same terminal update is accepted, a different one is not
    assert d.transfer_status(tid, state="complete", bytes_completed=64 * MiB).ok
    assert not d.transfer_status(tid, state="failed").ok
    assert "unknown transfer" in d.transfer_status("nope").error


def test_failed_status_releases_leases_and_audits_reason():
    d = daemon()
    sid = setup_job(d)
    tid = plan(d, sid).payload["transfer_id"]
    assert d.transfer_status(tid, state="failed", error="lane 2 timed out").ok
    desc = d.describe().payload
    assert desc["reservations"] == {}
    fails = [a for a in desc["audit_records"] if a["event_type"] == "worker_failure"]
    assert fails and fails[-1]["failure_reason"] == "lane 2 timed out"


# ---- manual reservations ----------------------------------------------------------------------------

def test_manual_reservation_rules():
    d = daemon()
    sid = d.register_session(0, [1], max_inflight_chunks=4).payload["session"]["session_id"]
    assert "not assigned" in d.reserve_transfer(sid, 2, 1).error
    assert "limit" in d.reserve_transfer(sid, 1, 5).error
    assert "positive" in d.reserve_transfer(sid, 1, 0).error
    assert "direction" in d.reserve_transfer(sid, 1, 1, direction="sideways").error
    r = d.reserve_transfer(sid, 1, 3, bytes_=3 * MiB, direction="h2d")
    assert r.ok
    assert "quota" in d.reserve_transfer(sid, 1, 2).error, "3 of 4 session chunks are taken"
    assert d.release_transfer(r.payload["reservation"]["reservation_id"]).ok
    assert d.reserve_transfer(sid, 1, 4).ok
    assert "unknown reservation" in d.release_transfer("nope").error


def test_release_of_a_planned_lease_requires_completion():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    lid = p["lease_tokens"][0]["lease_id"]
    assert "not complete" in d.release_transfer(lid).error
    assert d.transfer_status(p["transfer_id"], state="complete", bytes_completed=64 * MiB).ok
    assert d.release_transfer(lid).ok


# ---- reaping, expiry, reschedule ------------------------------------------------------------------

def test_stale_sessions_are_reaped_after_timeout():
    clock = Clock()
    d = daemon(clock, session_timeout_seconds=10.0)
    sid = d.register_session(0, [1]).payload["session"]["session_id"]
    clock.t += 11.0
    assert sid in d.reap_stale_sessions()
    assert "unknown" in d.reserve_transfer(sid, 1, 1).error


def test_reschedule_makes_old_leases_stale_and_issues_new_ones():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    r = d.reschedule_transfer(p["transfer_id"])
    assert r.ok and r.payload["plan_generation"] == 2
    old = p["lease_tokens"][0]
    assert not d.validate_lease(old["lease_id"], old["token"]).ok
    for tok in r.payload["lease_tokens"]:
        assert d.validate_lease(tok["lease_id"], tok["token"]).ok
    assert not d.reschedule_transfer("nope").ok


def test_reschedule_of_terminal_transfer_fails():
    d = daemon()
    sid = setup_job(d)
    tid = plan(d, sid).payload["transfer_id"]
    assert d.transfer_status(tid, state="canceled").ok
    assert "terminal" in d.reschedule_transfer(tid).error


def test_delayed_admission_waits_for_a_busy_relay_then_reschedule_admits():
    """With delayed admission a plan through a relay whose link is busy is
    parked (no leases); once the busy transfer ends, rescheduling admits it
    (intents are re-planned by the daemon itself)."""
    d = daemon(inflight=4096)
    d.put_profile(0, [1], profile(1))
    sid_a = setup_job(d, "a", relays=(1,))
    a = plan(d, sid_a, "a").payload
    assert a["lease_tokens"]
    sid_b = setup_job(d, "b", relays=(1,))
    b = plan(d, sid_b, "b", allow_delayed_admission=True).payload

    def admission_state(tid):
        recs = d.describe().payload["runtime_resource_state"]["transfers"]
        return next(r["admission_state"] for r in recs if r["transfer_id"] == tid)

    if b["admission"]["state"] == "delayed":
        assert not b["lease_tokens"] and admission_state(b["transfer_id"]) == "delayed"
        assert d.transfer_status(a["transfer_id"], state="complete", bytes_completed=64 * MiB).ok
        for t in a["lease_tokens"]:
            d.release_transfer(t["lease_id"])
        r = d.reschedule_transfer(b["transfer_id"])
        assert r.ok and r.payload["plan_generation"] == 2
        assert admission_state(b["transfer_id"]) == "admitted"
    else:  # the planner left the busy relay out instead
        assert all(t["relay_gpu"] != 1 for t in b["lease_tokens"])


# ---- intents ----------------------------------------------------------------------------------------

def _intent(sid: str, iid: str = "i1", total: int = 32 * MiB) -> TransferIntent:
    return TransferIntent(iid, "job", sid, "src-job", "dst-job", "h2d", total,
                          ({"src_offset": 0, "dst_offset": 0, "bytes": total},), workload_kind="model_weights",
                          metadata={"chunk_bytes": 8 * MiB})


def test_intent_is_idempotent_by_id_and_conflicts_are_rejected():
    d = daemon()
    sid = setup_job(d)
    r1 = d.submit_transfer_intent(_intent(sid))
    assert r1.ok, r1.error
    r2 = d.submit_transfer_intent(_intent(sid))
    assert r2.ok and r2.payload["transfer_id"] == r1.payload["transfer_id"]
    r3 = d.submit_transfer_intent(_intent(sid, total=16 * MiB))
    assert not r3.ok and "different" in r3.error


def test_intent_receipt_carries_trace_metadata():
    d = daemon()
    sid = setup_job(d)
    r = d.submit_transfer_intent(_intent(sid))
    rec = d.wait_transfer_receipt("i1").payload["receipt"]
    assert rec["intent_id"] == "i1"
    md = rec["metadata"]
    for k in ("transfer_id", "admission_state", "plan_generation"):
        assert k in md, k
    assert md["transfer_id"] == r.payload["transfer_id"]
    assert "unknown" in d.wait_transfer_receipt("nope").error or not d.wait_transfer_receipt("nope").ok


# ---- cleanup ----------------------------------------------------------------------------------------

def test_cleanup_targets_and_force():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    assert not d.cleanup("job", "ghost", "t").ok
    assert d.cleanup("job", "ghost", "t", force=True).ok
    assert not d.cleanup("planet", "x", "t").ok
    r = d.cleanup("reservation", p["lease_tokens"][0]["lease_id"], "operator")
    assert r.ok and r.payload["removed"]["reservations"] == 1
    r = d.cleanup("buffer", "src-job", "operator")
    assert r.ok and r.payload["removed"]["buffers"] == 1
    assert d.transfer_status(p["transfer_id"]).payload["status"]["state"] == "canceled"
    assert d.cleanup("session", sid, "operator").ok
    assert not d.cleanup("session", sid, "operator").ok
    kinds = [c["target_kind"] for c in d.describe().payload["cleanup_events"]]
    assert kinds[-3:] == ["reservation", "buffer", "session"]


# ---- profiles ---------------------------------------------------------------------------------------

def test_profile_validation():
    d = daemon()
    bad = profile()
    bad["direct_h2d_bw_gbps"] = 0.0
    r = d.put_profile(0, [1, 2, 3], bad)
    assert not r.ok and "direct_h2d_bw_gbps" in r.error
    assert d.put_profile(0, [1], profile(1)).ok
    got = d.get_profile(0, [1]).payload["profile"]
    assert got["relay_gpus"] == [1] or tuple(got["relay_gpus"]) == (1,)
    assert got["profile"]["relays"][0]["relay_device"] == 1


def test_audit_records_have_the_full_field_set():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    assert d.authorize_worker_transfer(_auth_request(p, sid)).ok
    rec = d.describe().payload["audit_records"][-1]
    for k in ("audit_id", "event_type", "transfer_id", "lease_id", "session_id", "job_id", "relay_gpu",
              "direction", "state", "reason"):
        assert k in rec, k


def test_history_is_bounded_and_recent_receipts_stay_available():
    from pcie_pool_b200.daemon import IntentExecutor
    from pcie_pool_b200.mock import MockDataPlane, MockWorld

    world = MockWorld(gpu_count=4)
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_inflight_chunks_per_relay=4096,
                       topology_provider=StaticTopologyProvider(gpu_count=4), executor=IntentExecutor(
                           MockDataPlane(world)), history_limit=5, audit_limit=8)
    d.put_profile(0, [1, 2, 3], world.profile(0))
    c = InProcessDaemonClient(d)
    sid = d.register_session(0, [1, 2, 3], max_inflight_chunks=4096).payload["session"]["session_id"]
    assert d.register_job("job", session_id=sid).ok
    import numpy as np

    src, dst = np.zeros(4 * MiB, np.uint8), world.alloc(0, 4 * MiB)
    assert d.register_buffer("src-job", "job", "cpu_pinned", 4 * MiB, address=src.ctypes.data, pinned=True).ok
    assert d.register_buffer("dst-job", "job", "gpu", 4 * MiB, device_index=0, address=dst.ctypes.data).ok
    from pcie_pool_b200 import TurboBusClient

    client = TurboBusClient(daemon=c)
    for i in range(20):
        it = TransferIntent(f"h{i}", "job", sid, "src-job", "dst-job", "h2d", 4 * MiB,
                            ({"src_offset": 0, "dst_offset": 0, "bytes": 4 * MiB},), metadata={"chunk_bytes": MiB})
        assert client.transfer(it, timeout_seconds=30).state.value == "complete"
    desc = d.describe().payload
    assert len(desc["transfer_queue"]) <= 6 and len(desc["transfer_statuses"]) <= 6
    assert len(desc["audit_records"]) <= 16, "audit records are trimmed as transfers finish"
    assert d.wait_transfer_receipt("h19").ok and not d.wait_transfer_receipt("h0").ok


def test_receipts_carry_queue_execution_and_lease_wait_times():
    from pcie_pool_b200.daemon.server import transfer_timing

    clock = Clock()
    d = daemon(clock)
    sid = setup_job(d)
    r = d.submit_transfer_intent(_intent(sid, "t1"))
    assert r.ok
    tid = r.payload["transfer_id"]
    clock.t += 0.25
    d.executor_started(tid)
    clock.t += 0.5
    d.executor_finished(tid, ok_=True, bytes_completed=32 * MiB)
    t = d.wait_transfer_receipt("t1").payload["receipt"]["metadata"]["timing"]
    assert (t["queue_ms"], t["execution_ms"], t["total_ms"], t["lease_wait_ms"]) == (250.0, 500.0, 750.0, 0.0)
    parked = transfer_timing({"queued_at": 1.0, "delayed_at": 1.0, "admitted_at": 1.2, "started_at": 1.3}, 1.5)
    assert parked["lease_wait_ms"] == 200.0 and parked["total_ms"] == 500.0
