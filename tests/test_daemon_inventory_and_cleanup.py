"""The daemon's inventory, relay eligibility, profile cache, request
dispatch and cleanup paths, one rule per test: duplicate relays, closing and
cleaning sessions and jobs (direct transfers included), peer ownership of
sessions, intents and leases, the injected inventory and topology
invalidation, relay discovery across jobs, plans that keep only relays with
an enabled fabric path or fall back to direct, the profile cache's
round trip / invalidation / ageing, wire requests that are malformed (and
leave the state as it was), status mismatches and what they release, and
expiry before data movement.  Behaviours follow the remaining cases of
integration/test_daemon_state.py of the reference with independent
fixtures."""

from __future__ import annotations

import json
from dataclasses import replace

import pytest
from test_daemon_state import MiB, Clock, daemon, peer, plan, profile, setup_job

from pcie_pool_b200.daemon import TurboBusDaemon
from pcie_pool_b200.schema import (DaemonRequest, PeerIdentity, RequestType, TransferIntent,
                                   WorkerTransferAuthorizationRequest)
from pcie_pool_b200.topology import StaticTopologyProvider, TopologyProvider, synthetic_inventory


def state(d: TurboBusDaemon, key: str):
    return d.describe().payload[key]


def status(d: TurboBusDaemon, tid: str) -> str:
    return d.transfer_status(tid).payload["status"]["state"]


def worker_auth(p: dict, sid: str, job: str = "job", k: int = 0) -> WorkerTransferAuthorizationRequest:
    tok = p["lease_tokens"][k]
    return WorkerTransferAuthorizationRequest(transfer_id=p["transfer_id"], lease_id=tok["lease_id"],
                                              token=tok["token"], session_id=sid, job_id=job,
                                              src_buffer_id=f"src-{job}", dst_buffer_id=f"dst-{job}",
                                              direction="h2d", relay_gpu=tok["relay_gpu"])


def with_links(enabled: dict[int, bool]) -> StaticTopologyProvider:
    """A 4-GPU fixture inventory whose relay->GPU0 links are enabled as given."""
    inv = synthetic_inventory(4, source=StaticTopologyProvider.FIXTURE_SOURCE)
    links = tuple(replace(l, enabled=enabled.get(l.dst_device_id if l.src_device_id == 0 else l.src_device_id,
                                                 True)) if 0 in (l.src_device_id, l.dst_device_id) else l
                  for l in inv.fabric_links)
    return StaticTopologyProvider(replace(inv, fabric_links=links))


def relays_in(p: dict) -> list[int]:
    return sorted(a["path"]["relay_device"] for a in p["plan"]["assignments"] if a["path"]["kind"] == "relay")


# ---- sessions, jobs and cleanup ----------------------------------------------------------------------

def test_register_session_normalises_duplicate_relays():
    d = daemon()
    s = d.register_session(0, [3, 1, 3, 1], max_inflight_chunks=8).payload["session"]
    assert tuple(s["relay_gpus"]) == (1, 3)


def test_close_session_removes_its_jobs_buffers_and_cancels_planned_work():
    d = daemon(sessions_per_relay=1)
    sid = setup_job(d)
    p = plan(d, sid).payload
    r = d.close_session(sid)
    assert r.ok and r.payload["removed"] == {"jobs": 1, "buffers": 2, "sessions": 1, "reservations": 3,
                                             "staging_records": 0, "transfers": 1}
    assert status(d, p["transfer_id"]) == "canceled"
    assert state(d, "jobs") == {} and state(d, "buffers") == {} and state(d, "reservations") == {}
    assert d.register_session(0, [1, 2, 3]).ok, "the relays' one session slot is free again"
    assert not d.close_session(sid).ok


def test_cleanup_of_a_session_reports_what_it_removed():
    d = daemon()
    sid = setup_job(d)
    plan(d, sid)
    r = d.cleanup("session", sid, "operator")
    assert r.ok and r.payload["removed"]["jobs"] == 1 and r.payload["removed"]["buffers"] == 2
    assert r.payload["removed"]["transfers"] == 1
    assert not d.cleanup("session", sid, "operator").ok
    assert d.cleanup("session", sid, "operator", force=True).ok


def test_cleanup_of_a_job_cancels_its_direct_transfer_without_a_reservation():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid, mode="direct").payload
    assert p["lease_tokens"] == [] and relays_in(p) == []
    r = d.cleanup("job", "job", "job ended")
    assert r.ok and r.payload["removed"]["transfers"] == 1 and r.payload["removed"]["reservations"] == 0
    assert status(d, p["transfer_id"]) == "canceled"


# ---- peers ------------------------------------------------------------------------------------------

def test_a_job_cannot_join_a_session_that_another_peer_owns():
    d = daemon()
    alice, bob = peer("alice", 1), peer("bob", 2)
    sid = d.register_session(0, [1], peer_identity=alice).payload["session"]["session_id"]
    r = d.register_job("j-bob", session_id=sid, peer_identity=bob)
    assert not r.ok and "session" in r.error
    assert d.register_job("j-alice", session_id=sid, peer_identity=alice).ok


def test_an_unauthenticated_peer_leaves_ownership_to_the_request():
    d = daemon()
    anon = PeerIdentity(authenticated=False, source="unsupported")
    sid = setup_job(d, who=anon)
    assert state(d, "jobs")["job"]["job_id"] == "job"
    assert plan(d, sid).ok, "requests without an authenticated peer name their owner explicitly"


def test_a_peer_cannot_use_another_jobs_buffers_in_intents_or_leases():
    d = daemon(sessions_per_relay=2)
    alice, bob = peer("alice", 1), peer("bob", 2)
    sa = setup_job(d, "a", who=alice)
    setup_job(d, "b", who=bob)
    intent = TransferIntent("i-steal", "b", sa, "src-a", "dst-a", "h2d", 64 * MiB,
                            ({"src_offset": 0, "dst_offset": 0, "bytes": 64 * MiB},))
    r = d.submit_transfer_intent(intent, peer_identity=bob)
    assert not r.ok and ("owner" in r.error or "peer" in r.error)
    p = plan(d, sa, "a", peer_identity=alice).payload
    tok = p["lease_tokens"][0]
    v = d.validate_lease(tok["lease_id"], tok["token"], session_id=sa, job_id="a", peer_identity=bob)
    assert not v.ok and "peer" in v.error
    assert d.validate_lease(tok["lease_id"], tok["token"], session_id=sa, job_id="a", peer_identity=alice).ok


def test_plan_infers_the_job_from_the_buffers_owner():
    d = daemon()
    sid = setup_job(d)
    r = d.plan_transfer(sid, 64 * MiB, 16 * MiB, buffer_ids=["src-job", "dst-job"])
    assert r.ok, r.error
    assert r.payload["transfer_status"]["job_id"] == "job"


# ---- inventory and topology -------------------------------------------------------------------------

def test_the_injected_inventory_is_what_the_daemon_reports():
    prov = StaticTopologyProvider(gpu_count=4)
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], topology_provider=prov)
    inv = d.get_inventory().payload
    assert len(inv["inventory"]["gpus"]) == 4 and inv["inventory"]["source"] == "test_fixture_static"
    assert inv["topology_snapshot"]["snapshot_id"] == prov.snapshot().topology_snapshot_id()
    assert not TurboBusDaemon(relay_gpus=[1]).get_inventory().ok, "no provider, no inventory"


def test_invalidate_topology_refreshes_or_reports_an_unsupported_provider():
    prov = StaticTopologyProvider(gpu_count=4)
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], topology_provider=prov)
    r = d.invalidate_topology()
    assert r.ok and prov.invalidations == 1 and r.payload["inventory_source"] == "test_fixture_static"
    assert r.payload["topology_snapshot_id"] == prov.snapshot().topology_snapshot_id()

    class Frozen(TopologyProvider):
        def snapshot(self):
            return prov.snapshot()

    r = TurboBusDaemon(relay_gpus=[1], topology_provider=Frozen()).invalidate_topology()
    assert not r.ok and "does not support invalidation" in r.error


def test_relay_discovery_reports_sessions_and_leases_across_jobs():
    d = daemon(sessions_per_relay=2)
    sa, sb = setup_job(d, "a"), setup_job(d, "b")
    pa = plan(d, sa, "a").payload
    pb = plan(d, sb, "b").payload
    # job a's active relay paths keep job b's plan off those links
    assert relays_in(pa) == [1, 2, 3] and relays_in(pb) == []
    disc = d.discover_relays(0).payload["relay_discovery"]
    assert disc["summary"]["relay_count"] == 3 and disc["summary"]["eligible_relay_count"] == 3
    assert disc["summary"]["active_session_count"] == 6 and disc["summary"]["active_lease_count"] == 3
    r1 = next(r for r in disc["relays"] if r["relay_gpu"] == 1)
    assert sorted(j for s in r1["sessions"] for j in s["job_ids"]) == ["a", "b"]
    assert len(r1["reservations"]) == 1 and r1["eligibility"]["eligible"] is True
    assert r1["leases"][0]["job_id"] == "a"
    assert d.discover_relays().payload["relay_discovery"]["relays"][0]["eligibility"]["eligible"] is None


def test_plans_use_only_relays_with_an_enabled_fabric_link():
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_sessions_per_relay=4, max_inflight_chunks_per_relay=4096,
                       topology_provider=with_links({3: False}), clock=Clock())
    d.put_profile(0, [1, 2, 3], profile())
    sid = setup_job(d)
    p = plan(d, sid).payload
    assert sorted(set(relays_in(p))) == [1, 2]
    filtered = p["planning"]["relay_eligibility"]["filtered_relays"]
    assert filtered == [{"relay_gpu": 3, "reason": "missing enabled fabric link"}]
    assert sorted(t["relay_gpu"] for t in p["lease_tokens"]) == [1, 2]


def test_plans_fall_back_to_direct_without_any_enabled_fabric_path():
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_sessions_per_relay=4, max_inflight_chunks_per_relay=4096,
                       topology_provider=with_links({1: False, 2: False, 3: False}), clock=Clock())
    d.put_profile(0, [1, 2, 3], profile())
    sid = setup_job(d)
    rec = d.discover_relays(0, [1]).payload["relay_discovery"]["relays"][0]
    assert rec["eligibility"] == {"target_gpu": 0, "eligible": False, "reason": "missing enabled fabric link"}
    caps = rec["inventory"]["path_capabilities"]
    assert caps["has_pcie_path"] and caps["enabled_fabric_link_count"] == 0
    p = plan(d, sid).payload
    assert relays_in(p) == [] and p["lease_tokens"] == [] and p["reservations"] == []
    assert (p["stats"]["resolved_mode"], p["stats"]["relay_bytes"]) == ("direct", 0)
    assert p["admission"]["reason"] == "direct_or_fallback_plan"


def test_plans_fall_back_to_direct_when_relay_quota_is_taken():
    d = daemon(sessions_per_relay=2, inflight=4)
    sid = setup_job(d, inflight=64)
    other = d.register_session(0, [1, 2, 3], max_inflight_chunks=64).payload["session"]["session_id"]
    for g in (1, 2, 3):
        assert d.reserve_transfer(other, g, 4).ok
    p = plan(d, sid).payload
    assert relays_in(p) == [] and "relay" in p["decision"]["fallback_reason"]
    for g in (1, 2, 3):
        d.release_transfer(next(rid for rid, r in state(d, "reservations").items() if r["relay_gpu"] == g))
    assert relays_in(plan(d, sid).payload) == [1, 2, 3], "released quota is usable again"


# ---- profile cache ----------------------------------------------------------------------------------

def test_profile_cache_round_trip_invalidation_and_ageing():
    clock = Clock()
    d = TurboBusDaemon(relay_gpus=[1, 2], topology_provider=StaticTopologyProvider(gpu_count=3), clock=clock,
                       profile_max_age_seconds=60.0)
    assert d.get_profile(0, [1, 2]).payload["profile"] is None
    put = d.put_profile(0, [2, 1, 2], profile(2), profile_bytes=64 * MiB)
    assert put.ok and list(put.payload["profile"]["relay_gpus"]) == [1, 2]
    got = d.get_profile(0, [1, 2]).payload["profile"]
    assert got["profile_bytes"] == 64 * MiB and got["updated_at"] == clock.t
    assert got["profile"]["relays"][1]["relay_device"] == 2
    assert d.invalidate_profile(0, [1, 2]).payload["removed"] is True
    assert d.invalidate_profile(0, [1, 2]).payload["removed"] is False
    d.put_profile(0, [1, 2], profile(2))
    clock.t += 61.0
    assert d.get_profile(0, [1, 2]).payload["profile"] is None, "entries older than the max age are purged"
    assert "profile_cache" in d.describe().payload and d.describe().payload["profile_cache"] == {}


def test_profile_requests_over_the_wire(tmp_path):
    d = daemon()
    put = d.handle_request(DaemonRequest(RequestType.PUT_PROFILE, payload={
        "target_gpu": 0, "relay_gpus": [1], "profile": profile(1), "profile_bytes": 8 * MiB}))
    assert put.ok
    got = d.handle_request(DaemonRequest(RequestType.GET_PROFILE, payload={"target_gpu": 0, "relay_gpus": [1]}))
    assert got.payload["profile"]["profile_bytes"] == 8 * MiB
    bad = d.handle_request(DaemonRequest(RequestType.PUT_PROFILE, payload={
        "target_gpu": 0, "relay_gpus": [1], "profile": {**profile(1), "direct_h2d_bw_gbps": -1}}))
    assert not bad.ok
    gone = d.handle_request(DaemonRequest(RequestType.INVALIDATE_PROFILE, payload={"target_gpu": 0,
                                                                                   "relay_gpus": [1]}))
    assert gone.payload["removed"] is True


# ---- malformed requests -----------------------------------------------------------------------------

def test_requests_missing_required_fields_are_rejected():
    d = daemon()
    for t, payload in ((RequestType.REGISTER_JOB, {}), (RequestType.REGISTER_BUFFER, {"job_id": "j"}),
                       (RequestType.REGISTER_SESSION, {"relay_gpus": [1]}), (RequestType.CLEANUP, {"reason": "x"}),
                       (RequestType.TRANSFER_STATUS, {}), (RequestType.VALIDATE_LEASE, {"lease_id": "l"})):
        r = d.handle_request(DaemonRequest(t, payload=payload))
        assert not r.ok and r.error.startswith("invalid request"), (t, r)
    for t in (RequestType.PLAN_TRANSFER, RequestType.CLOSE_SESSION, RequestType.RESERVE_TRANSFER):
        assert "session_id is required" in d.handle_request(DaemonRequest(t, payload={"relay_gpu": 1})).error
    assert "intent is required" in d.handle_request(DaemonRequest(RequestType.SUBMIT_TRANSFER_INTENT)).error


def test_malformed_wire_messages_leave_the_state_untouched():
    d = daemon()
    sid = setup_job(d)
    plan(d, sid)
    keys = ("sessions", "jobs", "buffers", "reservations", "transfer_statuses")
    before = json.dumps({k: state(d, k) for k in keys}, sort_keys=True, default=str)
    for msg in (b"\xff\xfe", "not json", "[1, 2]", '{"payload": {}}', '{"request_type": "NOPE"}',
                '{"request_type": "REGISTER_JOB", "payload": []}',
                '{"request_type": "REGISTER_BUFFER", "payload": {"buffer_id": "x", "job_id": "nobody"}}',
                '{"request_type": "CLEANUP", "payload": {"target_kind": "planet", "target_id": "x"}}',
                json.dumps({"request_type": "RESERVE_TRANSFER", "session_id": sid,
                            "payload": {"relay_gpu": 1, "chunks": -2}})):
        r = d.handle_wire_message(msg)
        assert not r.ok, msg
    after = json.dumps({k: state(d, k) for k in keys}, sort_keys=True, default=str)
    assert after == before


# ---- statuses, releases and expiry ------------------------------------------------------------------

def test_a_completion_that_does_not_account_for_every_byte_fails_and_releases():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    r = d.transfer_status(p["transfer_id"], "complete", bytes_completed=64 * MiB - 1)
    assert status(d, p["transfer_id"]) == "failed"
    assert not r.ok or r.payload["status"]["state"] == "failed"
    assert state(d, "reservations") == {}
    assert not d.transfer_status(p["transfer_id"], "complete", bytes_completed=64 * MiB).ok, "failed is final"


def test_releasing_after_a_failure_does_not_rewrite_it():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    assert d.transfer_status(p["transfer_id"], "failed", error="lane 2 lost").ok
    for tok in p["lease_tokens"]:
        d.release_transfer(tok["lease_id"])
    st = d.transfer_status(p["transfer_id"]).payload["status"]
    assert st["state"] == "failed" and st["error"] == "lane 2 lost"


def test_a_worker_failure_releases_reservations_and_staging_records():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    a = d.authorize_worker_transfer(worker_auth(p, sid))
    assert a.ok, a.error
    assert state(d, "staging_records"), "authorization records the worker's staging"
    assert d.transfer_status(p["transfer_id"], "failed", error="worker lost its device").ok
    assert state(d, "reservations") == {} and state(d, "staging_records") == {}


def test_reaping_a_stale_session_releases_staging_and_owner_state():
    clock = Clock()
    d = daemon(clock=clock, session_timeout_seconds=30.0)
    alice = peer("alice")
    sid = setup_job(d, who=alice)
    p = plan(d, sid, peer_identity=alice).payload
    assert d.authorize_worker_transfer(worker_auth(p, sid), peer_identity=alice).ok
    clock.t += 31.0
    d.reap_stale_sessions()
    for k in ("sessions", "jobs", "buffers", "reservations", "staging_records", "job_peer_identities",
              "session_peer_identities"):
        assert not state(d, k), k
    assert status(d, p["transfer_id"]) in ("canceled", "failed")


def test_an_expired_plan_is_refused_before_any_data_moves():
    clock = Clock()
    d = daemon(clock=clock)
    sid = setup_job(d)
    p = plan(d, sid).payload
    clock.t = p["plan_expires_at"] + 1.0
    r = d.authorize_worker_transfer(worker_auth(p, sid))
    assert not r.ok and "expired" in r.error
    assert state(d, "staging_records") == {}


def test_a_rescheduled_plan_makes_the_old_ticket_stale_for_the_worker():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid).payload
    new = d.reschedule_transfer(p["transfer_id"]).payload
    assert new["plan_generation"] == p["plan_generation"] + 1
    r = d.authorize_worker_transfer(worker_auth(p, sid))
    assert not r.ok
    fresh = d.authorize_worker_transfer(worker_auth(new, sid))
    assert fresh.ok and fresh.payload["plan_generation"] == new["plan_generation"]
    assert len(fresh.payload["relay_gpus"]) == 3 and len(fresh.payload["lease_ids"]) == 3


@pytest.mark.parametrize("hint", ["relay_gpus", "relay_gpu", "paths", "Route", "target_gpu", "mode"])
def test_intents_cannot_carry_physical_path_hints(hint):
    with pytest.raises(ValueError):
        TransferIntent("i", "job", "s", "a", "b", "h2d", 16, ({"src_offset": 0, "dst_offset": 0, "bytes": 16},),
                       policy_hints={hint: [1]})


# ---- scheduler decisions seen through the daemon ----------------------------------------------------

def test_without_a_profile_the_plan_falls_back_to_direct():
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_inflight_chunks_per_relay=4096,
                       topology_provider=StaticTopologyProvider(gpu_count=4), clock=Clock())
    sid = setup_job(d)
    p = plan(d, sid).payload
    assert relays_in(p) == [] and p["stats"]["resolved_mode"] == "direct"
    assert "profile" in p["decision"]["fallback_reason"]


@pytest.mark.parametrize("kw,msg", [({"total": -1}, "total_bytes"), ({"chunk": 0}, "chunk_bytes"),
                                    ({"direction": "sideways"}, "direction"), ({"mode": "teleport"}, "mode"),
                                    ({"mode": "AUTO"}, None), ({"mode": "relay"}, None)])
def test_plan_request_values_are_checked(kw, msg):
    d = daemon()
    sid = setup_job(d)
    r = plan(d, sid, **kw)
    if msg is None:
        assert r.ok, r.error
    else:
        assert not r.ok and msg in r.error
    assert state(d, "reservations") == {} or r.ok


def test_the_workload_kind_reaches_the_decision_and_its_leases():
    d = daemon()
    sid = setup_job(d)
    p = plan(d, sid, workload_kind="kv_cache").payload
    leases = p["decision"]["metadata"]["leases"]
    assert len(leases) == 3 and {l["job_id"] for l in leases} == {"job"}
    assert p["transfer_status"]["job_id"] == "job"
    (rec,) = state(d, "transfer_queue")
    assert rec["workload_kind"] == "kv_cache" and rec["transfer_id"] == p["transfer_id"]


# ---- checkpoint / resume of the profile cache ---------------------------------------------------------

def test_a_restarted_daemon_resumes_from_its_profile_store(tmp_path):
    store = tmp_path / "profiles.json"

    def start(clock):
        return TurboBusDaemon(relay_gpus=[1, 2, 3], topology_provider=StaticTopologyProvider(gpu_count=4),
                              clock=clock, profile_store_path=str(store), profile_max_age_seconds=600.0)

    clock = Clock(1000.0)
    first = start(clock)
    assert first.put_profile(0, [1, 2, 3], profile(), profile_bytes=64 * MiB).ok
    assert first.put_profile(1, [2], {**profile(1), "target_device": 1,
                                      "relays": [{**profile(1)["relays"][0], "relay_device": 2,
                                                  "target_device": 1}]}).ok
    assert json.loads(store.read_text())["profiles"], "the cache is written through on every update"
    again = start(clock)
    got = again.get_profile(0, [3, 2, 1]).payload["profile"]
    assert got["profile_bytes"] == 64 * MiB and got["updated_at"] == 1000.0
    assert again.get_profile(1, [2]).payload["profile"]["profile"]["relays"][0]["relay_device"] == 2
    sid = setup_job(again)
    assert relays_in(plan(again, sid).payload) == [1, 2, 3], "plans use the resumed profile without re-profiling"
    assert again.invalidate_profile(1, [2]).payload["removed"]
    assert start(clock).get_profile(1, [2]).payload["profile"] is None, "invalidation is persisted too"
    clock.t += 601.0
    assert start(clock).get_profile(0, [1, 2, 3]).payload["profile"] is None, "stale entries are not resumed"
    store.write_text("{not json")
    assert start(clock).get_profile(0, [1, 2, 3]).ok, "a damaged store starts an empty cache"
