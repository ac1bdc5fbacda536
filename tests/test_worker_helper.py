"""Worker helper, stage by stage: parsing the daemon's authorization payload
into a ticketed request (and every way a payload can disagree with itself),
plan checks that must fail before a staging slot is taken, the status
reporter's mapping, the cleanup coordinator over one and several leases,
binding order of the client's buffers around the executor, the payload
parser, the request/response codec and the message endpoint.  The daemon is
real (in-process) where a valid ticket is needed; reporters and cleanups run
against recording fakes.  Behaviours follow integration/test_worker_helper.py
of the reference with independent fixtures."""

from __future__ import annotations

import copy
import json
from dataclasses import asdict, replace

import pytest
from test_worker_lifecycle import MiB, N, Rig

from pcie_pool_b200.daemon import InProcessDaemonClient
from pcie_pool_b200.planner_types import assignment_chunks
from pcie_pool_b200.schema import BufferRegistration, DaemonResponse, WorkerTransferAuthorizationRequest
from pcie_pool_b200.transfer import TransferRequest
from pcie_pool_b200.worker import (WorkerDataPlaneResourceBinder, WorkerServiceEndpoint,
                                   WorkerServiceRequestEnvelope, WorkerServiceResponseEnvelope, WorkerStagingPool,
                                   WorkerTransferClient, WorkerTransferService)
from pcie_pool_b200.worker.codec import (WorkerMessageCodecError, decode_worker_request_envelope,
                                         decode_worker_response_envelope, encode_worker_request_envelope,
                                         encode_worker_response_envelope, handle_worker_service_message)
from pcie_pool_b200.worker.cuda_executor import CudaWorkerExecutor
from pcie_pool_b200.worker.helper import (WorkerAuthorizationError, WorkerCleanupError, WorkerStatusReportError,
                                          WorkerTransferAuthorizer, WorkerTransferCleanupCoordinator,
                                          WorkerTransferRequest, WorkerTransferResult, WorkerTransferState,
                                          WorkerTransferStatusReporter, parse_worker_authorization_request_payload)


@pytest.fixture
def rig():
    r = Rig()
    yield r
    r.close()


def authorized(rig, **over):
    """A live authorization request and the daemon's (deep-copied) answer."""
    req, plan = rig.authorization(**over)
    resp = InProcessDaemonClient(rig.daemon).authorize_worker_transfer(req)
    assert resp.ok, resp.error
    return req, plan, copy.deepcopy(dict(resp.payload))


def relay_chunks(plan, relay=None):
    """(src, dst, bytes) of the plan's relay chunks, optionally of one relay."""
    return [triple(c) for a in plan["assignments"] if a["path"]["kind"] == "relay"
            and (relay is None or a["path"]["relay_device"] == relay) for c in assignment_chunks(a)]


def triple(c):
    return (c["src_offset"], c["dst_offset"], c["bytes"])


def edit_plans(payload, fn):
    """Apply ``fn`` to the ticket's plan and the decision's (they must agree)."""
    for key in ("ticket", "decision"):
        if payload.get(key) is not None:
            fn(payload[key]["plan"])
    return payload


class CountingPool(WorkerStagingPool):
    def __init__(self):
        super().__init__()
        self.allocations = 0

    def allocate(self, request):
        self.allocations += 1
        return super().allocate(request)


class Canned:
    """Daemon client whose worker authorization answers with a fixed payload;
    everything else goes to the real daemon."""

    def __init__(self, inner, payload):
        self.inner, self.payload = inner, payload

    def authorize_worker_transfer(self, request, *a, **kw):
        return DaemonResponse(ok=True, payload=self.payload)

    def __getattr__(self, name):
        return getattr(self.inner, name)


class Recorder:
    """Daemon client fake that records status reports, cleanups and releases;
    ``fail`` maps a method name (or ``"cleanup:<target_id>"``) to an error."""

    def __init__(self, fail=None):
        self.calls, self.fail = [], dict(fail or {})

    def _answer(self, key, payload):
        err = self.fail.get(key) or self.fail.get(key.split(":")[0])
        return DaemonResponse(ok=False, error=err) if err else DaemonResponse(ok=True, payload=payload)

    def transfer_status(self, transfer_id, state=None, bytes_completed=None, error=None):
        self.calls.append(("status", transfer_id, state, bytes_completed, error))
        return self._answer("transfer_status", {"status": {"state": state}})

    def cleanup(self, target_kind, target_id, reason, force):
        self.calls.append(("cleanup", target_kind, target_id, reason, force))
        return self._answer(f"cleanup:{target_id}", {"reservation_id": target_id})

    def release_transfer(self, lease_id):
        self.calls.append(("release", lease_id))
        return self._answer(f"release_transfer:{lease_id}", {"reservation_id": lease_id})


# ---- parsing the daemon's answer into a ticketed request --------------------------------------------

def test_request_needs_the_daemon_ticket(rig):
    _, _, payload = authorized(rig)
    with pytest.raises(ValueError, match="execution ticket"):
        WorkerTransferRequest.from_authorization_payload({k: v for k, v in payload.items() if k != "ticket"})
    with pytest.raises(ValueError, match="mapping"):
        WorkerTransferRequest.from_authorization_payload(["ticket"])
    with pytest.raises(ValueError, match="ExecutionTicket"):
        WorkerTransferRequest.from_authorization(object())


def test_request_parses_a_multi_relay_ticket(rig):
    _, plan, payload = authorized(rig)
    wr = WorkerTransferRequest.from_authorization_payload(payload)
    planned = tuple(sorted({a["path"]["relay_device"] for a in plan["plan"]["assignments"]
                            if a["path"]["kind"] == "relay"}))
    assert len(planned) > 1 and wr.relay_gpus == planned
    assert wr.lease_ids == tuple(payload["lease_ids"]) and wr.transfer_id == plan["transfer_id"]
    dp = wr.data_plane
    assert [triple(c) for c in dp.ranges] == relay_chunks(plan["plan"])
    by_gpu = dp.metadata["relay_ranges_by_gpu"]
    assert {int(k) for k in by_gpu} == set(planned)
    for r in planned:
        assert [triple(c) for c in by_gpu[str(r)]] == relay_chunks(plan["plan"], r)
    assert (dp.src_handle.buffer_id, dp.dst_handle.buffer_id, dp.direction) == ("host", "dev", "h2d")


def test_explicit_ticket_payload_defaults_to_every_planned_relay_and_lease(rig):
    _, plan, payload = authorized(rig)
    bare = {k: payload[k] for k in ("ticket", "src_buffer", "dst_buffer")}
    wr = WorkerTransferRequest.from_execution_ticket_payload(bare)
    assert wr.lease_ids == tuple(payload["ticket"]["lease_ids"])
    assert wr.relay_gpus == tuple(sorted(wr.relay_gpus)) and len(wr.relay_gpus) == len(wr.lease_ids)
    assert wr.transfer_id == payload["ticket"]["metadata"]["transfer_id"] == plan["transfer_id"]


def test_one_relay_of_the_ticket_narrows_the_ranges(rig):
    _, plan, payload = authorized(rig)
    payload.update(relay_gpus=None, relay_gpu=2, lease_ids=None)
    wr = WorkerTransferRequest.from_execution_ticket_payload(payload)
    assert wr.relay_gpus == (2,) and [triple(c) for c in wr.data_plane.ranges] == relay_chunks(plan["plan"], 2)
    payload.update(relay_gpus=(1, 3), relay_gpu=2)
    with pytest.raises(ValueError, match="relay_gpus"):
        WorkerTransferRequest.from_execution_ticket_payload(payload)
    payload.update(relay_gpus=None, relay_gpu=0)
    with pytest.raises(ValueError, match="daemon plan"):
        WorkerTransferRequest.from_execution_ticket_payload(payload)


@pytest.mark.parametrize("mutate,msg", [
    (lambda p: p["decision"].update(intent_id="someone-else"), "intent_id differs from the scheduling decision"),
    (lambda p: p["decision"].update(session_id="other-session"), "session_id differs"),
    (lambda p: p["decision"]["plan"].update(total_bytes=1), "plan differs from the scheduling decision"),
    (lambda p: p["src_buffer"].update(buffer_id="other"), "source buffer differs"),
    (lambda p: p["dst_buffer"].update(buffer_id="other"), "destination buffer differs"),
    (lambda p: p["ticket"]["metadata"].update(issuer="not-the-daemon"), "issued by"),
    (lambda p: p.update(plan_generation=p["plan_generation"] + 1), "stale"),
    (lambda p: p["ticket"]["metadata"].pop("plan_generation"), "no plan_generation"),
    (lambda p: p["ticket"]["metadata"].update(plan_generation=0), "positive"),
    (lambda p: p["ticket"]["metadata"].update(transfer_id=" "), "transfer_id"),
    (lambda p: p.update(lease_id="not-a-lease"), "not one of the requested lease_ids"),
    (lambda p: p.update(lease_ids=()), "lease_ids is empty"),
], ids=["decision-intent", "decision-session", "decision-plan", "src-buffer", "dst-buffer", "issuer",
        "stale-generation", "no-generation", "zero-generation", "no-transfer-id", "foreign-lease", "no-leases"])
def test_ticket_payload_rejections(rig, mutate, msg):
    _, _, payload = authorized(rig)
    mutate(payload)
    with pytest.raises(ValueError, match=msg):
        WorkerTransferRequest.from_authorization_payload(payload)


def test_data_plane_must_match_the_authority_and_handles(rig):
    _, _, payload = authorized(rig)
    wr = WorkerTransferRequest.from_authorization_payload(payload)
    a = wr.authorization
    with pytest.raises(ValueError, match="data-plane request's lease_id disagrees"):
        WorkerTransferRequest(authorization=replace(a, lease_id=wr.lease_ids[1]), ticket=wr.ticket,
                              data_plane=wr.data_plane)
    other = BufferRegistration(**{**asdict(a.src_buffer), "buffer_id": "elsewhere"})
    with pytest.raises(ValueError, match="data-plane request's src handle disagrees"):
        WorkerTransferRequest(authorization=replace(a, src_buffer=other), ticket=wr.ticket, data_plane=wr.data_plane)
    with pytest.raises(ValueError, match="data-plane request's ranges"):
        WorkerTransferRequest(authorization=replace(a, ranges=a.ranges[:1]), ticket=wr.ticket,
                              data_plane=wr.data_plane)
    # without an explicit data plane the authorization's own is built, and the ticket must still agree
    with pytest.raises(ValueError, match="ticket's relay ranges disagree"):
        WorkerTransferRequest(authorization=replace(a, ranges=a.ranges[:1]), ticket=wr.ticket)


# ---- plan checks before any staging slot is taken --------------------------------------------------

def _first_relay_path(plan):
    return next(a for a in plan["assignments"] if a["path"]["kind"] == "relay")


def _move_first_chunk(plan, key, value):
    """Point the first relay chunk (or chunk run) somewhere else; daemon plans
    carry compact chunk runs [src, dst, bytes, chunk]."""
    a = _first_relay_path(plan)
    if a.get("chunk_runs"):
        a["chunk_runs"][0][0 if key == "src_offset" else 1] = value
    else:
        a["chunks"][0][key] = value


@pytest.mark.parametrize("edit,msg", [
    (lambda pl: pl.update(assignments=[]), "no relay lane"),
    (lambda pl: _move_first_chunk(pl, "dst_offset", N), "exceeds dst buffer size"),
    (lambda pl: _move_first_chunk(pl, "src_offset", N), "exceeds src buffer size"),
    (lambda pl: pl.update(total_bytes=pl["total_bytes"] + MiB), "total"),
    (lambda pl: [a["path"].update(target_device=3) for a in pl["assignments"]], "target"),
    (lambda pl: _first_relay_path(pl)["path"].update(enabled=False), "disabled"),
    (lambda pl: _first_relay_path(pl)["path"].update(direction="d2h"), "direction"),
    (lambda pl: _first_relay_path(pl)["path"].update(kind="nvme"), "daemon plan"),
], ids=["no-plan", "dst-out-of-bounds", "src-out-of-bounds", "total-mismatch", "target-mismatch", "disabled",
        "direction-mismatch", "unknown-path"])
def test_bad_daemon_plans_fail_before_staging(rig, edit, msg):
    req, _, payload = authorized(rig)
    edit_plans(payload, edit)
    pool = CountingPool()
    client = WorkerTransferClient(Canned(rig.dc, payload), executor=rig.client.executor, staging_pool=pool,
                                  resource_binder=rig.client.resource_binder)
    with pytest.raises(WorkerAuthorizationError, match=msg):
        client.submit(req)
    assert pool.allocations == 0


def test_handle_mismatch_fails_before_staging(rig):
    req, _, payload = authorized(rig)
    payload["dst_buffer"]["buffer_id"] = "not-the-ticket-buffer"
    pool = CountingPool()
    client = WorkerTransferClient(Canned(rig.dc, payload), executor=rig.client.executor, staging_pool=pool)
    with pytest.raises(WorkerAuthorizationError, match="destination buffer"):
        client.submit(req)
    lc = client.submit_report_cleanup_lifecycle(req)
    assert lc.final_state == "authorization_failed" and lc.staging_slot is None and pool.allocations == 0


def test_authorizer_builds_the_request_or_raises_the_daemon_denial(rig):
    req, plan, _ = authorized(rig)
    wr = WorkerTransferAuthorizer(rig.dc).authorize(req)
    assert wr.transfer_id == plan["transfer_id"] and wr.data_plane.plan == plan["plan"]
    with pytest.raises(WorkerAuthorizationError, match="invalid lease token"):
        WorkerTransferAuthorizer(rig.dc).authorize(replace(req, token="forged"))


def test_client_defaults_to_the_cuda_executor_and_binder():
    c = WorkerTransferClient(Recorder())
    assert isinstance(c.executor, CudaWorkerExecutor)
    assert isinstance(c.resource_binder, WorkerDataPlaneResourceBinder)
    assert isinstance(c.staging_pool, WorkerStagingPool)
    bare = WorkerTransferClient(Recorder(), executor=object())
    assert bare.resource_binder is None  # a caller's executor binds its own resources


def test_client_submit_runs_the_bound_executor_path(rig):
    req, plan, _ = authorized(rig)
    result = rig.client.submit(req)
    assert result.state is WorkerTransferState.COMPLETE
    assert result.bytes_completed == sum(c[2] for c in relay_chunks(plan["plan"]))
    assert result.metadata.get("executor") and len(rig.pool) == 0


# ---- results, status reports and cleanups ----------------------------------------------------------

def test_results_map_to_completion_reports():
    ok = WorkerTransferResult("t", WorkerTransferState.COMPLETE, bytes_completed=64, metadata={"x": 1})
    c = ok.data_plane_completion("lease-1")
    assert (c.state, c.bytes_completed, c.error, c.lease_id) == ("complete", 64, None, "lease-1")
    bad = WorkerTransferResult("t", "failed")
    c = bad.data_plane_completion("lease-1")
    assert c.state == "failed" and c.error == "worker transfer failed"
    with pytest.raises(ValueError):
        WorkerTransferResult("t", "complete", bytes_completed=-1)
    with pytest.raises(ValueError):
        WorkerTransferResult(" ", "complete")


def test_status_reporter_maps_states_and_raises_on_rejection():
    d = Recorder()
    rep = WorkerTransferStatusReporter(d)
    rep.report(WorkerTransferResult("t1", "complete", bytes_completed=8))
    rep.report(WorkerTransferResult("t2", "failed"))
    rep.report(WorkerTransferResult("t3", "failed", error="lane 2 timed out", bytes_completed=4))
    assert d.calls == [("status", "t1", "complete", 8, None), ("status", "t2", "failed", 0, "worker transfer failed"),
                       ("status", "t3", "failed", 4, "lane 2 timed out")]
    with pytest.raises(WorkerStatusReportError, match="terminal"):
        WorkerTransferStatusReporter(Recorder({"transfer_status": "transfer is terminal"})).report(
            WorkerTransferResult("t", "complete"))
    with pytest.raises(TypeError):
        rep.report({"state": "complete"})


def _single_and_multi(rig):
    _, _, payload = authorized(rig)
    multi = WorkerTransferRequest.from_authorization_payload(payload)
    lone = dict(payload, relay_gpus=None, relay_gpu=1, lease_ids=None)
    single = WorkerTransferRequest.from_execution_ticket_payload(lone)
    assert len(single.lease_ids) == 1 and len(multi.lease_ids) == 3
    return single, multi


def test_cleanup_after_authorization_failure_targets_the_lease_or_session():
    d = Recorder()
    cc = WorkerTransferCleanupCoordinator(d)
    auth = WorkerTransferAuthorizationRequest(transfer_id="t", lease_id="L", token="k", session_id="S", job_id="j",
                                              src_buffer_id="a", dst_buffer_id="b", direction="h2d")
    cc.cleanup_authorization_failure(auth)
    cc.cleanup_authorization_failure(auth, target_kind="session")
    assert d.calls == [("cleanup", "reservation", "L", "worker_authorization_failed", True),
                       ("cleanup", "session", "S", "worker_authorization_failed", True)]
    with pytest.raises(ValueError, match="reservation or session"):
        cc.cleanup_authorization_failure(auth, target_kind="job")


def test_cleanup_of_a_complete_transfer_releases_each_lease(rig):
    single, multi = _single_and_multi(rig)
    d = Recorder()
    cc = WorkerTransferCleanupCoordinator(d)
    done = WorkerTransferResult(single.transfer_id, "complete", bytes_completed=1)
    r = cc.cleanup_execution_failure(single, done)
    assert r.ok and d.calls == [("release", single.lease_ids[0])]
    d.calls.clear()
    r = cc.cleanup_execution_failure(multi, done)
    assert d.calls == [("release", lid) for lid in multi.lease_ids]
    assert r.payload["released_reservation_ids"] == multi.lease_ids and r.payload["cleanup_mode"] == "release"


def test_cleanup_of_a_failed_transfer_cleans_each_lease(rig):
    single, multi = _single_and_multi(rig)
    d = Recorder()
    cc = WorkerTransferCleanupCoordinator(d)
    failed = WorkerTransferResult(multi.transfer_id, "failed", error="x")
    cc.cleanup_execution_failure(single, failed)
    assert d.calls == [("cleanup", "reservation", single.lease_ids[0], "worker_failed", True)]
    d.calls.clear()
    r = cc.cleanup_execution_failure(multi, failed)
    assert [c[2] for c in d.calls] == list(multi.lease_ids) and r.payload["cleanup_mode"] == "cleanup"
    d.calls.clear()
    cc.cleanup_execution_failure(multi, failed, target_kind="session")
    assert d.calls == [("cleanup", "session", multi.authorization.session_id, "worker_failed", True)]


def test_cleanup_rejections_name_every_lease_that_failed(rig):
    single, multi = _single_and_multi(rig)
    bad = multi.lease_ids[1]
    d = Recorder({f"cleanup:{bad}": "unknown reservation"})
    with pytest.raises(WorkerCleanupError, match=f"{bad}: unknown reservation"):
        WorkerTransferCleanupCoordinator(d).cleanup_execution_failure(
            multi, WorkerTransferResult(multi.transfer_id, "failed"))
    assert len(d.calls) == 3  # the other leases were still cleaned
    with pytest.raises(WorkerCleanupError, match="release"):
        WorkerTransferCleanupCoordinator(Recorder({"release_transfer": "release refused"})).cleanup_execution_failure(
            multi, WorkerTransferResult(multi.transfer_id, "complete"))

    class NoRelease:
        def cleanup(self, **kw):
            return DaemonResponse(ok=True)

    with pytest.raises(WorkerCleanupError, match="cannot release"):
        WorkerTransferCleanupCoordinator(NoRelease()).cleanup_execution_failure(
            single, WorkerTransferResult(single.transfer_id, "complete"))


def test_lifecycle_record_serialises_to_json(rig):
    req, p, _ = authorized(rig)
    lc = rig.client.submit_report_cleanup_lifecycle(req)
    d = json.loads(json.dumps(lc.as_dict()))
    assert d["final_state"] == "complete" and d["cleanup_target"] == {"target_kind": "reservation",
                                                                     "target_id": lc.lease_id}
    assert d["status_update"]["state"] == "complete" and d["staging_release"]["state"] == "released"
    assert d["lease_ids"] == list(lc.lease_ids) and d["worker_request"]["ticket"]["ticket_id"]
    env = lc.completion_envelope().as_dict()
    assert env["staging_slot"]["slot_id"] == env["staging_release"]["slot_id"]
    assert env["daemon_status_response"]["ok"] and env["daemon_cleanup_response"]["ok"]


def test_status_failure_still_releases_staging_in_the_envelope(rig):
    req, p, _ = authorized(rig)
    rig.dc.fail["transfer_status"] = "status store offline"
    lc = rig.client.submit_report_cleanup_lifecycle(req)
    env = lc.completion_envelope().as_dict()
    assert lc.final_state == "status_failed" and env["staging_release"]["state"] == "released"
    assert env["daemon_status_response"] is None and env["daemon_cleanup_response"]["ok"]


# ---- binding the client's buffers around the executor ----------------------------------------------

class BindingProbe:
    """Executor that records what the backend has bound when it runs."""

    def __init__(self, backend):
        self.backend, self.seen = backend, None

    def execute_bound(self, request, slot, resources):
        self.seen = dict(registered=dict(self.backend.registered), open=dict(self.backend.open),
                         device=self.backend.device, host_ptr=resources.host_ptr, dev_ptr=resources.device_ptr,
                         direction=request.data_plane.direction)
        return WorkerTransferResult(request.transfer_id, "complete",
                                    bytes_completed=sum(c["bytes"] for c in request.data_plane.ranges))


def _d2h_authorization(rig):
    sid = rig.daemon.register_session(0, [1, 2, 3], max_inflight_chunks=4096).payload["session"]["session_id"]
    assert rig.daemon.register_job("job", session_id=sid).ok
    for reg in (rig.host.buffer_registration(), rig.dev.buffer_registration()):
        assert rig.daemon.register_buffer(**asdict(reg)).ok
    req = TransferRequest.from_ranges([(0, 0, N)], chunk_bytes=MiB, direction="d2h", mode="relay", job_id="job",
                                      metadata={"buffer_ids": ("dev", "host")})
    p = InProcessDaemonClient(rig.daemon).plan_transfer_request(sid, req, mode="relay").payload
    tok = p["lease_tokens"][0]
    return WorkerTransferAuthorizationRequest(transfer_id=p["transfer_id"], lease_id=tok["lease_id"],
                                              token=tok["token"], session_id=sid, job_id="job", src_buffer_id="dev",
                                              dst_buffer_id="host", direction="d2h")


@pytest.mark.parametrize("direction", ["h2d", "d2h"])
def test_buffers_are_bound_before_the_executor_and_closed_after(rig, direction):
    probe = BindingProbe(rig.backend)
    client = WorkerTransferClient(rig.dc, executor=probe, staging_pool=rig.pool,
                                  resource_binder=WorkerDataPlaneResourceBinder(rig.backend))
    rig.backend.device = 7  # the binder selects the buffer's device before opening its handle
    req = rig.authorization()[0] if direction == "h2d" else _d2h_authorization(rig)
    lc = client.submit_report_cleanup_lifecycle(req)
    assert lc.final_state == "complete", lc.error
    s = probe.seen
    assert s["direction"] == direction and s["device"] == 0
    assert s["dev_ptr"] == rig.dev_arr.ctypes.data and s["dev_ptr"] in s["open"]
    assert s["registered"], "the shared CPU buffer is page-locked before the executor runs"
    assert rig.backend.open == {} and rig.backend.registered == {}


def test_a_resource_binding_failure_is_a_failed_transfer(rig):
    req, p = rig.authorization()
    rig.backend.handles.clear()  # the device handle can no longer be opened
    lc = rig.service.handle_lifecycle(req)
    assert lc.final_state == "failed" and "bind" in (lc.error or "")
    assert rig.status(p["transfer_id"]) == "failed" and len(rig.pool) == 0
    assert rig.daemon.describe().payload["reservations"] == {}
    assert rig.backend.registered == {}, "the host registration is undone"


def test_authorization_failure_takes_no_staging(rig):
    req, _ = rig.authorization(token="forged")
    pool = CountingPool()
    client = WorkerTransferClient(rig.dc, executor=rig.client.executor, staging_pool=pool)
    lc = client.submit_report_cleanup_lifecycle(req)
    assert lc.final_state == "authorization_failed" and pool.allocations == 0
    assert lc.cleanup_response is not None and lc.cleanup_response.ok
    assert rig.daemon.describe().payload["reservations"] == {} or req.lease_id not in \
        rig.daemon.describe().payload["reservations"]


# ---- payload parser, envelopes, codec and endpoint -------------------------------------------------

AUTH = {"transfer_id": "t", "lease_id": "l", "token": "k", "session_id": "s", "job_id": "j", "src_buffer_id": "a",
        "dst_buffer_id": "b", "direction": "h2d"}


def test_payload_parser_accepts_plain_and_nested_dicts():
    a = parse_worker_authorization_request_payload(AUTH)
    b = parse_worker_authorization_request_payload({"authorization": dict(AUTH, relay_gpu=2)})
    assert a.transfer_id == b.transfer_id == "t" and b.relay_gpu == 2 and a.relay_gpu is None
    c = parse_worker_authorization_request_payload(dict(AUTH, ranges=[{"src_offset": 0, "dst_offset": 0,
                                                                        "bytes": 16}]))
    assert c.ranges[0]["bytes"] == 16


@pytest.mark.parametrize("payload,msg", [
    ({k: v for k, v in AUTH.items() if k != "token"}, "token"),
    (dict(AUTH, direction="sideways"), "direction"),
    (dict(AUTH, ranges=[{"src_offset": 0, "dst_offset": 0, "bytes": -4}]), "bytes"),
    ({"authorization": 5}, "mapping"),
    ([AUTH], "mapping"),
], ids=["missing-field", "bad-direction", "bad-range", "nested-not-mapping", "not-mapping"])
def test_payload_parser_rejections(payload, msg):
    with pytest.raises(ValueError, match=msg):
        parse_worker_authorization_request_payload(payload)


def test_request_envelope_serialises_and_checks_its_cleanup_target():
    env = WorkerServiceRequestEnvelope(payload={"authorization": AUTH}, cleanup_target_kind="session")
    assert env.as_dict() == {"payload": {"authorization": AUTH}, "cleanup_target_kind": "session"}
    with pytest.raises(ValueError, match="reservation or session"):
        WorkerServiceRequestEnvelope(payload={}, cleanup_target_kind="job")
    with pytest.raises(ValueError, match="mapping"):
        WorkerServiceRequestEnvelope(payload=[1])


def test_request_codec_round_trip_bytes_and_errors():
    env = WorkerServiceRequestEnvelope(payload={"authorization": AUTH})
    line = encode_worker_request_envelope(env)
    assert decode_worker_request_envelope(line.encode()) == env
    for bad in ("{not json", '{"cleanup_target_kind": "reservation"}', '{"payload": 3}', "[]"):
        with pytest.raises(WorkerMessageCodecError):
            decode_worker_request_envelope(bad)
    with pytest.raises(WorkerMessageCodecError):
        decode_worker_request_envelope('{"payload": {}, "cleanup_target_kind": "job"}')
    with pytest.raises(TypeError):
        encode_worker_request_envelope({"payload": {}})


def test_response_codec_round_trips_errors_and_completions(rig):
    err = WorkerServiceResponseEnvelope.from_error("lease expired")
    assert decode_worker_response_envelope(encode_worker_response_envelope(err)) == err
    req, _ = rig.authorization()
    done = WorkerServiceResponseEnvelope.from_lifecycle(rig.service.handle_lifecycle(req))
    back = decode_worker_response_envelope(encode_worker_response_envelope(done).encode())
    assert back.as_dict() == json.loads(json.dumps(done.as_dict()))  # tuples come back as lists
    assert back.ok and back.completion["final_state"] == "complete"
    for bad in ("{", '{"completion": {}}', '{"ok": true, "completion": 3}'):
        with pytest.raises(WorkerMessageCodecError):
            decode_worker_response_envelope(bad)


def _line(req, kind="reservation"):
    return encode_worker_request_envelope(WorkerServiceRequestEnvelope(payload={"authorization": asdict(req)},
                                                                       cleanup_target_kind=kind))


def test_message_handler_answers_success_parse_errors_and_status_failures(rig):
    req, _ = rig.authorization()
    ok = decode_worker_response_envelope(handle_worker_service_message(rig.service, _line(req)))
    assert ok.ok and ok.final_state == "complete" and ok.completion["transfer_id"] == req.transfer_id
    bad = decode_worker_response_envelope(handle_worker_service_message(rig.service, "{broken"))
    assert not bad.ok and bad.error
    other = Rig()  # a second session on the same node would find its relays taken
    try:
        req2, _ = other.authorization()
        other.dc.fail["transfer_status"] = "status store offline"
        st = decode_worker_response_envelope(handle_worker_service_message(other.service, _line(req2)))
    finally:
        other.close()
    assert st.ok and st.final_state == "status_failed" and "offline" in st.error
    assert st.completion["staging_release"]["state"] == "released"


def test_endpoint_matches_the_message_handler(rig):
    ep = WorkerServiceEndpoint(service=rig.service)
    assert WorkerServiceEndpoint(rig.service).service is rig.service
    for line in ("{broken", '{"payload": {"authorization": {"transfer_id": "x"}}}'):
        assert ep.handle_message(line) == handle_worker_service_message(rig.service, line)
    req, _ = rig.authorization(token="forged")
    a = decode_worker_response_envelope(ep.handle_message(_line(req)))
    assert a.ok and a.final_state == "authorization_failed" and "token" in a.error
    with pytest.raises(ValueError, match="daemon client"):
        WorkerServiceEndpoint()
    with pytest.raises(TypeError):
        WorkerServiceEndpoint(service=object())
    assert isinstance(WorkerServiceEndpoint(Recorder()).service, WorkerTransferService)


def test_service_envelopes_for_each_final_state(rig):
    req, _ = rig.authorization()
    rig.dc.fail["cleanup"] = "cleanup store offline"
    rig.dc.fail["release_transfer"] = "release store offline"
    env = rig.service.handle_envelope({"payload": {"authorization": asdict(req)}})
    assert env.ok and env.final_state == "cleanup_failed" and "offline" in env.error
    assert env.completion["staging_release"]["state"] == "released"
    malformed = rig.service.handle_envelope({"payload": {"authorization": {"transfer_id": "x"}}})
    assert not malformed.ok and "missing worker authorization field" in malformed.error
    assert rig.service.handle_envelope_payload({"payload": 4})["ok"] is False
    with pytest.raises(ValueError, match="daemon_client or transfer_client"):
        WorkerTransferService()
    with pytest.raises(TypeError):
        rig.service.handle_lifecycle(asdict(req))
