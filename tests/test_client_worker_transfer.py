"""App-side worker-managed transfer client: direct-only plans run in the app
process under a daemon ticket, relay plans go to the worker; every check the
client makes on plans, leases, tickets, worker completions and the daemon's
final status, each with the case that must be refused.  The daemon is real
(in-process), the data plane is the mock lanes.  Behaviours follow
integration/test_client_worker_transfer.py of the reference with
independent fixtures."""

from __future__ import annotations

import pytest

from pcie_pool_b200.client_transfer import (_CompletionError, check_direct_plan, check_plan_matches_leases,
                                            check_worker_completion, direct_ticket, is_direct_only_plan,
                                            require_daemon_complete)
from pcie_pool_b200.schema import WorkerTransferAuthorizationRequest
from pcie_pool_b200.transfer import TransferRequest
from pcie_pool_b200.worker import WorkerServiceResponseEnvelope

MiB = 1 << 20


def _plan(kind="direct", direction="h2d", chunks=((0, 0, 4 * MiB),), target=0, relay=-1, total=None, enabled=True):
    ch = [{"src_offset": s, "dst_offset": d, "bytes": n} for s, d, n in chunks]
    return {"total_bytes": sum(c["bytes"] for c in ch) if total is None else total, "chunk_bytes": 4 * MiB,
            "assignments": [{"path": {"kind": kind, "direction": direction, "target_device": target,
                                      "relay_device": relay, "enabled": enabled}, "chunks": ch}]}


@pytest.mark.parametrize("plan,msg", [
    (_plan(kind="relay", relay=1), "direct paths"),
    (_plan(direction="d2h"), "direction"),
    (_plan(target=1), "target"),
    (_plan(enabled=False), "disabled"),
    (_plan(chunks=((0, 0, 0),)), "positive"),
    (_plan(chunks=((8 * MiB, 0, 4 * MiB),)), "source buffer"),
    (_plan(chunks=((0, 8 * MiB, 4 * MiB),)), "destination buffer"),
    (_plan(total=5), "total bytes"),
    ({"assignments": []}, "no assignments"),
])
def test_direct_plan_checks(plan, msg):
    with pytest.raises(RuntimeError, match=msg):
        check_direct_plan(plan, 0, "h2d", 8 * MiB, 8 * MiB)


def test_direct_plan_accepts_a_valid_plan_and_swaps_sizes_for_d2h():
    check_direct_plan(_plan(), 0, "h2d", 8 * MiB, 8 * MiB)
    # d2h: the source is the device buffer
    check_direct_plan(_plan(direction="d2h", chunks=((4 * MiB, 0, 4 * MiB),)), 0, "d2h", 4 * MiB, 8 * MiB)


def test_direct_only_detection():
    assert is_direct_only_plan({"plan": _plan()})
    assert not is_direct_only_plan({"plan": _plan(), "reservations": [{}]})
    assert not is_direct_only_plan({"plan": _plan(kind="relay", relay=2)})
    assert not is_direct_only_plan({"plan": {}})


def test_plan_must_match_leases():
    p = {"plan": _plan(kind="relay", relay=2)}
    check_plan_matches_leases(p, [{"relay_gpu": 2}], "h2d")
    with pytest.raises(RuntimeError, match="do not match"):
        check_plan_matches_leases(p, [{"relay_gpu": 3}], "h2d")
    with pytest.raises(RuntimeError, match="requires relay leases"):
        check_plan_matches_leases(p, [], "h2d")
    with pytest.raises(RuntimeError, match="direction"):
        check_plan_matches_leases({"plan": _plan(kind="relay", relay=2, direction="d2h")}, [{"relay_gpu": 2}], "h2d")
    with pytest.raises(RuntimeError, match="did not include worker chunks"):
        check_plan_matches_leases({"plan": _plan()}, [{"relay_gpu": 2}], "h2d")


def _auth():
    return WorkerTransferAuthorizationRequest(transfer_id="t", lease_id="l", token="k", session_id="s", job_id="j",
                                              src_buffer_id="a", dst_buffer_id="b", direction="h2d")


def _completion(**over):
    c = {"ok": True, "transfer_id": "t", "lease_id": "l",
         "worker_result": {"state": "complete", "transfer_id": "t", "bytes_completed": 64},
         "daemon_status_update": {"transfer_id": "t", "state": "complete", "bytes_completed": 64},
         "daemon_status_response": {"ok": True}, "daemon_cleanup_response": {"ok": True},
         "staging_release": {"transfer_id": "t"}}
    c.update(over)
    return c


def test_worker_completion_accepts_a_consistent_record():
    env = WorkerServiceResponseEnvelope(ok=True, completion=_completion(), final_state="complete")
    assert check_worker_completion(env, _auth(), 64)["transfer_id"] == "t"
    failed = WorkerServiceResponseEnvelope(ok=True, completion=_completion(worker_result=None), final_state="failed")
    assert check_worker_completion(failed, _auth(), 64), "a failed lifecycle is returned for the caller to raise"


@pytest.mark.parametrize("over,msg", [
    ({"ok": False}, "not ok"),
    ({"transfer_id": "x"}, "transfer mismatch"),
    ({"lease_id": ""}, "missing lease"),
    ({"worker_result": {"state": "failed", "transfer_id": "t", "bytes_completed": 0}}, "did not complete"),
    ({"worker_result": {"state": "complete", "transfer_id": "t", "bytes_completed": 60}}, "60 of 64"),
    ({"daemon_status_update": {"transfer_id": "t", "state": "complete", "bytes_completed": 1}}, "byte count"),
    ({"daemon_status_response": {"ok": False}}, "not accepted"),
    ({"daemon_cleanup_response": None}, "release was not accepted"),
    ({"staging_release": {"transfer_id": "other"}}, "staging release"),
])
def test_worker_completion_rejections(over, msg):
    env = WorkerServiceResponseEnvelope(ok=True, completion=_completion(**over), final_state="complete")
    with pytest.raises(_CompletionError, match=msg):
        check_worker_completion(env, _auth(), 64)


def test_worker_error_envelope_is_rejected():
    with pytest.raises(_CompletionError, match="boom"):
        check_worker_completion(WorkerServiceResponseEnvelope(ok=False, error="boom"), _auth(), 64)


def test_daemon_final_status_must_account_for_every_byte():
    require_daemon_complete({"state": "complete", "bytes_completed": 10}, 10)
    with pytest.raises(RuntimeError, match="not complete"):
        require_daemon_complete({"state": "failed", "bytes_completed": 0}, 10)
    with pytest.raises(RuntimeError, match="9 of 10"):
        require_daemon_complete({"state": "complete", "bytes_completed": 9}, 10)


def test_direct_ticket_checks_against_the_request():
    """A real direct-mode plan from the daemon: its ticket passes, and each
    field a client checks is refused when it does not match."""
    from pcie_pool_b200.daemon import TurboBusDaemon
    from pcie_pool_b200.topology import StaticTopologyProvider

    d = TurboBusDaemon(relay_gpus=[1], topology_provider=StaticTopologyProvider(gpu_count=2))
    sid = d.register_session(0, [1]).payload["session"]["session_id"]
    assert d.register_job("j", session_id=sid).ok
    assert d.register_buffer("a", "j", "cpu_pinned", 8 * MiB, address=4096, pinned=True).ok
    assert d.register_buffer("b", "j", "gpu", 8 * MiB, device_index=0, address=8192).ok
    req = TransferRequest.from_ranges([(0, 0, 8 * MiB)], chunk_bytes=2 * MiB, direction="h2d", mode="direct",
                                      job_id="j", metadata={"buffer_ids": ("a", "b")})
    from pcie_pool_b200.daemon import InProcessDaemonClient

    p = InProcessDaemonClient(d).plan_transfer_request(sid, req, mode="direct").payload
    tid = p["transfer_id"]
    t = direct_ticket(p, req, tid, "j", "a", "b")
    assert t.metadata["issuer"] == "turbobus-daemon" and not t.lease_ids
    for args, msg in (((tid, "other", "a", "b"), "job"), ((tid, "j", "b", "a"), "source buffer"),
                      (("other-tid", "j", "a", "b"), "transfer")):
        with pytest.raises(RuntimeError, match=msg):
            direct_ticket(p, req, *args)
    smaller = TransferRequest.from_ranges([(0, 0, 4 * MiB)], chunk_bytes=2 * MiB, direction="h2d", mode="direct",
                                          job_id="j")
    with pytest.raises(RuntimeError, match="byte total"):
        direct_ticket(p, smaller, tid, "j", "a", "b")
    with pytest.raises(RuntimeError, match="did not include execution ticket"):
        direct_ticket({**p, "ticket": None}, req, tid, "j", "a", "b")
    forged = {**p, "ticket": {**p["ticket"], "metadata": {**p["ticket"]["metadata"], "issuer": "me"}}}
    with pytest.raises(RuntimeError, match="issued by"):
        direct_ticket(forged, req, tid, "j", "a", "b")


def test_direct_fallback_runs_in_the_app_process_on_the_mock_world():
    """mode='direct': no worker is involved; the client executes the daemon's
    direct ticket on its own data plane and reports completion."""
    from test_worker_lifecycle import Rig

    from pcie_pool_b200.client_transfer import WorkerManagedTransferClient

    class NoWorker:
        def submit(self, env):  # pragma: no cover - must not be reached
            raise AssertionError("a direct-only plan must not reach the worker")

    rig = Rig()
    try:
        moved = []
        c = WorkerManagedTransferClient(daemon_client=rig.dc, worker_client=NoWorker(), target_gpu=0,
                                        relay_gpus=[1, 2, 3], max_inflight_chunks=4096)

        def run_direct(direction, ticket, source, target):
            # stands in for the app-side engine (which needs a GPU): check the
            # ticket's plan against the buffers and "move" the bytes
            check_direct_plan(ticket.plan, 0, direction, source.size_bytes, target.size_bytes)
            moved.append(ticket.total_bytes)
            return {"bytes": ticket.total_bytes, "cuda_ms": 1.0, "gb_per_s": 1.0}

        c._run_direct = run_direct
        res = c.fetch_shared_cpu_to_cuda_ipc(rig.host, rig.dev, chunk_bytes=2 * MiB, mode="direct")
        assert res.state == "complete" and moved == [8 * MiB] and res.path != "worker"
        assert rig.daemon.describe().payload["reservations"] == {}
    finally:
        rig.close()
