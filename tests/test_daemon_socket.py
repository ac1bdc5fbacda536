"""The daemon over a real AF_UNIX socket (served on a thread): every RPC
stub round-trips, persistent connections, connection-scoped sessions that
end with their connection, SO_PEERCRED identities bound to jobs and
buffers, malformed and unknown messages, and the socket lifecycle.
Behaviours follow integration/test_daemon_socket.py of the reference with
independent fixtures."""

from __future__ import annotations

import json
import os
import socket
import threading
import time

import pytest

from pcie_pool_b200.daemon import TurboBusDaemon
from pcie_pool_b200.daemon.client import TurboBusDaemonClient
from pcie_pool_b200.daemon.wire import serve_unix
from pcie_pool_b200.schema import TransferIntent
from pcie_pool_b200.topology import StaticTopologyProvider
from pcie_pool_b200.transfer import TransferRequest

MiB = 1 << 20


def _profile():
    return {"target_device": 0, "direct_h2d_bw_gbps": 20.0, "direct_d2h_bw_gbps": 20.0,
            "relays": [{"relay_device": r, "target_device": 0, "h2d_bw_gbps": 20.0, "d2h_bw_gbps": 20.0,
                        "p2p_bw_gbps": 400.0, "effective_bw_gbps": 20.0, "effective_d2h_bw_gbps": 20.0,
                        "p2p_enabled": True} for r in (1, 2, 3)]}


@pytest.fixture
def served(tmp_path):
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_sessions_per_relay=8, max_inflight_chunks_per_relay=4096,
                       topology_provider=StaticTopologyProvider(gpu_count=4))
    path = str(tmp_path / "daemon.sock")
    stop, ready = threading.Event(), threading.Event()
    t = threading.Thread(target=serve_unix, args=(d, path), kwargs={"stop_event": stop, "ready_event": ready},
                         daemon=True)
    t.start()
    assert ready.wait(5)
    yield d, path
    stop.set()
    t.join(5)
    assert not os.path.exists(path), "the socket file is removed when serving stops"


def _raw(path: str, line: bytes) -> dict:
    with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as c:
        c.settimeout(5)
        c.connect(path)
        c.sendall(line)
        data = b""
        while b"\n" not in data:
            chunk = c.recv(65536)
            if not chunk:
                break
            data += chunk
    return json.loads(data.split(b"\n", 1)[0])


def _setup(c: TurboBusDaemonClient, job: str = "job") -> str:
    s = c.register_session(0, [1, 2, 3], max_inflight_chunks=64)
    assert s.ok, s.error
    sid = s.payload["session"]["session_id"]
    assert c.register_job(job, session_id=sid).ok
    assert c.register_buffer(f"src-{job}", job, "cpu_pinned", 64 * MiB, address=4096, pinned=True).ok
    assert c.register_buffer(f"dst-{job}", job, "gpu", 64 * MiB, device_index=0, address=8192).ok
    return sid


def test_every_stub_round_trips(served):
    d, path = served
    c = TurboBusDaemonClient(path, timeout=10)
    assert c.get_inventory().ok
    assert c.invalidate_topology().ok
    assert c.discover_relays(0, [1, 2]).ok
    assert c.put_profile(0, [1, 2, 3], _profile()).ok
    assert c.get_profile(0, [1, 2, 3]).payload["profile"]["profile"]["direct_h2d_bw_gbps"] == 20.0
    sid = _setup(c)
    req = TransferRequest.from_ranges([(0, 0, 64 * MiB)], chunk_bytes=16 * MiB, direction="h2d", mode="pool",
                                      job_id="job", metadata={"buffer_ids": ("src-job", "dst-job")})
    p = c.plan_transfer_request(sid, req)
    assert p.ok, p.error
    tok = p.payload["lease_tokens"][0]
    assert c.validate_lease(tok["lease_id"], tok["token"]).ok
    tid = p.payload["transfer_id"]
    assert c.transfer_status(tid).payload["status"]["state"] == "submitted"
    r = c.reschedule_transfer(tid)
    assert r.ok and r.payload["plan_generation"] == 2
    assert c.transfer_status(tid, state="complete", bytes_completed=64 * MiB).ok
    for t in r.payload["lease_tokens"]:
        assert c.release_transfer(t["lease_id"]).ok
    res = c.reserve_transfer(sid, 1, 2, bytes_=MiB, direction="h2d")
    assert res.ok and c.release_transfer(res.payload["reservation"]["reservation_id"]).ok
    assert c.reap_expired_leases().ok
    assert c.invalidate_profile(0, [1, 2, 3]).payload["removed"]
    assert c.cleanup("job", "job", "test").ok
    assert c.close_session(sid).ok
    assert c.describe().ok


def test_intents_over_the_socket_are_idempotent(served):
    d, path = served
    c = TurboBusDaemonClient(path, timeout=10)
    assert c.put_profile(0, [1, 2, 3], _profile()).ok
    sid = _setup(c)
    it = TransferIntent("wire-i1", "job", sid, "src-job", "dst-job", "h2d", 32 * MiB,
                        ({"src_offset": 0, "dst_offset": 0, "bytes": 32 * MiB},), metadata={"chunk_bytes": 8 * MiB})
    a = c.submit_transfer_intent(it)
    b = c.submit_transfer_intent(it)
    assert a.ok and b.ok and a.payload["transfer_id"] == b.payload["transfer_id"]
    rec = c.wait_transfer_receipt("wire-i1").payload["receipt"]
    assert rec["intent_id"] == "wire-i1" and rec["metadata"]["transfer_id"] == a.payload["transfer_id"]


def test_persistent_connection_serves_many_requests(served):
    _d, path = served
    c = TurboBusDaemonClient(path, persistent=True, timeout=10)
    try:
        t0 = time.perf_counter()
        for _ in range(50):
            assert c.get_inventory().ok
        assert time.perf_counter() - t0 < 10
    finally:
        c.close()


def test_connection_scoped_session_ends_with_its_connection(served):
    d, path = served
    c = TurboBusDaemonClient(path, persistent=True, timeout=10)
    s = c.register_session(0, [1], max_inflight_chunks=8, connection_scoped=True)
    assert s.ok and s.payload.get("connection_scoped")
    sid = s.payload["session"]["session_id"]
    assert sid in d.describe().payload["sessions"]
    c.close()
    for _ in range(200):
        if sid not in d.describe().payload["sessions"]:
            break
        time.sleep(0.01)
    assert sid not in d.describe().payload["sessions"], "closing the connection closed the session"
    # a session that is not connection scoped outlives its (one-shot) connection
    plain = TurboBusDaemonClient(path, timeout=10).register_session(0, [2])
    assert plain.payload["session"]["session_id"] in d.describe().payload["sessions"]


def test_peer_credentials_bind_jobs(served):
    d, path = served
    c = TurboBusDaemonClient(path, timeout=10)
    assert c.register_job("mine").ok
    ident = d.describe().payload["job_peer_identities"]["mine"]
    assert ident["authenticated"] and ident["process_id"] == os.getpid()
    assert ident["user_id"] == str(os.getuid())
    r = c.register_job("spoof", user_id="somebody-else")
    assert not r.ok and "does not match" in r.error


def test_malformed_and_unknown_messages_get_error_replies(served):
    _d, path = served
    assert not _raw(path, b"{not json}\n")["ok"]
    assert not _raw(path, b"[1, 2]\n")["ok"]
    assert not _raw(path, json.dumps({"request_type": "NO_SUCH_TYPE"}).encode() + b"\n")["ok"]
    assert not _raw(path, json.dumps({"request_type": "register_session", "payload": "x"}).encode() + b"\n")["ok"]
    bad = _raw(path, json.dumps({"request_type": "register_session", "payload": {}}).encode() + b"\n")
    assert not bad["ok"] and "invalid request" in bad["error"]
    # the server is still healthy afterwards
    assert TurboBusDaemonClient(path, timeout=10).get_inventory().ok


def test_concurrent_clients(served):
    _d, path = served
    errors = []

    def worker(i):
        try:
            c = TurboBusDaemonClient(path, timeout=10)
            s = c.register_session(0, [1 + i % 3], max_inflight_chunks=4)
            assert s.ok, s.error
            assert c.close_session(s.payload["session"]["session_id"]).ok
        except Exception as exc:  # noqa: BLE001 - collected for the assertion
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(12)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(10)
    assert not errors, errors
