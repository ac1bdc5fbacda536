"""Worker-managed transfers on the CPU: real daemon (planning, leases,
authorization, status, cleanup), real worker helper lifecycle, codec and
unix-socket transport; the byte movement goes through the mock lanes and the
CUDA calls through a mock backend.  Mirrors the reference's
test_worker_helper / test_worker_transport / test_worker_process /
test_client_worker_transfer / test_worker_staging_pool suites with its own
fixtures."""

import os
import tempfile
import threading
from dataclasses import asdict

import numpy as np
import pytest

from pcie_pool_b200.client import CudaIpcDeviceBuffer, SharedPinnedCpuBuffer
from pcie_pool_b200.client_transfer import WorkerManagedTransferClient, is_direct_only_plan
from pcie_pool_b200.daemon import InProcessDaemonClient, TurboBusDaemon
from pcie_pool_b200.mock import FaultPlan, MockCudaBackend, MockDataPlane, MockWorkerExecutor, MockWorld
from pcie_pool_b200.schema import ExecutionTicket, WorkerTransferAuthorizationRequest
from pcie_pool_b200.topology import StaticTopologyProvider
from pcie_pool_b200.worker import (WorkerDataPlaneCompletionEnvelope, WorkerDataPlaneResourceBinder, WorkerMessageCodecError,
                                   WorkerServiceRequestEnvelope, WorkerServiceSocketClient,
                                   WorkerServiceUnixSocketTransport, WorkerStagingPool, WorkerStagingPoolError,
                                   WorkerTransferClient, WorkerTransferService, build_worker_helper_transport,
                                   decode_worker_request_envelope, decode_worker_response_envelope,
                                   encode_worker_request_envelope)
from pcie_pool_b200.worker.helper import WorkerTransferRequest, validate_daemon_ticket

MiB = 1 << 20


class Node:
    def __init__(self, gpus=4, faults=None):
        self.world = MockWorld(gpu_count=gpus)
        self.daemon = TurboBusDaemon(relay_gpus=range(1, gpus), max_inflight_chunks_per_relay=4096,
                                     topology_provider=StaticTopologyProvider(gpu_count=gpus))
        self.daemon.put_profile(0, list(range(1, gpus)), self.world.profile(0))
        self.dc = InProcessDaemonClient(self.daemon)
        self.backend = MockCudaBackend()
        self.executor = MockWorkerExecutor(MockDataPlane(self.world, faults=faults))
        self.service = WorkerTransferService(transfer_client=WorkerTransferClient(
            self.dc, executor=self.executor, resource_binder=WorkerDataPlaneResourceBinder(self.backend)))

    def client(self, worker=None, relays=(1, 2, 3)):
        return WorkerManagedTransferClient(daemon_client=self.dc, worker_client=worker or self.service,
                                           target_gpu=0, relay_gpus=list(relays), max_inflight_chunks=4096)

    def buffers(self, n, job="job", seed=0):
        host = SharedPinnedCpuBuffer.allocate("host", job, n)
        host.numpy()[:] = np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)
        dev_arr = self.world.alloc(0, n)
        dev = CudaIpcDeviceBuffer("dev", job, 0, n, self.backend.export_device_ipc_handle(dev_arr.ctypes.data),
                                  device_ptr=dev_arr.ctypes.data)
        return host, dev, dev_arr


@pytest.fixture
def node():
    return Node()


def test_worker_managed_h2d_then_d2h_roundtrip(node):
    host, dev, dev_arr = node.buffers(32 * MiB)
    c = node.client()
    try:
        r = c.fetch_shared_cpu_to_cuda_ipc(host, dev, chunk_bytes=2 * MiB, mode="pool")
        assert r.state == "complete" and r.bytes_completed == 32 * MiB
        assert np.array_equal(dev_arr, host.numpy())
        assert r.path == "pool_h2d" and len(r.lease_tokens) == 3
        assert r.worker_completion["final_state"] == "complete"
        dev_arr[:] ^= 0x5A
        r2 = c.offload_cuda_ipc_to_shared_cpu(dev, host, chunk_bytes=2 * MiB, mode="relay")
        assert r2.state == "complete" and np.array_equal(host.numpy(), dev_arr)
        assert r2.path == "relay_d2h"
        desc = node.daemon.describe().payload
        assert desc["reservations"] == {}, "leases released after both transfers"
        # the worker opened and closed the IPC handle and the shm host registration each time
        assert node.backend.open == {} and node.backend.registered == {}
    finally:
        host.release()


def test_worker_lifecycle_reports_failure_and_cleans_leases():
    node = Node(faults=FaultPlan(fail_lane=2))
    host, dev, _ = node.buffers(8 * MiB)
    c = node.client()
    try:
        with pytest.raises(RuntimeError, match="injected failure"):
            c.fetch_shared_cpu_to_cuda_ipc(host, dev, chunk_bytes=1 * MiB, mode="relay")
        desc = node.daemon.describe().payload
        assert desc["reservations"] == {}
        states = {q["state"] for q in desc["transfer_queue"]}
        assert states == {"failed"}
    finally:
        host.release()


def test_authorization_failure_is_recorded_and_cleaned(node):
    host, dev, _ = node.buffers(8 * MiB)
    c = node.client()
    try:
        sid = c.open_session()
        node.dc.register_job(job_id="job", session_id=sid)
        for reg in (host.buffer_registration(), dev.buffer_registration()):
            node.dc.register_buffer(**{k: v for k, v in asdict(reg).items()})
        from pcie_pool_b200.transfer import TransferRequest

        req = TransferRequest.from_ranges([(0, 0, 8 * MiB)], chunk_bytes=MiB, direction="h2d", mode="relay",
                                          job_id="job", metadata={"buffer_ids": ("host", "dev")})
        p = node.dc.plan_transfer_request(sid, req, mode="relay").payload
        tok = p["lease_tokens"][0]
        bad = WorkerTransferAuthorizationRequest(transfer_id=p["transfer_id"], lease_id=tok["lease_id"],
                                                 token="not-the-token", session_id=sid, job_id="job",
                                                 src_buffer_id="host", dst_buffer_id="dev", direction="h2d",
                                                 relay_gpu=tok["relay_gpu"])
        lc = node.service.handle_lifecycle(bad)
        assert lc.final_state == "authorization_failed" and "token" in lc.error
        assert lc.cleanup_response.ok and lc.cleanup_target_id == tok["lease_id"]
        env = node.service.handle_envelope_payload({"payload": {"authorization": asdict(bad)}})
        assert env["ok"] and env["final_state"] in ("authorization_failed", "cleanup_failed")
    finally:
        host.release()


def test_ticket_validation_rules(node):
    t = ExecutionTicket(ticket_id="t", decision_id="d", intent_id="i", topology_snapshot_id="s", job_id="j",
                        session_id="x", source_buffer_id="a", destination_buffer_id="b", direction="h2d",
                        total_bytes=16, ranges=({"src_offset": 0, "dst_offset": 0, "bytes": 16},),
                        plan={"assignments": []}, issued_at=0.0, expires_at=1.0, lease_ids=("l",),
                        metadata={"issuer": "someone-else", "plan_generation": 1, "transfer_id": "x"})
    with pytest.raises(ValueError, match="issued by"):
        validate_daemon_ticket(t)
    t2 = ExecutionTicket(**{**asdict(t), "metadata": {"issuer": "turbobus-daemon", "plan_generation": 0,
                                                      "transfer_id": "x"}})
    with pytest.raises(ValueError, match="positive"):
        validate_daemon_ticket(t2)
    t3 = ExecutionTicket(**{**asdict(t), "metadata": {"issuer": "turbobus-daemon", "plan_generation": 2,
                                                      "transfer_id": "x"}})
    with pytest.raises(ValueError, match="stale"):
        validate_daemon_ticket(t3, plan_generation=3)
    with pytest.raises(ValueError, match="ExecutionTicket"):
        WorkerTransferRequest.from_authorization(None)


def test_staging_pool_ids_alignment_and_validation(node):
    host, dev, _ = node.buffers(4 * MiB + 100)
    try:
        c = node.client()
        sid = c.open_session()
        node.dc.register_job(job_id="job", session_id=sid)
        for reg in (host.buffer_registration(), dev.buffer_registration()):
            node.dc.register_buffer(**{k: v for k, v in asdict(reg).items()})
        from pcie_pool_b200.transfer import TransferRequest

        req = TransferRequest.from_ranges([(0, 0, 4 * MiB + 100)], chunk_bytes=MiB, direction="h2d", mode="relay",
                                          job_id="job", metadata={"buffer_ids": ("host", "dev")})
        p = node.dc.plan_transfer_request(sid, req, mode="relay").payload
        tok = p["lease_tokens"][0]
        auth = WorkerTransferAuthorizationRequest(transfer_id=p["transfer_id"], lease_id=tok["lease_id"],
                                                  token=tok["token"], session_id=sid, job_id="job",
                                                  src_buffer_id="host", dst_buffer_id="dev", direction="h2d",
                                                  relay_gpu=tok["relay_gpu"])
        wr = WorkerTransferClient(node.dc, executor=node.executor).authorize(auth)
        pool = WorkerStagingPool()
        s1, s2 = pool.allocate(wr.data_plane), pool.allocate(wr.data_plane)
        assert (s1.slot_id, s2.slot_id) == ("staging-1", "staging-2")
        assert s1.allocated_bytes % 256 == 0 and s1.allocated_bytes >= s1.requested_bytes
        assert pool.validate_slot_for_request("staging-1", wr.data_plane) == s1
        assert pool.release("staging-1", wr.data_plane).state == "released"
        with pytest.raises(WorkerStagingPoolError):
            pool.release("staging-1")
        assert len(pool) == 1
        node.dc.cleanup(target_kind="session", target_id=sid, reason="test", force=True)
    finally:
        host.release()


def test_codec_roundtrip_and_errors():
    env = WorkerServiceRequestEnvelope(payload={"authorization": {"b": 1, "a": 2}})
    line = encode_worker_request_envelope(env)
    assert line == '{"cleanup_target_kind":"reservation","payload":{"authorization":{"a":2,"b":1}}}'
    assert decode_worker_request_envelope(line) == env
    with pytest.raises(WorkerMessageCodecError):
        decode_worker_request_envelope("[1]")
    with pytest.raises(WorkerMessageCodecError):
        decode_worker_response_envelope('{"completion": 3, "ok": true}')
    with pytest.raises(ValueError):
        WorkerServiceRequestEnvelope(payload={}, cleanup_target_kind="everything")


def test_worker_over_unix_sockets_with_threaded_daemon():
    """Daemon and worker each behind their own AF_UNIX socket; the client
    talks to both over the wire (one JSON line per request)."""
    from pcie_pool_b200.daemon.client import TurboBusDaemonClient
    from pcie_pool_b200.daemon.wire import serve_unix

    node = Node()
    tmp = tempfile.mkdtemp(prefix="ppb-")
    dsock, wsock = os.path.join(tmp, "d.sock"), os.path.join(tmp, "w.sock")
    stop = threading.Event()
    dthread = threading.Thread(target=serve_unix, args=(node.daemon, dsock), kwargs={"stop_event": stop},
                               daemon=True)
    dthread.start()
    for _ in range(200):
        if os.path.exists(dsock):
            break
        threading.Event().wait(0.01)
    transport = build_worker_helper_transport(dsock, wsock, executor=node.executor,
                                              resource_binder=WorkerDataPlaneResourceBinder(node.backend))
    assert isinstance(transport, WorkerServiceUnixSocketTransport)
    ready = threading.Event()
    wthread = threading.Thread(target=transport.serve_forever, kwargs={"stop_event": stop, "ready_event": ready},
                               daemon=True)
    wthread.start()
    assert ready.wait(5)
    host, dev, dev_arr = node.buffers(16 * MiB, seed=3)
    try:
        c = WorkerManagedTransferClient(daemon_client=TurboBusDaemonClient(dsock),
                                        worker_client=WorkerServiceSocketClient(wsock, 60.0), target_gpu=0,
                                        relay_gpus=[1, 2, 3], max_inflight_chunks=4096)
        r = c.fetch_shared_cpu_to_cuda_ipc(host, dev, chunk_bytes=MiB, mode="pool")
        assert r.state == "complete" and np.array_equal(dev_arr, host.numpy())
        assert c.close_session().ok
        # a malformed line gets an error envelope, not a dropped connection
        bad = decode_worker_response_envelope(WorkerServiceSocketClient(wsock, 10.0).send_message("{not json"))
        assert not bad.ok and bad.error
        # submit_envelope folds the response into a completion envelope
        env = WorkerServiceSocketClient(wsock, 10.0).submit_envelope(
            WorkerServiceRequestEnvelope(payload={"authorization": {"bogus": True}}))
        assert isinstance(env, WorkerDataPlaneCompletionEnvelope) and not env.ok and env.error
    finally:
        stop.set()
        wthread.join(5)
        dthread.join(5)
        host.release()


def test_direct_only_plan_detection():
    assert is_direct_only_plan({"plan": {"assignments": [{"path": {"kind": "direct"}, "chunks": []}]}})
    assert not is_direct_only_plan({"plan": {"assignments": [{"path": {"kind": "relay"}}]}})
    assert not is_direct_only_plan({"lease_tokens": [{}], "plan": {"assignments": [{"path": {"kind": "direct"}}]}})


def test_example_config_maps_physical_gpus(monkeypatch):
    from pcie_pool_b200.example_config import configure_cuda_runtime_mapping, parse_gpu_list

    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    m = configure_cuda_runtime_mapping(3, "5,6")
    assert (m.runtime_target_gpu, m.runtime_relay_gpus, m.cuda_visible_devices) == (0, (1, 2), "3,5,6")
    assert os.environ["CUDA_VISIBLE_DEVICES"] == "3,5,6"
    m2 = configure_cuda_runtime_mapping(3, "5,6")  # already set: identity
    assert (m2.runtime_target_gpu, m2.runtime_relay_gpus) == (3, (5, 6))
    assert parse_gpu_list(" 1, 2,,3 ") == [1, 2, 3]


def test_verification_pattern_and_daemon_seed():
    from pcie_pool_b200.verification import build_verification_daemon, make_pattern

    p = make_pattern(300)
    assert p[0] == 17 and p[1] == (131 + 17) & 0xFF and p[299] == (299 * 131 + 17) & 0xFF
    d = build_verification_daemon(0, 1, 8, 1 << 20)
    prof = d.get_profile(0, [1])
    assert prof.ok


def test_engine_data_plane_lane_failover_logic():
    """EngineDataPlane re-runs the chunks of a failed lane over a surviving
    lane (CPU: a fake engine that fails lane 1 once, then moves bytes)."""
    import ctypes

    from pcie_pool_b200.daemon.executor import EngineDataPlane
    from pcie_pool_b200.parallel.engine import LaneResult, TransferResult
    from pcie_pool_b200.schema import BufferRegistration, ExecutionTicket

    n = 8 * MiB
    host = np.random.default_rng(4).integers(0, 256, n, dtype=np.uint8)
    dev = np.zeros(n, dtype=np.uint8)

    class FakeEngine:
        def __init__(self):
            self.calls = []

        def run(self, direction, target, hp, hb, dp, db, lanes, checksum=False, **kw):
            self.calls.append(([l.device for l in lanes], kw))
            first = len(self.calls) == 1
            stats = []
            for i, l in enumerate(lanes):
                if first and i == 1:
                    continue
                for s, d, b in zip(l.src_off, l.dst_off, l.bytes):
                    ctypes.memmove(dp + int(d), hp + int(s), int(b))
                stats.append(LaneResult(l.device, l.device == target, l.total_bytes, len(l.bytes), 1.0))
            if first:
                return TransferResult(1, False, 1, "timeout waiting for a staged chunk", 0, 1000.0, 0.0, 0.0,
                                      stats, np.zeros((sum(len(l.bytes) for l in lanes), 2), np.uint64),
                                      error_lane=1, error_chunk=3)
            return TransferResult(2, True, 0, "", sum(l.total_bytes for l in lanes), 5.0, 0.0, 0.0, stats,
                                  np.ones((sum(len(l.bytes) for l in lanes), 2), np.uint64))

    eng = FakeEngine()
    plane = EngineDataPlane(engine=eng, checksum=True)
    plan = {"total_bytes": n, "assignments": [
        {"path": {"kind": "direct", "direction": "h2d", "target_device": 0},
         "chunks": [{"src_offset": o, "dst_offset": o, "bytes": MiB} for o in range(0, 4 * MiB, MiB)]},
        {"path": {"kind": "relay", "direction": "h2d", "target_device": 0, "relay_device": 1},
         "chunks": [{"src_offset": o, "dst_offset": o, "bytes": MiB} for o in range(4 * MiB, n, MiB)]}]}
    t = ExecutionTicket(ticket_id="t", decision_id="d", intent_id="i", topology_snapshot_id="s", job_id="j",
                        session_id="x", source_buffer_id="h", destination_buffer_id="g", direction="h2d",
                        total_bytes=n, ranges=({"src_offset": 0, "dst_offset": 0, "bytes": n},), plan=plan,
                        issued_at=0.0, expires_at=1.0)
    src = BufferRegistration("h", "j", "cpu_pinned", n, address=host.ctypes.data, pinned=True)
    dst = BufferRegistration("g", "j", "gpu", n, device_index=0, address=dev.ctypes.data)
    res = plane.execute(t, src, dst, None)
    assert res.ok and res.bytes_completed == n
    assert np.array_equal(dev, host)
    assert eng.calls[1][0] == [0], "failed relay chunks re-ran on the direct lane"
    fo = res.measured["failover"]
    assert fo["failed_lane_device"] == 1 and fo["rerun_on_device"] == 0 and fo["rerun_bytes"] == 4 * MiB
    assert "lane failover" in res.measured["fallback_reason"]
    # the re-run's checksums replaced the failed lane's entries (chunks 4..7)
    assert res.measured["chunk_checksums"][4:] == [[1, 1]] * 4 and res.measured["chunk_checksums"][0] == [0, 0]


def test_ipc_buffer_inside_an_allocation_lands_at_its_offset(node):
    """A device buffer that starts inside a larger allocation (a caching
    allocator's segment) travels as the allocation's handle plus an offset;
    the worker writes at the buffer, not at the allocation base."""
    n, off = 8 * MiB, 3 * MiB + 4096
    host = SharedPinnedCpuBuffer.allocate("host", "job", n)
    host.numpy()[:] = np.random.default_rng(5).integers(0, 256, n, dtype=np.uint8)
    seg = node.world.alloc(0, off + n)
    node.backend.allocations[seg.ctypes.data] = seg.nbytes
    dev = CudaIpcDeviceBuffer.from_device_pointer("dev", "job", 0, n, seg.ctypes.data + off, backend=node.backend)
    assert dev.ipc_offset == off and dev.metadata["cuda_ipc_offset"] == off
    try:
        r = node.client().fetch_shared_cpu_to_cuda_ipc(host, dev, chunk_bytes=2 * MiB, mode="pool")
        assert r.state == "complete"
        assert not seg[:off].any(), "nothing written below the buffer"
        assert np.array_equal(seg[off:], host.numpy())
    finally:
        host.release()
