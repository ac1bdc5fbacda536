"""The worker helper and a daemon as real processes on the CPU, with no GPU
visible (``python -m pcie_pool_b200.worker`` and the verification daemon, a
declared two-GPU node): the worker serves envelopes over its socket,
answers malformed input with error envelopes, records a failed lifecycle
when the data plane cannot run (no GPU here) and releases the daemon's
leases, honours ``--max-requests`` and stops on SIGTERM.  Behaviours follow
integration/test_worker_process.py and test_worker_transport.py of the
reference with independent fixtures."""

from __future__ import annotations

import os
import signal
import subprocess
import sys
import time
from dataclasses import asdict

import pytest

from pcie_pool_b200.daemon.client import TurboBusDaemonClient
from pcie_pool_b200.schema import WorkerTransferAuthorizationRequest
from pcie_pool_b200.transfer import TransferRequest
from pcie_pool_b200.worker import (WorkerServiceRequestEnvelope, WorkerServiceSocketClient,
                                   decode_worker_response_envelope)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MiB = 1 << 20


def _wait_socket(path, proc, timeout=60.0):
    end = time.monotonic() + timeout
    while time.monotonic() < end:
        if os.path.exists(path):
            return
        if proc.poll() is not None:
            raise RuntimeError(f"process exited early: {proc.stdout.read() if proc.stdout else ''}")
        time.sleep(0.05)
    raise TimeoutError(path)


def _daemon_cmd(sock):
    # the verification daemon: a declared 2-GPU node (target 0, relay 1) with a seeded profile; the
    # production CLI refuses declared topologies
    return [sys.executable, "-c", "import sys; from pcie_pool_b200.verification import _serve_daemon; "
            "_serve_daemon(sys.argv[1], 0, 1, 64, 8 << 20)", sock]


@pytest.fixture
def procs(tmp_path):
    env = {**os.environ, "PYTHONPATH": ROOT, "CUDA_VISIBLE_DEVICES": ""}
    dsock, wsock = str(tmp_path / "d.sock"), str(tmp_path / "w.sock")
    started = []

    def start(cmd, sock):
        p = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        started.append(p)
        _wait_socket(sock, p)
        return p

    yield start, dsock, wsock
    for p in started:
        if p.poll() is None:
            p.terminate()
            try:
                p.wait(10)
            except subprocess.TimeoutExpired:
                p.kill()


def test_worker_process_serves_and_cleans_up_after_a_failed_data_plane(procs):
    start, dsock, wsock = procs
    start(_daemon_cmd(dsock), dsock)
    worker = start([sys.executable, "-m", "pcie_pool_b200.worker", "--daemon-socket-path", dsock,
                    "--socket-path", wsock], wsock)
    dc = TurboBusDaemonClient(dsock, timeout=30)
    sid = dc.register_session(0, [1], max_inflight_chunks=64).payload["session"]["session_id"]
    assert dc.register_job("job", session_id=sid).ok
    from pcie_pool_b200.client import SharedPinnedCpuBuffer

    host = SharedPinnedCpuBuffer.allocate("host", "job", 8 * MiB, name_prefix="ppbproc")
    try:
        assert dc.register_buffer(**asdict(host.buffer_registration())).ok
        assert dc.register_buffer("dev", "job", "gpu", 8 * MiB, device_index=0, handle_type="cuda_ipc_device",
                                  metadata={"cuda_ipc_handle": "ab" * 64}).ok
        req = TransferRequest.from_ranges([(0, 0, 8 * MiB)], chunk_bytes=MiB, direction="h2d", mode="relay",
                                          job_id="job", metadata={"buffer_ids": ("host", "dev")})
        p = dc.plan_transfer_request(sid, req, mode="relay").payload
        tok = p["lease_tokens"][0]
        auth = WorkerTransferAuthorizationRequest(transfer_id=p["transfer_id"], lease_id=tok["lease_id"],
                                                  token=tok["token"], session_id=sid, job_id="job",
                                                  src_buffer_id="host", dst_buffer_id="dev", direction="h2d",
                                                  relay_gpu=tok["relay_gpu"])
        client = WorkerServiceSocketClient(wsock, 60.0)
        env = client.submit(WorkerServiceRequestEnvelope(payload={"authorization": asdict(auth)}))
        # no GPU in this process tree: binding the device buffer fails, the
        # lifecycle is recorded as failed and the leases are released
        assert env.ok and env.final_state in ("failed", "cleanup_failed"), env
        status = dc.transfer_status(p["transfer_id"]).payload["status"]
        assert status["state"] == "failed"
        assert dc.describe().payload["reservations"] == {}
        bad = decode_worker_response_envelope(client.send_message("{not json"))
        assert not bad.ok and bad.error
        assert worker.poll() is None, "the worker keeps serving after errors"
    finally:
        host.release()
    worker.send_signal(signal.SIGTERM)
    assert worker.wait(20) == 0


def test_worker_process_stops_after_max_requests(procs):
    start, dsock, wsock = procs
    start(_daemon_cmd(dsock), dsock)
    worker = start([sys.executable, "-m", "pcie_pool_b200.worker", "--daemon-socket-path", dsock,
                    "--socket-path", wsock, "--max-requests", "2"], wsock)
    client = WorkerServiceSocketClient(wsock, 30.0)
    for _ in range(2):
        assert not decode_worker_response_envelope(client.send_message('{"payload": 1}')).ok
    assert worker.wait(20) == 0
