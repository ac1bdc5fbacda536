"""Worker helper lifecycle, one failure stage per test: a complete transfer,
an executor that raises, a short completion, a daemon that rejects the
status report, cleanups that fail after each stage, typed errors from
``submit_report_and_cleanup``, staging-slot accounting, envelopes and the
resource binder.  The daemon is real (in-process); the data plane is the
mock lanes; failures are injected on the host by a daemon-client wrapper.
Behaviours follow integration/test_worker_helper.py of the reference with
independent fixtures."""

from __future__ import annotations

from dataclasses import asdict

import numpy as np
import pytest

from pcie_pool_b200.client import CudaIpcDeviceBuffer, SharedPinnedCpuBuffer
from pcie_pool_b200.daemon import InProcessDaemonClient, TurboBusDaemon
from pcie_pool_b200.mock import FaultPlan, MockCudaBackend, MockDataPlane, MockWorkerExecutor, MockWorld
from pcie_pool_b200.planner_types import assignment_chunks
from pcie_pool_b200.schema import DaemonResponse, WorkerTransferAuthorizationRequest
from pcie_pool_b200.topology import StaticTopologyProvider
from pcie_pool_b200.transfer import TransferRequest
from pcie_pool_b200.worker import (WorkerDataPlaneResourceBinder, WorkerDataPlaneResourceError, WorkerStagingPool,
                                   WorkerTransferClient, WorkerTransferService)
from pcie_pool_b200.worker.helper import (WorkerAuthorizationError, WorkerCleanupError, WorkerStatusReportError,
                                          WorkerTransferResult, WorkerTransferState)

MiB = 1 << 20
N = 8 * MiB


class FlakyDaemon:
    """Daemon client that fails chosen calls (``fail`` maps a method name to
    the error returned) and records every call name."""

    def __init__(self, inner) -> None:
        self.inner = inner
        self.fail: dict[str, str] = {}
        self.calls: list[str] = []

    def __getattr__(self, name):
        target = getattr(self.inner, name)
        if not callable(target):
            return target

        def call(*args, **kwargs):
            self.calls.append(name)
            if name in self.fail and (name != "transfer_status" or kwargs.get("state") or len(args) > 1):
                return DaemonResponse(ok=False, error=self.fail[name])
            return target(*args, **kwargs)

        return call


class Rig:
    def __init__(self, executor=None, faults=None) -> None:
        self.world = MockWorld(gpu_count=4)
        self.daemon = TurboBusDaemon(relay_gpus=[1, 2, 3], max_inflight_chunks_per_relay=4096,
                                     topology_provider=StaticTopologyProvider(gpu_count=4))
        self.daemon.put_profile(0, [1, 2, 3], self.world.profile(0))
        self.dc = FlakyDaemon(InProcessDaemonClient(self.daemon))
        self.backend = MockCudaBackend()
        self.pool = WorkerStagingPool()
        self.client = WorkerTransferClient(self.dc, executor=executor or MockWorkerExecutor(
            MockDataPlane(self.world, faults=faults)), staging_pool=self.pool,
            resource_binder=WorkerDataPlaneResourceBinder(self.backend))
        self.service = WorkerTransferService(transfer_client=self.client)
        self.host = SharedPinnedCpuBuffer.allocate("host", "job", N)
        self.host.numpy()[:] = np.random.default_rng(1).integers(0, 256, N, dtype=np.uint8)
        self.dev_arr = self.world.alloc(0, N)
        self.dev = CudaIpcDeviceBuffer("dev", "job", 0, N, self.backend.export_device_ipc_handle(
            self.dev_arr.ctypes.data), device_ptr=self.dev_arr.ctypes.data)

    def authorization(self, mode: str = "relay", **over) -> tuple[WorkerTransferAuthorizationRequest, dict]:
        sid = self.daemon.register_session(0, [1, 2, 3], max_inflight_chunks=4096).payload["session"]["session_id"]
        assert self.daemon.register_job("job", session_id=sid).ok
        for reg in (self.host.buffer_registration(), self.dev.buffer_registration()):
            assert self.daemon.register_buffer(**asdict(reg)).ok
        req = TransferRequest.from_ranges([(0, 0, N)], chunk_bytes=MiB, direction="h2d", mode=mode, job_id="job",
                                          metadata={"buffer_ids": ("host", "dev")})
        p = InProcessDaemonClient(self.daemon).plan_transfer_request(sid, req, mode=mode).payload
        tok = p["lease_tokens"][0]
        kw = dict(transfer_id=p["transfer_id"], lease_id=tok["lease_id"], token=tok["token"], session_id=sid,
                  job_id="job", src_buffer_id="host", dst_buffer_id="dev", direction="h2d")
        kw.update(over)
        return WorkerTransferAuthorizationRequest(**kw), p

    def status(self, tid: str) -> str:
        return self.daemon.transfer_status(tid).payload["status"]["state"]

    def close(self) -> None:
        self.host.release()


@pytest.fixture
def rig():
    r = Rig()
    yield r
    r.close()


def test_complete_lifecycle_moves_bytes_reports_and_releases(rig):
    req, p = rig.authorization()
    lc = rig.service.handle_lifecycle(req)
    assert lc.final_state == "complete" and lc.error is None
    assert lc.result.bytes_completed == N and rig.status(p["transfer_id"]) == "complete"
    relay_ranges = [c for a in p["plan"]["assignments"] if a["path"]["kind"] == "relay" for c in assignment_chunks(a)]
    for c in relay_ranges:  # every relayed range landed
        s, b = c["dst_offset"], c["bytes"]
        assert np.array_equal(rig.dev_arr[s:s + b], rig.host.numpy()[c["src_offset"]:c["src_offset"] + b])
    assert rig.daemon.describe().payload["reservations"] == {}
    assert lc.staging_release is not None and len(rig.pool) == 0
    env = lc.completion_envelope()
    assert env.ok and env.final_state == "complete" and env.transfer_id == p["transfer_id"]


def test_executor_failure_fails_the_transfer_and_cleans_leases():
    rig = Rig(faults=FaultPlan(fail_lane=1))
    try:
        req, p = rig.authorization()
        lc = rig.service.handle_lifecycle(req)
        assert lc.final_state == "failed" and "injected" in (lc.error or "")
        assert rig.status(p["transfer_id"]) == "failed"
        assert rig.daemon.describe().payload["reservations"] == {}
        assert len(rig.pool) == 0
    finally:
        rig.close()


class ShortExecutor:
    """Reports success with half the bytes."""

    def execute_bound(self, request, slot, resources):
        return WorkerTransferResult(request.transfer_id, WorkerTransferState.COMPLETE,
                                    bytes_completed=N // 2)


class RaisingExecutor:
    def execute_bound(self, request, slot, resources):
        raise RuntimeError("device lost")


def test_short_completion_is_a_failure():
    rig = Rig(executor=ShortExecutor())
    try:
        req, p = rig.authorization()
        lc = rig.service.handle_lifecycle(req)
        assert lc.final_state == "failed" and "bytes" in lc.error
        assert rig.status(p["transfer_id"]) == "failed"
    finally:
        rig.close()


def test_raising_executor_becomes_a_failed_result():
    rig = Rig(executor=RaisingExecutor())
    try:
        req, p = rig.authorization()
        lc = rig.service.handle_lifecycle(req)
        assert lc.final_state == "failed" and "device lost" in lc.error
        assert rig.daemon.describe().payload["reservations"] == {}
    finally:
        rig.close()


def test_rejected_status_report_is_status_failed_and_still_cleans(rig):
    req, p = rig.authorization()
    rig.dc.fail["transfer_status"] = "daemon busy"
    lc = rig.service.handle_lifecycle(req)
    assert lc.final_state == "status_failed" and "daemon busy" in lc.error
    assert lc.cleanup_response is not None and lc.cleanup_response.ok
    assert rig.daemon.describe().payload["reservations"] == {}
    assert len(rig.pool) == 0


def test_rejected_status_report_with_failing_cleanup_is_cleanup_failed(rig):
    req, _p = rig.authorization()
    rig.dc.fail["transfer_status"] = "daemon busy"
    rig.dc.fail["cleanup"] = "cleanup refused"
    lc = rig.service.handle_lifecycle(req)
    assert lc.final_state == "cleanup_failed" and "cleanup refused" in lc.error
    assert len(rig.pool) == 0, "the staging slot is released even then"


def test_release_failure_after_completion_is_cleanup_failed(rig):
    req, p = rig.authorization()
    rig.dc.fail["release_transfer"] = "release refused"
    lc = rig.service.handle_lifecycle(req)
    assert lc.final_state == "cleanup_failed" and "release refused" in lc.error
    assert rig.status(p["transfer_id"]) == "complete", "the data made it; only the release failed"


def test_authorization_failure_with_failing_cleanup(rig):
    req, _p = rig.authorization(token="forged")
    rig.dc.fail["cleanup"] = "cleanup refused"
    lc = rig.service.handle_lifecycle(req)
    assert lc.final_state == "cleanup_failed"


@pytest.mark.parametrize("setup,exc", [({"token": "forged"}, WorkerAuthorizationError),
                                       ("status", WorkerStatusReportError), ("cleanup", WorkerCleanupError)])
def test_submit_report_and_cleanup_raises_typed_errors(rig, setup, exc):
    if isinstance(setup, dict):
        req, _p = rig.authorization(**setup)
    else:
        req, _p = rig.authorization()
        if setup == "status":
            rig.dc.fail["transfer_status"] = "no"
        else:
            rig.dc.fail["release_transfer"] = "no"
    with pytest.raises(exc):
        rig.client.submit_report_and_cleanup(req)


def test_session_cleanup_target_kind(rig):
    req, _p = rig.authorization(token="forged")
    lc = rig.service.handle_lifecycle(req, cleanup_target_kind="session")
    assert lc.final_state == "authorization_failed"
    assert lc.cleanup_target_kind == "session" and lc.cleanup_target_id == req.session_id


def test_submit_without_report_leaves_status_to_the_caller(rig):
    req, p = rig.authorization()
    res = rig.client.submit(req)
    assert res.state is WorkerTransferState.COMPLETE and res.bytes_completed == N
    assert rig.status(p["transfer_id"]) == "submitted"
    assert "transfer_status" not in [c for c in rig.dc.calls if c == "transfer_status"]
    rig.client.status_reporter.report(res)
    assert rig.status(p["transfer_id"]) == "complete"


def test_envelope_errors_become_error_envelopes(rig):
    out = rig.service.handle_envelope_payload({"payload": {"authorization": {"transfer_id": ""}}})
    assert out["ok"] is False and out["error"]
    out = rig.service.handle_envelope_payload({"payload": "not a mapping"})
    assert out["ok"] is False


def test_resource_binder_rejects_an_ipc_handle_it_cannot_open(rig):
    req, _p = rig.authorization()
    wr = rig.client.authorize(req)
    dp = wr.data_plane
    bad_dst = type(dp.dst_handle)(**{**asdict(dp.dst_handle),
                                     "metadata": {**dp.dst_handle.metadata, "cuda_ipc_handle": "ab" * 64}})
    bad = type(dp)(**{**{f: getattr(dp, f) for f in dp.__dataclass_fields__}, "dst_handle": bad_dst})
    with pytest.raises(WorkerDataPlaneResourceError):
        with WorkerDataPlaneResourceBinder(rig.backend).bind(bad):
            pass
    with WorkerDataPlaneResourceBinder(rig.backend).bind(dp) as res:
        assert res.device_ptr == rig.dev_arr.ctypes.data and res.host_bytes == N
    assert rig.backend.open == {} and rig.backend.registered == {}, "closed and unregistered on exit"
