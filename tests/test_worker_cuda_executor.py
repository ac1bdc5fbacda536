"""The CUDA worker executor over a stand-in engine: H2D and D2H plans in
relay mode and pool mode (direct lane plus one or several relays), the lanes
and byte split it hands the engine (taken from the daemon's plan, never
re-derived), the path label and per-lane statistics of the result, and the
checks that stop a transfer before the engine runs: no plan, a plan whose
total disagrees with its chunks, unauthorized relays, staging slots and
bound resources of another request.  Behaviours follow
unit/test_worker_cuda_executor.py of the reference with independent fakes."""

from __future__ import annotations

import copy
from dataclasses import asdict
from types import SimpleNamespace

import pytest
from test_backends_and_buffers import FakeEngine
from test_worker_lifecycle import MiB, N, Rig

from pcie_pool_b200.daemon import InProcessDaemonClient
from pcie_pool_b200.parallel.engine import D2H, H2D
from pcie_pool_b200.schema import WorkerTransferAuthorizationRequest
from pcie_pool_b200.transfer import TransferRequest
from pcie_pool_b200.worker.cuda_executor import CudaWorkerExecutor, scoped_plan
from pcie_pool_b200.worker.helper import WorkerTransferState
from pcie_pool_b200.planner_types import assignment_chunks


@pytest.fixture
def rig():
    r = Rig()
    yield r
    r.close()


def ticketed(rig, mode="pool", direction="h2d", relays=(1, 2, 3)):
    """Plan a transfer on the rig's daemon and authorize it as the worker."""
    prof = rig.world.profile(0)
    prof["relays"] = [r for r in prof["relays"] if r["relay_device"] in relays]
    assert rig.daemon.put_profile(0, list(relays), prof).ok
    sid = rig.daemon.register_session(0, list(relays), max_inflight_chunks=4096).payload["session"]["session_id"]
    assert rig.daemon.register_job("job", session_id=sid).ok
    for reg in (rig.host.buffer_registration(), rig.dev.buffer_registration()):
        assert rig.daemon.register_buffer(**asdict(reg)).ok
    ids = ("host", "dev") if direction == "h2d" else ("dev", "host")
    req = TransferRequest.from_ranges([(0, 0, N)], chunk_bytes=MiB, direction=direction, mode=mode, job_id="job",
                                      metadata={"buffer_ids": ids})
    p = InProcessDaemonClient(rig.daemon).plan_transfer_request(sid, req, mode=mode).payload
    tok = p["lease_tokens"][0]
    auth = WorkerTransferAuthorizationRequest(transfer_id=p["transfer_id"], lease_id=tok["lease_id"],
                                              token=tok["token"], session_id=sid, job_id="job",
                                              src_buffer_id=ids[0], dst_buffer_id=ids[1], direction=direction)
    return rig.client.authorize(auth), p


def plan_split(p) -> dict[int, int]:
    """Bytes per lane device (the target for the direct path) in the daemon's plan."""
    out: dict[int, int] = {}
    for a in p["plan"]["assignments"]:
        dev = 0 if a["path"]["kind"] == "direct" else a["path"]["relay_device"]
        out[dev] = out.get(dev, 0) + sum(c["bytes"] for c in assignment_chunks(a))
    return out


def run(rig, wr, factory=None):
    engines = []

    def make(devs):
        engines.append(FakeEngine(devs))
        return engines[-1]

    ex = CudaWorkerExecutor(engine_factory=factory or make)
    slot = rig.pool.allocate(wr.data_plane)
    try:
        with rig.client.resource_binder.bind(wr.data_plane) as res:
            result = ex.execute_bound(wr, slot, res)
            ptrs = (res.host_ptr, res.host_bytes, res.device_ptr, res.device_bytes)
    finally:
        rig.pool.release(slot.slot_id, wr.data_plane)
    return result, engines, ptrs


@pytest.mark.parametrize("mode,direction,relays,label", [
    ("relay", "h2d", (1,), "relay_h2d"), ("pool", "h2d", (1,), "pool_h2d"), ("pool", "h2d", (1, 2, 3), "pool_h2d"),
    ("relay", "d2h", (2,), "relay_d2h"), ("pool", "d2h", (1, 2, 3), "pool_d2h"),
], ids=["h2d-relay", "h2d-pool-1", "h2d-pool-3", "d2h-relay", "d2h-pool-3"])
def test_executor_runs_the_daemon_plan_on_the_engine(rig, mode, direction, relays, label):
    wr, p = ticketed(rig, mode, direction, relays)
    result, engines, (hp, hb, dp_, db) = run(rig, wr)
    assert result.state is WorkerTransferState.COMPLETE and result.bytes_completed == N
    (eng,) = engines
    assert sorted(eng.devices) == sorted({0, *wr.relay_gpus})
    d, target, lanes, checksum = eng.runs[0]
    assert (d, target, checksum) == (H2D if direction == "h2d" else D2H, 0, True)
    got = {dev: sum(b) for dev, b in lanes}
    assert got == plan_split(p), "the engine gets the daemon's byte split, lane by lane"
    md = result.metadata
    assert md["path"] == label and md["plan_source"] == "daemon" and md["target_device"] == 0
    assert md["direct_bytes"] == plan_split(p).get(0, 0) and md["relay_bytes"] == N - md["direct_bytes"]
    assert (md["direct_chunks"] > 0) == (mode == "pool")
    assert {l["device"] for l in md["lanes"]} == set(got) and md["relay_gpus"] == list(wr.relay_gpus)
    # the worker's own mapping of the shared host buffer, and the client's device buffer through its IPC handle
    assert hp != 0 and (hb, dp_, db) == (N, rig.dev_arr.ctypes.data, N)
    assert (md["src_buffer_id"], md["dst_buffer_id"]) == (("host", "dev") if direction == "h2d" else ("dev", "host"))


def test_one_engine_per_device_set_is_reused(rig):
    wr, _ = ticketed(rig, "pool", "h2d", (1, 2, 3))
    made = []

    def factory(devs):
        made.append(tuple(devs))
        return FakeEngine(devs)

    ex = CudaWorkerExecutor(engine_factory=factory)
    assert ex.engine_for([3, 0, 1, 2]) is ex.engine_for([0, 1, 2, 3, 3])
    assert ex.engine_for([0, 1]) is not ex.engine_for([0, 1, 2])
    assert made == [(0, 1, 2, 3), (0, 1), (0, 1, 2)]


def _tampered(wr, **plan_edits):
    dp = copy.copy(wr.data_plane)
    object.__setattr__(dp, "plan", {**wr.data_plane.plan, **plan_edits})
    out = copy.copy(wr)
    object.__setattr__(out, "data_plane", dp)
    return out


def test_plan_problems_stop_the_transfer_before_the_engine(rig):
    wr, _ = ticketed(rig, "pool", "h2d", (1, 2, 3))
    made = []
    ex = CudaWorkerExecutor(engine_factory=lambda d: made.append(d) or FakeEngine(d))
    slot = rig.pool.allocate(wr.data_plane)
    for bad, msg in ((_tampered(wr, total_bytes=N + 1), "total bytes"),
                     (_tampered(wr, assignments=[]), "no authorized relay chunks")):
        with rig.client.resource_binder.bind(bad.data_plane) as res:
            r = ex.execute_bound(bad, slot, res)
        assert r.state is WorkerTransferState.FAILED and msg in r.error
    assert made == [], "no engine was built for a rejected plan"
    with rig.client.resource_binder.bind(wr.data_plane) as res:
        r = ex.execute_bound(_tampered(wr), slot, res)  # same plan, but a different request object: fine
        assert r.state is WorkerTransferState.COMPLETE
        other = _tampered(wr, chunk_bytes=2 * MiB)
        r = ex.execute_bound(other, slot, res)
    assert r.state is WorkerTransferState.FAILED and "bound resources do not match" in r.error


def test_scoped_plan_checks():
    def req(plan, relays=(1,), ranges=(), direction="h2d"):
        dp = SimpleNamespace(plan=plan, direction=direction, ranges=tuple(ranges),
                             staging=SimpleNamespace(max_chunk_bytes=MiB))
        return SimpleNamespace(data_plane=dp, relay_gpus=tuple(relays))

    def path(kind, relay=-1, **kw):
        return {"kind": kind, "direction": "h2d", "target_device": 0, "relay_device": relay, **kw}

    c = {"src_offset": 0, "dst_offset": 0, "bytes": MiB}
    with pytest.raises(ValueError, match="daemon-issued transfer plan"):
        scoped_plan(req({}), 0)
    with pytest.raises(ValueError, match="not authorized"):
        scoped_plan(req({"assignments": [{"path": path("relay", 2), "chunks": [c]}]}, ranges=[c]), 0)
    with pytest.raises(ValueError, match="disabled"):
        scoped_plan(req({"assignments": [{"path": path("relay", 1, enabled=False), "chunks": [c]}]}), 0)
    with pytest.raises(ValueError, match="direction"):
        scoped_plan(req({"assignments": [{"path": path("relay", 1), "chunks": [c]}]}, direction="d2h"), 0)
    with pytest.raises(ValueError, match="authorized ranges"):
        scoped_plan(req({"assignments": [{"path": path("relay", 1), "chunks": [c]}]}, ranges=[]), 0)
    with pytest.raises(ValueError, match="mapping"):
        scoped_plan(req({"assignments": ["relay"]}), 0)
    ok = scoped_plan(req({"assignments": [{"path": path("direct", 5), "chunks": [c]},
                                          {"path": path("relay", 1), "chunks": [c]},
                                          {"path": path("relay", 1), "chunks": []}]}, ranges=[c]), 0)
    assert [a["path"]["relay_device"] for a in ok["assignments"]] == [-1, 1], "empty paths are dropped"
    assert ok["total_bytes"] == 2 * MiB and ok["chunk_bytes"] == MiB


def test_slot_and_request_must_belong_together(rig):
    wr, _ = ticketed(rig, "pool", "h2d", (1, 2, 3))
    ex = CudaWorkerExecutor(engine_factory=FakeEngine)
    slot = rig.pool.allocate(wr.data_plane)
    for field, value, msg in (("transfer_id", "someone-else", "transfer"), ("lease_id", "other-lease", "lease"),
                              ("relay_gpu", 7, "relay")):
        wrong = copy.copy(slot)
        object.__setattr__(wrong, field, value)
        with pytest.raises(ValueError, match=f"staging slot {msg} does not match"):
            ex.execute(wr, wrong)
    with pytest.raises(TypeError):
        ex.execute(wr, object())
    with pytest.raises(TypeError):
        ex.execute_bound(wr, slot, object())
    r = ex.execute(wr, slot)
    assert r.state is WorkerTransferState.FAILED and "bound data-plane resources" in r.error
    assert r.metadata["staging_slot_id"] == slot.slot_id
