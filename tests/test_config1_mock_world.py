"""BASELINE config 1 on the CPU: daemon + planner + client on a mock world
of 4 simulated GPUs (1 direct + 3 relay lanes), seed 0.  A 256 MiB fp32
N(0,1) tensor goes host -> "GPU0" in 4 MiB chunks and back; the round trip
is byte-exact and the trace assigns every chunk to exactly one lane, the lane
the plan chose."""

import numpy as np
import pytest

from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
from pcie_pool_b200.daemon import InProcessDaemonClient, IntentExecutor, TurboBusDaemon
from pcie_pool_b200.mock import MockDataPlane, MockWorld, chunk_lane_map
from pcie_pool_b200.topology import StaticTopologyProvider
from pcie_pool_b200.planner_types import assignment_chunks

MiB = 1 << 20


def make_node(gpu_count=4, checksum=True):
    world = MockWorld(gpu_count=gpu_count)
    plane = MockDataPlane(world, checksum=checksum)
    daemon = TurboBusDaemon(relay_gpus=range(1, gpu_count), max_inflight_chunks_per_relay=1024,
                            topology_provider=StaticTopologyProvider(gpu_count=gpu_count),
                            executor=IntentExecutor(plane))
    daemon.put_profile(0, list(range(1, gpu_count)), world.profile(0))
    return world, plane, daemon


def register(dc, job, session, name, arr, kind, device=None):
    r = dc.register_buffer(name, job, kind, arr.nbytes, device_index=device, address=arr.ctypes.data,
                           pinned=kind == "cpu_pinned")
    assert r.ok, r.error


@pytest.fixture
def node():
    return make_node()


def test_config1_roundtrip_256mib_fp32(node):
    world, plane, daemon = node
    dc = InProcessDaemonClient(daemon)
    s = dc.register_session(0, [1, 2, 3], max_inflight_chunks=4096)
    assert s.ok, s.error
    sid = s.payload["session"]["session_id"]
    assert dc.register_job("job-a", session_id=sid).ok
    host = np.random.default_rng(0).standard_normal(64 * MiB, dtype=np.float32)  # 256 MiB
    back = np.zeros_like(host)
    gpu0 = world.alloc(0, host.nbytes)
    register(dc, "job-a", sid, "host", host, "cpu_pinned")
    register(dc, "job-a", sid, "back", back, "cpu_pinned")
    register(dc, "job-a", sid, "gpu0", gpu0, "gpu", device=0)
    client = TurboBusClient(daemon=dc)
    n = host.nbytes
    up = TransferIntent("up-1", "job-a", sid, "host", "gpu0", "h2d", n,
                        ({"src_offset": 0, "dst_offset": 0, "bytes": n},), metadata={"chunk_bytes": 4 * MiB})
    r1 = client.transfer(up, timeout_seconds=120)
    assert r1.state is TransferStatusState.COMPLETE, r1.error
    assert r1.bytes_completed == n and r1.completed_at is not None
    assert np.array_equal(gpu0.view(np.float32), host)
    down = TransferIntent("down-1", "job-a", sid, "gpu0", "back", "d2h", n,
                          ({"src_offset": 0, "dst_offset": 0, "bytes": n},), metadata={"chunk_bytes": 4 * MiB})
    r2 = client.transfer(down, timeout_seconds=120)
    assert r2.state is TransferStatusState.COMPLETE, r2.error
    assert back.tobytes() == host.tobytes()
    # every chunk moved exactly once, on the lane its plan assigned
    desc = daemon.describe().payload
    for tid_key, rec in (("up", r1), ("down", r2)):
        tid = rec.metadata["transfer_id"]
        trace = [t for t in plane.trace if t["transfer_id"] == tid]
        lanes = chunk_lane_map(trace)
        assert len(lanes) == n // (4 * MiB)
        decision = desc["transfer_queue"]
        plan = next(q for q in decision if q["transfer_id"] == tid)
        assert plan["state"] == "complete"
    used = {t["lane"] for t in plane.trace}
    assert used == {0, 1, 2, 3}, "all four lanes carried chunks"
    # leases were released once the transfers completed
    assert desc["reservations"] == {}
    assert all(q["active_chunks"] == 0 for q in desc["relay_quotas"].values())


def test_plan_assigns_each_chunk_to_exactly_one_lane(node):
    world, plane, daemon = node
    dc = InProcessDaemonClient(daemon)
    sid = dc.register_session(0, [1, 2, 3], max_inflight_chunks=4096).payload["session"]["session_id"]
    resp = dc.plan_transfer(sid, 256 * MiB, 4 * MiB)
    assert resp.ok, resp.error
    plan = resp.payload["plan"]
    offs = [c["src_offset"] for a in plan["assignments"] for c in assignment_chunks(a)]
    assert sorted(offs) == list(range(0, 256 * MiB, 4 * MiB))
    assert len({a["path"]["relay_device"] for a in plan["assignments"]}) == 4


def test_corrupted_chunk_fails_the_transfer():
    from pcie_pool_b200.mock import FaultPlan

    world, plane, daemon = make_node()
    plane.faults = FaultPlan(corrupt_lane=2)
    dc = InProcessDaemonClient(daemon)
    sid = dc.register_session(0, [1, 2, 3], max_inflight_chunks=4096).payload["session"]["session_id"]
    dc.register_job("j", session_id=sid)
    host = np.arange(8 * MiB, dtype=np.uint8)
    gpu0 = world.alloc(0, host.nbytes)
    register(dc, "j", sid, "h", host, "cpu_pinned")
    register(dc, "j", sid, "g", gpu0, "gpu", device=0)
    it = TransferIntent("bad", "j", sid, "h", "g", "h2d", host.nbytes,
                        ({"src_offset": 0, "dst_offset": 0, "bytes": host.nbytes},), metadata={"chunk_bytes": MiB})
    r = TurboBusClient(daemon=dc).transfer(it, timeout_seconds=60)
    assert r.state is TransferStatusState.FAILED
    assert "checksum mismatch" in r.error
    assert daemon.describe().payload["reservations"] == {}
