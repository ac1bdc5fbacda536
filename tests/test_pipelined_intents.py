"""A session's next intent queues behind its own running transfer.

The daemon admits an intent whose relays are busy only with the same
session's transfer to the same target in the same direction (the data plane
runs them in submit order on those lanes), so a client that submits ahead
keeps the PCIe links busy between intents.  Another tenant's intent on those
relays is still delayed until the links are free.  CPU only: the engine is a
stand-in that holds each transfer until the test releases it."""

import threading
import time

import numpy as np

from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
from pcie_pool_b200.daemon import InProcessDaemonClient
from pcie_pool_b200.e2e import build_inprocess_node
from pcie_pool_b200.parallel.engine import LaneResult, TransferResult

MiB = 1 << 20
N = 64 * MiB


class GatedEngine:
    """Completes transfer k only after ``release(k)``; records submit order."""

    def __init__(self):
        self.started: list[tuple[int, list[int]]] = []
        self._gates: dict[int, threading.Event] = {}
        self._lock = threading.Lock()

    def gate(self, k: int) -> threading.Event:
        with self._lock:
            return self._gates.setdefault(k, threading.Event())

    def run(self, direction, target, host_ptr, host_bytes, dev_ptr, dev_bytes, lanes, checksum=False, **kw):
        with self._lock:
            k = len(self.started)
            self.started.append((k, [l.device for l in lanes]))
        assert self.gate(k).wait(20), "test never released the transfer"
        stats = [LaneResult(l.device, l.device == target, int(l.bytes.sum()), int(l.bytes.size), 1.0) for l in lanes]
        n = sum(s.chunks for s in stats)
        return TransferResult(id=k, ok=True, status_code=0, error="", bytes=sum(s.bytes for s in stats), cuda_ms=1.0,
                              submit_to_complete_ms=1.0, gib_per_s=1.0, lanes=stats,
                              checksums=np.zeros((n, 2), dtype=np.uint64))


PROFILE = {"target_device": 0, "direct_h2d_bw_gbps": 50.0, "direct_d2h_bw_gbps": 50.0,
           "relays": [{"relay_device": r, "target_device": 0, "h2d_bw_gbps": 50.0, "d2h_bw_gbps": 50.0,
                       "p2p_bw_gbps": 700.0, "effective_bw_gbps": 50.0, "effective_d2h_bw_gbps": 50.0,
                       "p2p_enabled": True} for r in (1, 2, 3)]}


def _node():
    eng = GatedEngine()
    daemon, dc = build_inprocess_node(eng, [0, 1, 2, 3], 0, PROFILE, workers=4)
    return eng, daemon, dc


def _session(dc, job, relays=(1, 2, 3)):
    sid = dc.register_session(0, list(relays), max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job(job, session_id=sid).ok
    assert dc.register_buffer(f"{job}-h", job, "cpu_pinned", N, address=4096, pinned=True).ok
    assert dc.register_buffer(f"{job}-g", job, "gpu", N, device_index=0, address=1 << 30).ok
    return sid


def _intent(i, job, sid):
    return TransferIntent(f"{job}-{i}", job, sid, f"{job}-h", f"{job}-g", "h2d", N,
                          ({"src_offset": 0, "dst_offset": 0, "bytes": N},), workload_kind="model_weights",
                          metadata={"chunk_bytes": 4 * MiB})


def _wait_started(eng, n, timeout=10.0):
    end = time.monotonic() + timeout
    while len(eng.started) < n:
        assert time.monotonic() < end, f"only {len(eng.started)} transfers reached the engine"
        time.sleep(0.005)


def test_same_session_intent_queues_behind_its_running_transfer():
    eng, daemon, dc = _node()
    sid = _session(dc, "job")
    client = TurboBusClient(daemon=dc)
    r0 = client.submit_transfer_intent(_intent(0, "job", sid))
    _wait_started(eng, 1)
    r1 = client.submit_transfer_intent(_intent(1, "job", sid))
    # admitted at once with its relay lanes and handed to the engine while #0 still runs
    _wait_started(eng, 2)
    assert sorted(eng.started[0][1]) == sorted(eng.started[1][1]) == [0, 1, 2, 3]
    assert r0.state is not TransferStatusState.FAILED and r1.state is not TransferStatusState.FAILED
    eng.gate(0).set()
    eng.gate(1).set()
    assert client.wait("job-0", timeout_seconds=20).state is TransferStatusState.COMPLETE
    assert client.wait("job-1", timeout_seconds=20).state is TransferStatusState.COMPLETE
    d = InProcessDaemonClient(daemon).describe().payload
    assert all(int(q.get("active_chunks", 0)) == 0 for q in (d.get("relay_quotas") or {}).values())


def test_other_session_on_busy_relays_is_still_delayed():
    eng, daemon, dc = _node()
    for q in daemon._quotas.values():  # two tenants may hold the same relays
        q.max_sessions = 2
    s1 = _session(dc, "a")
    s2 = _session(dc, "b")
    client = TurboBusClient(daemon=dc)
    client.submit_transfer_intent(_intent(0, "a", s1))
    _wait_started(eng, 1)
    client.submit_transfer_intent(_intent(0, "b", s2))
    time.sleep(0.2)
    # b's intent does not run on a's busy relays; it waits (or runs direct-only)
    assert len(eng.started) == 1 or eng.started[1][1] == [0]
    eng.gate(0).set()
    eng.gate(1).set()
    assert client.wait("a-0", timeout_seconds=20).state is TransferStatusState.COMPLETE
    assert client.wait("b-0", timeout_seconds=20).state is TransferStatusState.COMPLETE
