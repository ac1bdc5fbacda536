"""Lending a busy GPU to a more contended uplink group (opt-in).

By default a GPU whose link is moving its own data (or was a target within
the link-hold window) is never planned as a relay.  Given per-GPU rates
measured with every link busy (``set_uplink_rates``), the daemon may still
lend such a GPU to a target whose measured rate is lower by the lend ratio:
on the 8-GPU nodes of this pool GPUs 0-3 get ~18 GiB/s and GPUs 4-7 ~30
GiB/s when all links are busy, so a tenant on GPU0 may borrow GPU4's link
while GPU4 moves its own shard, and never the other way round.  CPU only:
the engine is a stand-in that holds each transfer until the test releases
it."""

import threading
import time

import numpy as np

from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
from pcie_pool_b200.daemon import InProcessDaemonClient, IntentExecutor, EngineDataPlane, TurboBusDaemon
from pcie_pool_b200.parallel.engine import LaneResult, TransferResult
from pcie_pool_b200.topology import StaticTopologyProvider, synthetic_inventory

MiB = 1 << 20
N = 64 * MiB


class GatedEngine:
    def __init__(self):
        self.started: list[tuple[int, int, list[int]]] = []
        self._gates: dict[int, threading.Event] = {}
        self._lock = threading.Lock()

    def gate(self, k):
        with self._lock:
            return self._gates.setdefault(k, threading.Event())

    def run(self, direction, target, host_ptr, host_bytes, dev_ptr, dev_bytes, lanes, checksum=False, **kw):
        with self._lock:
            k = len(self.started)
            self.started.append((k, int(target), sorted(l.device for l in lanes)))
        assert self.gate(k).wait(20), "test never released the transfer"
        stats = [LaneResult(l.device, l.device == target, int(l.bytes.sum()), int(l.bytes.size), 1.0) for l in lanes]
        n = sum(s.chunks for s in stats)
        return TransferResult(id=k, ok=True, status_code=0, error="", bytes=sum(s.bytes for s in stats), cuda_ms=1.0,
                              submit_to_complete_ms=1.0, gib_per_s=1.0, lanes=stats,
                              checksums=np.zeros((n, 2), dtype=np.uint64))


def _profile(target, relays):
    return {"target_device": target, "direct_h2d_bw_gbps": 50.0, "direct_d2h_bw_gbps": 50.0,
            "relays": [{"relay_device": r, "target_device": target, "h2d_bw_gbps": 50.0, "d2h_bw_gbps": 50.0,
                        "p2p_bw_gbps": 700.0, "effective_bw_gbps": 50.0, "effective_d2h_bw_gbps": 50.0,
                        "p2p_enabled": True} for r in relays]}


def _node(rates=None):
    eng = GatedEngine()
    daemon = TurboBusDaemon([0, 1], max_sessions_per_relay=2, max_inflight_chunks_per_relay=1 << 16,
                            topology_provider=StaticTopologyProvider(synthetic_inventory(2)),
                            executor=IntentExecutor(EngineDataPlane(engine=eng, checksum=True), max_workers=4),
                            uplink_rates=rates)
    dc = InProcessDaemonClient(daemon)
    sessions = {}
    for g in (0, 1):
        other = [1 - g]
        daemon.put_profile(g, other, _profile(g, other))
        sid = dc.register_session(g, other, max_inflight_chunks=1 << 16).payload["session"]["session_id"]
        assert dc.register_job(f"job{g}", session_id=sid).ok
        assert dc.register_buffer(f"h{g}", f"job{g}", "cpu_pinned", N, address=4096 + g * N, pinned=True).ok
        assert dc.register_buffer(f"d{g}", f"job{g}", "gpu", N, device_index=g, address=(1 << 30) + g * N).ok
        sessions[g] = sid
    return eng, daemon, TurboBusClient(daemon=dc), sessions


def _intent(g, i, sid):
    return TransferIntent(f"t{g}-{i}", f"job{g}", sid, f"h{g}", f"d{g}", "h2d", N,
                          ({"src_offset": 0, "dst_offset": 0, "bytes": N},), workload_kind="training_state",
                          metadata={"chunk_bytes": 4 * MiB})


def _wait_started(eng, n):
    end = time.monotonic() + 10
    while len(eng.started) < n:
        assert time.monotonic() < end
        time.sleep(0.005)


def _run(rates):
    eng, daemon, client, sess = _node(rates)
    client.submit_transfer_intent(_intent(1, 0, sess[1]))  # GPU1 moves its own shard (direct lane busy)
    _wait_started(eng, 1)
    client.submit_transfer_intent(_intent(0, 0, sess[0]))  # GPU0's tenant plans while GPU1 is busy
    _wait_started(eng, 2)
    client.submit_transfer_intent(_intent(1, 1, sess[1]))  # and GPU1's tenant while GPU0 is busy
    time.sleep(0.2)
    for k in range(3):
        eng.gate(k).set()
    for g, i in ((1, 0), (0, 0), (1, 1)):
        assert client.wait(f"t{g}-{i}", timeout_seconds=20).state is TransferStatusState.COMPLETE
    d = daemon.describe().payload
    assert all(int(q.get("active_chunks", 0)) == 0 for q in (d.get("relay_quotas") or {}).values())
    return eng.started


def test_without_rates_a_busy_gpu_is_never_lent():
    started = _run(None)
    assert [lanes for _k, t, lanes in started if t == 0] == [[0]]
    assert [lanes for _k, t, lanes in started if t == 1][-1] == [1]


def test_a_busy_gpu_is_lent_only_to_a_more_contended_group():
    started = _run({0: 18.0, 1: 30.0})
    into0 = [lanes for _k, t, lanes in started if t == 0]
    into1 = [lanes for _k, t, lanes in started if t == 1]
    assert into0 == [[0, 1]]   # GPU1 (faster group) relays for GPU0 while busy with its own shard
    assert into1[-1] == [1]    # GPU0 (slower group), busy, does not relay for GPU1


def test_rates_can_be_set_and_cleared():
    d = TurboBusDaemon([0, 1], topology_provider=StaticTopologyProvider(synthetic_inventory(2)))
    d.set_uplink_rates({0: 18.0, 1: 30.0, 2: 0.0})
    assert d._lendable(0) == frozenset({1}) and d._lendable(1) == frozenset()
    d.set_uplink_rates(None)
    assert d._lendable(0) == frozenset()
