"""Many concurrent clients against one daemon over its AF_UNIX socket
(CPU, mock data plane): sessions, jobs, buffers, executed intents, failures
and cleanups interleave; afterwards nothing may leak."""

import os
import random
import tempfile
import threading

import numpy as np

from pcie_pool_b200 import TransferIntent, TurboBusClient
from pcie_pool_b200.daemon import IntentExecutor, TurboBusDaemon
from pcie_pool_b200.daemon.client import TurboBusDaemonClient
from pcie_pool_b200.daemon.wire import serve_unix
from pcie_pool_b200.mock import FaultPlan, MockDataPlane, MockWorld
from pcie_pool_b200.topology import StaticTopologyProvider

KiB = 1 << 10


def test_concurrent_clients_leave_no_leases_behind():
    world = MockWorld(gpu_count=4)
    plane = MockDataPlane(world, faults=FaultPlan())
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_sessions_per_relay=64, max_inflight_chunks_per_relay=1 << 16,
                       topology_provider=StaticTopologyProvider(gpu_count=4),
                       executor=IntentExecutor(plane, max_workers=8))
    d.put_profile(0, [1, 2, 3], world.profile(0))
    sock = os.path.join(tempfile.mkdtemp(prefix="ppb-stress-"), "d.sock")
    stop, ready = threading.Event(), threading.Event()
    srv = threading.Thread(target=serve_unix, args=(d, sock), kwargs={"stop_event": stop, "ready_event": ready},
                           daemon=True)
    srv.start()
    assert ready.wait(5)
    errors, done = [], []
    n = 512 * KiB

    def worker(w):
        rng = random.Random(w)
        c = TurboBusDaemonClient(sock)
        client = TurboBusClient(daemon=c)
        try:
            for it in range(8):
                s = c.register_session(0, [1, 2, 3], max_inflight_chunks=1024)
                assert s.ok, s.error
                sid = s.payload["session"]["session_id"]
                job = f"job-{w}-{it}"
                assert c.register_job(job, session_id=sid).ok
                host = np.full(n, w & 0xFF, dtype=np.uint8)
                dev = world.alloc(0, n)
                assert c.register_buffer(f"h-{job}", job, "cpu_pinned", n, address=host.ctypes.data, pinned=True).ok
                assert c.register_buffer(f"g-{job}", job, "gpu", n, device_index=0, address=dev.ctypes.data).ok
                intent = TransferIntent(f"i-{job}", job, sid, f"h-{job}", f"g-{job}", "h2d", n,
                                        ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                                        metadata={"chunk_bytes": 64 * KiB})
                action = rng.random()
                if action < 0.7:
                    r = client.transfer(intent, timeout_seconds=60)
                    assert r.state.value == "complete", r.error
                    assert np.array_equal(dev, host)
                    done.append(job)
                    assert c.close_session(sid).ok
                elif action < 0.85:
                    client.submit_transfer_intent(intent)  # then clean the job up mid-flight
                    assert c.cleanup(target_kind="job", target_id=job, reason="stress", force=True).ok
                    assert c.close_session(sid).ok
                else:
                    assert c.close_session(sid).ok  # abandon: closing the session releases its state
        except Exception as exc:  # noqa: BLE001 - collected and asserted below
            errors.append(f"{w}: {type(exc).__name__}: {exc}")

    ths = [threading.Thread(target=worker, args=(w,)) for w in range(12)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(120)
    d._executor.shutdown(wait=True) if hasattr(d, "_executor") and d._executor else None
    stop.set()
    srv.join(5)
    assert not errors, errors[:3]
    assert len(done) > 20
    desc = d.describe().payload
    live = [q for q in desc["transfer_queue"] if q["state"] not in ("complete", "failed", "canceled")]
    assert not live, live[:2]
    assert desc["reservations"] == {}
    assert all(q["active_chunks"] == 0 for q in desc["relay_quotas"].values())
