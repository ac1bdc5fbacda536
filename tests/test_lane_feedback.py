"""The daemon's split follows the lane rates its data plane measures.

A probed profile holds plain-copy rates; a fused landing op loads the lanes
differently (the target GPU lands its own lane and every relay's chunks), so
the daemon folds each completed transfer's per-lane rates, per landing op,
into the concurrent rates the planner splits by.  CPU only: the engine is a
stand-in whose lanes run at fixed rates, with the direct lane at half the
rate the profile claims."""

import numpy as np

from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
from pcie_pool_b200.e2e import build_inprocess_node
from pcie_pool_b200.parallel.engine import LaneResult, TransferResult

MiB = 1 << 20
N = 256 * MiB
RATES = {0: 25.0, 1: 50.0}  # GiB/s the stand-in's lanes actually deliver

PROFILE = {"target_device": 0, "direct_h2d_bw_gbps": 50.0, "direct_d2h_bw_gbps": 50.0,
           "relays": [{"relay_device": 1, "target_device": 0, "h2d_bw_gbps": 50.0, "d2h_bw_gbps": 50.0,
                       "p2p_bw_gbps": 700.0, "effective_bw_gbps": 50.0, "effective_d2h_bw_gbps": 50.0,
                       "p2p_enabled": True}],
           "concurrent": {"h2d": {"lanes": [0, 1], "lane_gibps": {"0": 50.0, "1": 50.0}}}}


class RatedEngine:
    """Each lane takes bytes / its fixed rate; records each transfer's split."""

    def __init__(self):
        self.splits: list[dict[int, int]] = []

    def run(self, direction, target, host_ptr, host_bytes, dev_ptr, dev_bytes, lanes, checksum=False, **kw):
        stats = []
        for l in lanes:
            b = int(l.bytes.sum())
            stats.append(LaneResult(l.device, l.device == target, b, int(l.bytes.size),
                                    b / (RATES[l.device] * (1 << 30)) * 1e3))
        self.splits.append({s.device: s.bytes for s in stats})
        n = sum(s.chunks for s in stats)
        ms = max(s.cuda_ms for s in stats)
        return TransferResult(id=len(self.splits), ok=True, status_code=0, error="", bytes=sum(s.bytes for s in stats),
                              cuda_ms=ms, submit_to_complete_ms=ms, gib_per_s=1.0, lanes=stats,
                              checksums=np.zeros((n, 2), dtype=np.uint64))


def _run(k, lane_feedback=True):
    eng = RatedEngine()
    daemon, dc = build_inprocess_node(eng, [0, 1], 0, PROFILE, workers=1)
    daemon._feedback = daemon._feedback if lane_feedback else None
    sid = dc.register_session(0, [1], max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job("job", session_id=sid).ok
    assert dc.register_buffer("h", "job", "cpu_pinned", N, address=4096, pinned=True).ok
    assert dc.register_buffer("g", "job", "gpu", N, device_index=0, address=1 << 30).ok
    client = TurboBusClient(daemon=dc)
    for i in range(k):
        intent = TransferIntent(f"t{i}", "job", sid, "h", "g", "h2d", N,
                                ({"src_offset": 0, "dst_offset": 0, "bytes": N},),
                                workload_kind="model_weights", metadata={"chunk_bytes": 4 * MiB})
        client.submit_transfer_intent(intent)
        assert client.wait(f"t{i}", timeout_seconds=20).state is TransferStatusState.COMPLETE
    return eng.splits


def test_split_converges_to_measured_lane_rates():
    splits = _run(4)
    # first transfer: the profile's even rates
    assert abs(splits[0][0] - splits[0][1]) <= 4 * MiB
    # then the direct lane (measured at half the relay's rate) gets about a third
    last = splits[-1]
    assert abs(last[0] / N - 1 / 3) < 0.03, last


def test_without_feedback_the_split_stays_on_the_profile():
    splits = _run(3, lane_feedback=False)
    assert all(abs(s[0] - s[1]) <= 4 * MiB for s in splits)


def test_feedback_is_kept_per_landing_op():
    from pcie_pool_b200.daemon.server import TurboBusDaemon

    d = TurboBusDaemon(relay_gpus=[1])
    d._observe_lanes({"landing_op": "scatter_units", "path_stats": [
        {"direction": "h2d", "target_device": 0, "relay_device": -1, "cuda_ms": 10.0, "gib_per_second": 10.0},
        {"direction": "h2d", "target_device": 0, "relay_device": 1, "cuda_ms": 10.0, "gib_per_second": 40.0}]})
    assert d._feedback.rates(0, "h2d:scatter_units") == {0: 10.0, 1: 40.0}
    assert d._feedback.rates(0, "h2d:copy") == {}
    # a failed-over transfer's rates are not folded in
    d._observe_lanes({"landing_op": "copy", "failover": {"failed_lane_device": 1}, "path_stats": [
        {"direction": "h2d", "target_device": 0, "relay_device": -1, "cuda_ms": 10.0, "gib_per_second": 10.0}]})
    assert d._feedback.rates(0, "h2d:copy") == {}


def test_plan_cache_reuses_plans_only_for_the_same_shape_and_profile():
    from pcie_pool_b200.e2e import nominal_profile
    from pcie_pool_b200.schema import RelayQuota, Session
    from pcie_pool_b200.scheduler import DaemonScheduler

    sch = DaemonScheduler()
    sess = Session(session_id="s", target_gpu=0, relay_gpus=[1, 2, 3], max_inflight_chunks=1 << 16)
    quotas = {g: RelayQuota(relay_gpu=g, max_sessions=4, max_inflight_chunks=1 << 16) for g in (1, 2, 3)}

    def plan(total=N, profile=None, ranges=None, direction="h2d"):
        prof = profile or {"profile": nominal_profile(0, [1, 2, 3])}
        before = sch.plan_cache_hits
        d = sch.plan_transfer(session=sess, profile_entry=prof, relay_quotas=quotas, total_bytes=total,
                              chunk_bytes=4 * MiB, ranges=ranges, direction=direction)
        return d.plan, sch.plan_cache_hits - before

    a, miss = plan()
    b, hit = plan()
    assert (miss, hit) == (0, 1) and a == b  # same shape, same profile: the issued plan is reused
    assert len({x["path"]["relay_device"] for x in a["assignments"]}) == 4  # direct + 3 relays
    assert plan(total=N // 2)[1] == 0
    assert plan(direction="d2h")[1] == 0
    assert plan(ranges=({"src_offset": 4096, "dst_offset": 0, "bytes": N},))[1] == 0
    assert plan(profile={"profile": nominal_profile(0, [1, 2, 3], lane_gibps=20.0)})[1] == 0
    # the reused plan is what a fresh planner gives
    fresh = DaemonScheduler().plan_transfer(session=sess, profile_entry={"profile": nominal_profile(0, [1, 2, 3])},
                                            relay_quotas=quotas, total_bytes=N, chunk_bytes=4 * MiB)
    assert fresh.plan == a
