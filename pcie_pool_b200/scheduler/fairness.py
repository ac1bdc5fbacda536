"""Multi-tenant fair-share model used by the scheduler.

A request is charged ``bytes x workload multiplier`` (kv_cache 0.75,
training/optimizer state 1.25, otherwise 1.0), discounted for positive
priority by ``1 + 0.1 * min(priority, 9)``.  A job may use relay lanes only
while its projected weighted active bytes stay within 1.25x the weighted
average over all jobs; otherwise the plan degrades to the direct lane.  These
constants are the reference's (turbobus/scheduler/daemon.py:599-651) so that
mixed fleets arbitrate identically.
"""

from __future__ import annotations

from dataclasses import dataclass
from collections.abc import Mapping

from ..schema import WorkloadKind

WORKLOAD_CHARGE = {
    WorkloadKind.KV_CACHE.value: 0.75,
    WorkloadKind.TRAINING_STATE.value: 1.25,
    WorkloadKind.OPTIMIZER_STATE.value: 1.25,
}
FAIRNESS_SLACK = 1.25
PRIORITY_STEP = 0.1
PRIORITY_CAP = 9
FAIRNESS_FALLBACK = "weighted fairness limit prefers direct fallback"


def charge_bytes(total_bytes: int, workload_kind: str, priority: int) -> float:
    charge = float(total_bytes) * WORKLOAD_CHARGE.get(WorkloadKind(workload_kind).value, 1.0)
    if int(priority) > 0:
        charge /= 1.0 + min(int(priority), PRIORITY_CAP) * PRIORITY_STEP
    return charge


@dataclass(frozen=True)
class LoadView:
    """What the scheduler knows about everyone else when it plans a request."""

    job_id: str | None
    workload_kind: str
    priority: int
    busy_relays: frozenset[int]
    job_weight: float
    total_weight: float
    current_job_active_bytes: int
    total_active_bytes: int
    request_charge_bytes: float
    average_weighted_active_bytes: float
    current_weighted_active_bytes: float
    projected_weighted_active_bytes: float
    fairness_threshold_bytes: float
    active_transfer_count: int
    queued_transfer_count: int
    # GPUs that were a transfer's target within the daemon's link-hold window:
    # never planned as relays (a planning preference, unlike busy_relays,
    # which delayed admission waits out)
    held_relays: frozenset[int] = frozenset()

    def policy_metadata(self) -> dict[str, object]:
        return {
            "job_id": self.job_id, "job_weight": self.job_weight, "total_weight": self.total_weight,
            "workload_kind": self.workload_kind, "priority": self.priority,
            "request_charge_bytes": self.request_charge_bytes,
            "current_job_active_bytes": self.current_job_active_bytes,
            "total_active_bytes": self.total_active_bytes,
            "current_weighted_active_bytes": self.current_weighted_active_bytes,
            "projected_weighted_active_bytes": self.projected_weighted_active_bytes,
            "average_weighted_active_bytes": self.average_weighted_active_bytes,
            "fairness_threshold_bytes": self.fairness_threshold_bytes,
            "busy_relays": tuple(sorted(self.busy_relays)),
            "held_relays": tuple(sorted(self.held_relays)),
            "active_transfer_count": self.active_transfer_count,
            "queued_transfer_count": self.queued_transfer_count,
        }

    def relay_over_share(self) -> bool:
        """True when relays would push this job past its fair share."""
        return (self.total_active_bytes > 0
                and self.projected_weighted_active_bytes > self.fairness_threshold_bytes)


def load_view(runtime_state: Mapping[str, object] | None, *, job_id: str | None, total_bytes: int,
              workload_kind: str, priority: int) -> LoadView:
    job = None if job_id is None else str(job_id)
    workload = WorkloadKind(workload_kind).value
    busy: set[int] = set()
    jobs: Mapping[str, object] = {}
    active = queued = 0
    held: frozenset[int] = frozenset()
    if isinstance(runtime_state, Mapping):
        # GPUs that were a transfer's target within the daemon's link-hold
        # window keep their link for their own traffic.
        held = frozenset(int(g) for g in runtime_state.get("recent_targets", ()) or ())
        for rec in runtime_state.get("active_paths", ()) or ():
            if not isinstance(rec, Mapping):
                continue
            kind = str(rec.get("kind", "")).lower()
            if kind == "relay" and rec.get("relay_device") is not None:
                busy.add(int(rec["relay_device"]))
            elif kind == "direct" and rec.get("target_device") is not None:
                # A GPU whose own PCIe link is moving its own data has no link
                # bandwidth to lend: relaying through it would only split the
                # link between two transfers.
                busy.add(int(rec["target_device"]))
        # GPUs the daemon lends across contention groups despite their own
        # traffic (its ``set_uplink_rates``)
        lend = frozenset(int(g) for g in runtime_state.get("lendable_relays", ()) or ())
        held -= lend
        busy -= lend
        summary = runtime_state.get("summary", {})
        if isinstance(summary, Mapping):
            active = int(summary.get("active_transfer_count", 0) or 0)
            queued = int(summary.get("queued_transfer_count", 0) or 0)
            if isinstance(summary.get("job_runtime_state"), Mapping):
                jobs = summary["job_runtime_state"]
        if isinstance(runtime_state.get("job_runtime_state"), Mapping):
            jobs = runtime_state["job_runtime_state"]
    total_w = 0.0
    total_active = 0
    mine = 0
    my_w = 1.0
    for key, val in jobs.items():
        if not isinstance(val, Mapping):
            continue
        w = max(0.0, float(val.get("weight", 1.0) or 1.0))
        total_w += w
        b = int(val.get("active_bytes_remaining", 0) or 0)
        total_active += b
        if job is not None and str(key) == job:
            my_w, mine = (w or 1.0), b
    if total_w <= 0.0:
        total_w = max(1.0, my_w)
    if job is not None and job not in jobs:
        total_w += my_w
    charge = charge_bytes(total_bytes, workload, priority)
    avg = (total_active + charge) / max(total_w, 1e-12)
    return LoadView(
        job_id=job, workload_kind=workload, priority=int(priority), busy_relays=frozenset(busy),
        held_relays=held,
        job_weight=my_w, total_weight=total_w, current_job_active_bytes=mine,
        total_active_bytes=total_active, request_charge_bytes=charge,
        average_weighted_active_bytes=avg,
        current_weighted_active_bytes=mine / max(my_w, 1e-12),
        projected_weighted_active_bytes=(mine + charge) / max(my_w, 1e-12),
        fairness_threshold_bytes=avg * FAIRNESS_SLACK,
        active_transfer_count=active, queued_transfer_count=queued)
