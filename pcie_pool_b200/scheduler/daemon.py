"""Daemon-side scheduler: session + bandwidth profile + quotas + load
-> ``SchedulingDecision`` (plan, leases, stats, policy metadata).

Pipeline of one decision:
  1. filter the profile's relays to those owned by the session, with quota
     headroom and not busy in another transfer (skipped when relay admission
     is deferred to the daemon's admission step);
  2. plan (pool / relay / direct) with the planner engine;
  3. derive one lease per relay assignment (30 s TTL);
  4. check the fair-share model;
any failure in 3-4 degrades to a direct plan with a ``fallback_reason``
(reference behaviour: turbobus/scheduler/daemon.py:90-220).
"""

from __future__ import annotations

import threading
import uuid
from collections import OrderedDict
from dataclasses import dataclass
from collections.abc import Mapping
from typing import Callable

from ..planner_engine import PlannerEngine, PlannerEngineOptions
from ..planner_types import PlannerLease, PlannerStats, PlannerTransferPlan
from ..schema import (RelayQuota, SchedulingDecision, SchedulingDecisionState, Session, TransferMode,
                      WorkloadKind)
from .fairness import FAIRNESS_FALLBACK, LoadView, load_view

LEASE_SECONDS = 30.0

PROFILE_MISS = "daemon profile miss"
DIRECT_PROFILE_INVALID = "daemon direct profile invalid"
NO_APPROVED_RELAY = "no daemon-approved relay path"
SESSION_QUOTA = "session chunk quota is unavailable"
RELAY_NOT_ASSIGNED = "relay GPU is not assigned to this session"
RELAY_QUOTA = "relay chunk quota is unavailable"


@dataclass(frozen=True)
class RelayProfileView:
    relay_device: int
    target_device: int
    h2d_bw_gbps: float
    d2h_bw_gbps: float
    p2p_bw_gbps: float
    effective_bw_gbps: float
    effective_d2h_bw_gbps: float
    p2p_enabled: bool


@dataclass(frozen=True)
class ProfileView:
    target_device: int
    direct_h2d_bw_gbps: float
    direct_d2h_bw_gbps: float
    relays: tuple[RelayProfileView, ...]
    concurrent: Mapping[str, object] | None = None


def _direct_only_profile(target: int) -> ProfileView:
    return ProfileView(int(target), 1.0, 1.0, ())


class DaemonScheduler:
    def __init__(self, planner: PlannerEngine | None = None,
                 lease_id_factory: Callable[[], str] | None = None,
                 decision_id_factory: Callable[[], str] | None = None,
                 lease_seconds: float = LEASE_SECONDS) -> None:
        # Blocked layout: each lane takes one contiguous span (host-sequential
        # reads per lane) and the plan carries one chunk run per lane.
        self._planner = planner or PlannerEngine(PlannerEngineOptions(layout="blocked"))
        self._lease_id = lease_id_factory or (lambda: str(uuid.uuid4()))
        self._decision_id = decision_id_factory or (lambda: str(uuid.uuid4()))
        self._lease_seconds = max(0.0, float(lease_seconds))
        # Plans are pure functions of (bytes, ranges, chunk, profile view,
        # mode, direction) and immutable once issued, so a repeated intent
        # shape (a training step, a KV layer group, a benchmark loop) reuses
        # its plan, the plan's dict form and its path summary.
        self._plans: OrderedDict = OrderedDict()
        self._plans_lock = threading.Lock()
        self.plan_cache_size = 256
        self.plan_cache_hits = 0

    @property
    def planner(self) -> PlannerEngine:
        return self._planner

    def plan_transfer(self, *, session: Session, profile_entry: Mapping[str, object] | None,
                      relay_quotas: Mapping[int, RelayQuota], total_bytes: int, chunk_bytes: int,
                      ranges: tuple[Mapping[str, int], ...] | None = None,
                      mode: TransferMode | str = TransferMode.POOL, direction: str = "h2d",
                      runtime_state: Mapping[str, object] | None = None,
                      workload_kind: WorkloadKind | str = WorkloadKind.GENERIC, priority: int = 0,
                      now: float = 0.0, job_id: str | None = None, intent_id: str | None = None,
                      topology_snapshot_id: str | None = None,
                      defer_relay_admission: bool = False) -> SchedulingDecision:
        total = int(total_bytes)
        chunk = int(chunk_bytes)
        rs = _ranges(ranges)
        direction = str(direction).lower()
        if total < 0:
            raise ValueError("total_bytes must be non-negative")
        if chunk <= 0:
            raise ValueError("chunk_bytes must be positive")
        if rs is not None and sum(r["bytes"] for r in rs) != total:
            raise ValueError("range bytes must match total_bytes")
        if direction not in ("h2d", "d2h"):
            raise ValueError("direction must be h2d or d2h")
        if not session.active:
            raise ValueError("session is closed")
        requested = parse_mode(mode)
        planning = TransferMode.POOL if requested is TransferMode.AUTO else requested
        view = load_view(runtime_state, job_id=job_id, total_bytes=total,
                         workload_kind=WorkloadKind(workload_kind).value, priority=priority)
        profile, reason = self._profile(profile_entry, session, relay_quotas, direction, view,
                                        defer_relay_admission)
        if reason is None and planning is not TransferMode.DIRECT and session.relay_gpus \
                and not profile.relays:
            reason = NO_APPROVED_RELAY
        plan = self._plan_or_direct(total, chunk, rs, profile, planning, direction)
        leases, lease_err = self._leases(plan, session, relay_quotas, direction, now, job_id,
                                         defer_relay_admission)
        if any(a.path.kind == "relay" for a in plan.assignments) and view.relay_over_share():
            lease_err = FAIRNESS_FALLBACK
        if lease_err is not None:
            reason = lease_err
            plan = self._direct_plan(total, chunk, rs, profile, direction)
            leases = ()
        stats = plan_stats(plan, requested_mode=requested, fallback_reason=reason)
        plan_dict, summary = self._plan_forms(plan)
        return SchedulingDecision(
            decision_id=self._decision_id(),
            intent_id=_cid(intent_id, "intent", session.session_id),
            topology_snapshot_id=_cid(topology_snapshot_id, "topology", session.session_id),
            job_id=str(job_id or session.session_id),
            session_id=session.session_id,
            state=SchedulingDecisionState.FALLBACK if reason else SchedulingDecisionState.PLANNED,
            plan=plan_dict,
            path_summary=summary,
            fallback_reason=reason,
            issued_at=float(now),
            metadata={"leases": [l.as_dict() for l in leases], "stats": stats.as_dict(),
                      "runtime_state": runtime_state_metadata(runtime_state),
                      "policy": view.policy_metadata()})

    # ---- steps ----------------------------------------------------------------------
    def _profile(self, entry, session: Session, quotas, direction: str, view: LoadView,
                 defer: bool) -> tuple[ProfileView, str | None]:
        payload = profile_payload(entry)
        if payload is None:
            return _direct_only_profile(session.target_gpu), PROFILE_MISS
        allowed = {int(g) for g in session.relay_gpus}
        relays = []
        for r in payload.get("relays", []) or []:
            if not isinstance(r, Mapping):
                continue
            dev = int(r["relay_device"])
            if dev not in allowed:
                continue
            if dev in view.held_relays:
                continue
            if not defer and (not _has_capacity(session, quotas.get(dev)) or dev in view.busy_relays):
                continue
            relays.append(RelayProfileView(
                relay_device=dev, target_device=int(r.get("target_device", session.target_gpu)),
                h2d_bw_gbps=float(r.get("h2d_bw_gbps", 0.0) or 0.0),
                d2h_bw_gbps=float(r.get("d2h_bw_gbps", 0.0) or 0.0),
                p2p_bw_gbps=float(r.get("p2p_bw_gbps", 0.0) or 0.0),
                effective_bw_gbps=float(r.get("effective_bw_gbps", 0.0) or 0.0),
                effective_d2h_bw_gbps=float(r.get("effective_d2h_bw_gbps", 0.0) or 0.0),
                p2p_enabled=bool(r.get("p2p_enabled", False))))
        h2d = float(payload.get("direct_h2d_bw_gbps", 0.0) or 0.0)
        d2h = float(payload.get("direct_d2h_bw_gbps", 0.0) or h2d)
        if direction == "h2d" and h2d <= 0.0:
            return _direct_only_profile(session.target_gpu), DIRECT_PROFILE_INVALID
        if direction == "d2h" and d2h <= 0.0:
            d2h = h2d
        return ProfileView(int(payload.get("target_device", session.target_gpu)), h2d, d2h,
                           tuple(relays), dict(payload.get("concurrent", {}) or {})), None

    def _cached(self, key, make) -> PlannerTransferPlan:
        with self._plans_lock:
            hit = self._plans.get(key)
            if hit is not None:
                self._plans.move_to_end(key)
                self.plan_cache_hits += 1
                return hit[0]
        plan = make()
        with self._plans_lock:
            self._plans[key] = (plan, None)
            while len(self._plans) > self.plan_cache_size:
                self._plans.popitem(last=False)
        return plan

    def _plan_forms(self, plan: PlannerTransferPlan) -> tuple[dict, tuple]:
        """(dict form, path summary) of a plan, kept with the cached plan."""
        with self._plans_lock:
            for key in reversed(self._plans):
                p, forms = self._plans[key]
                if p is plan:
                    if forms is None:
                        forms = (plan.as_dict(), path_summary(plan))
                        self._plans[key] = (p, forms)
                    return forms
                break  # only the entry just used is looked at
        return plan.as_dict(), path_summary(plan)

    def _plan_or_direct(self, total, chunk, rs, profile, mode, direction) -> PlannerTransferPlan:
        def make():
            try:
                if rs is not None:
                    return self._planner.plan_ranges(rs, chunk, profile, mode, direction=direction)
                return self._planner.plan(total, chunk, profile, mode, direction=direction)
            except RuntimeError:
                return self._direct_plan(total, chunk, rs, profile, direction)

        return self._cached(_plan_key("plan", total, chunk, rs, profile, mode, direction), make)

    def _direct_plan(self, total, chunk, rs, profile: ProfileView, direction) -> PlannerTransferPlan:
        prof = ProfileView(profile.target_device, profile.direct_h2d_bw_gbps or 1.0,
                           profile.direct_d2h_bw_gbps or profile.direct_h2d_bw_gbps or 1.0, ())

        def make():
            if rs is not None:
                return self._planner.plan_ranges(rs, chunk, prof, TransferMode.DIRECT, direction=direction)
            return self._planner.plan(total, chunk, prof, TransferMode.DIRECT, direction=direction)

        return self._cached(_plan_key("direct", total, chunk, rs, prof, TransferMode.DIRECT, direction), make)

    def _leases(self, plan: PlannerTransferPlan, session: Session, quotas, direction, now, job_id,
                defer) -> tuple[tuple[PlannerLease, ...], str | None]:
        specs = [(int(a.path.relay_device), a.chunk_count, a.bytes)
                 for a in plan.assignments if a.path.kind == "relay" and a.chunk_count]
        if not specs:
            return (), None
        if not defer and session.active_chunks + sum(s[1] for s in specs) > session.max_inflight_chunks:
            return (), SESSION_QUOTA
        out = []
        for dev, chunks, nbytes in specs:
            if dev not in session.relay_gpus:
                return (), RELAY_NOT_ASSIGNED
            q = quotas.get(dev)
            if q is None or (not defer and not q.can_reserve(chunks)):
                return (), RELAY_QUOTA
            out.append(PlannerLease(lease_id=self._lease_id(), session_id=session.session_id,
                                    relay_device=dev, chunk_limit=chunks, bytes_limit=nbytes,
                                    direction=direction, granted_at=float(now),
                                    expires_at=float(now) + self._lease_seconds, job_id=job_id))
        return tuple(out), None


# ---- helpers shared with the daemon --------------------------------------------------

def parse_mode(mode: TransferMode | str) -> TransferMode:
    if isinstance(mode, TransferMode):
        return mode
    try:
        return TransferMode(str(mode))
    except ValueError:
        pass
    try:
        return TransferMode[str(mode).upper()]
    except KeyError:
        raise ValueError(f"mode must be one of {', '.join(m.value for m in TransferMode)}") from None


def resolved_mode(plan: PlannerTransferPlan) -> TransferMode:
    kinds = {a.path.kind for a in plan.assignments}
    if {"direct", "relay"} <= kinds:
        return TransferMode.POOL
    return TransferMode.RELAY if "relay" in kinds else TransferMode.DIRECT


def _plan_key(tag: str, total, chunk, rs, profile: ProfileView, mode, direction) -> tuple:
    conc = (profile.concurrent or {}).get(direction) if profile.concurrent else None
    ck = None
    if isinstance(conc, Mapping):
        ck = (tuple(int(x) for x in conc.get("lanes") or ()),
              tuple(sorted((str(k), float(v)) for k, v in (conc.get("lane_gibps") or {}).items())))
    ranges = None if rs is None else tuple((r["src_offset"], r["dst_offset"], r["bytes"]) for r in rs)
    return (tag, int(total), int(chunk), ranges, profile.target_device, profile.direct_h2d_bw_gbps,
            profile.direct_d2h_bw_gbps, profile.relays, ck, str(getattr(mode, "value", mode)), direction)


def plan_stats(plan: PlannerTransferPlan, *, requested_mode: TransferMode,
               fallback_reason: str | None) -> PlannerStats:
    d_b = r_b = d_c = r_c = r_p = 0
    for a in plan.assignments:
        if a.path.kind == "relay":
            r_b += a.bytes
            r_c += a.chunk_count
            r_p += 1
        else:
            d_b += a.bytes
            d_c += a.chunk_count
    return PlannerStats(bytes=int(plan.total_bytes), direct_bytes=d_b, relay_bytes=r_b,
                        direct_chunks=d_c, relay_chunks=r_c, path_count=len(plan.assignments),
                        relay_path_count=r_p, fallback_reason=fallback_reason,
                        requested_mode=requested_mode, resolved_mode=resolved_mode(plan))


def path_summary(plan: PlannerTransferPlan) -> tuple[dict[str, object], ...]:
    return tuple({"kind": a.path.kind, "direction": a.path.direction,
                  "target_device": a.path.target_device, "relay_device": a.path.relay_device,
                  "bytes": a.bytes, "chunk_count": a.chunk_count} for a in plan.assignments)


def runtime_state_metadata(state: Mapping[str, object] | None) -> dict[str, object]:
    if not isinstance(state, Mapping):
        return {"version": 0, "queued_transfer_count": 0, "running_transfer_count": 0,
                "active_transfer_count": 0}
    s = state.get("summary", {})
    s = s if isinstance(s, Mapping) else {}
    ints = ("queued_transfer_count", "running_transfer_count", "active_transfer_count",
            "active_reservation_count", "active_lease_count", "relay_staging_count",
            "relay_path_count", "relay_path_bytes_total")
    out: dict[str, object] = {"version": int(state.get("version", 0) or 0)}
    out.update({k: int(s.get(k, 0) or 0) for k in ints})
    for k in ("active_bytes_by_direction", "queued_bytes_by_direction", "active_resource_usage"):
        out[k] = dict(s.get(k, {}) or {})
    return out


def profile_payload(entry: Mapping[str, object] | None) -> Mapping[str, object] | None:
    if not entry:
        return None
    prof = entry.get("profile")
    return prof if isinstance(prof, Mapping) else entry


def scheduling_decision_leases(decision: SchedulingDecision) -> tuple[PlannerLease, ...]:
    """The decision's leases as records; parsed once per decision (a
    decision is immutable) and kept on it."""
    if not isinstance(decision, SchedulingDecision):
        raise TypeError("decision must be a SchedulingDecision")
    cached = decision.__dict__.get("_parsed_leases")
    if cached is not None:
        return cached
    out = _parse_leases(decision)
    object.__setattr__(decision, "_parsed_leases", out)
    return out


def _parse_leases(decision: SchedulingDecision) -> tuple[PlannerLease, ...]:
    leases = decision.metadata.get("leases", ())
    if not isinstance(leases, (tuple, list)):
        raise ValueError("scheduling decision metadata leases must be a sequence")
    out = []
    for p in leases:
        if not isinstance(p, Mapping):
            raise ValueError("scheduling decision lease must be a mapping")
        out.append(PlannerLease(
            lease_id=str(p["lease_id"]), session_id=str(p["session_id"]),
            relay_device=int(p["relay_device"]), chunk_limit=int(p["chunk_limit"]),
            bytes_limit=int(p.get("bytes_limit", 0)), direction=str(p.get("direction", "unknown")),
            granted_at=float(p.get("granted_at", 0.0)), expires_at=float(p.get("expires_at", 0.0)),
            active=bool(p.get("active", True)), job_id=p.get("job_id"), reason=p.get("reason")))
    return tuple(out)


def scheduling_decision_stats(decision: SchedulingDecision) -> PlannerStats:
    if not isinstance(decision, SchedulingDecision):
        raise TypeError("decision must be a SchedulingDecision")
    p = decision.metadata.get("stats", {})
    if not isinstance(p, Mapping):
        raise ValueError("scheduling decision metadata stats must be a mapping")
    return PlannerStats(
        bytes=int(p.get("bytes", 0)), direct_bytes=int(p.get("direct_bytes", 0)),
        relay_bytes=int(p.get("relay_bytes", 0)), direct_chunks=int(p.get("direct_chunks", 0)),
        relay_chunks=int(p.get("relay_chunks", 0)), path_count=int(p.get("path_count", 0)),
        relay_path_count=int(p.get("relay_path_count", 0)),
        fallback_reason=p.get("fallback_reason"),
        requested_mode=p.get("requested_mode", TransferMode.POOL),
        resolved_mode=p.get("resolved_mode", TransferMode.POOL))


def _has_capacity(session: Session, quota: RelayQuota | None) -> bool:
    return (quota is not None and session.active_chunks < session.max_inflight_chunks
            and quota.active_chunks < quota.max_inflight_chunks)


def _cid(value: str | None, prefix: str, fallback: str) -> str:
    return str(value) if value is not None and str(value).strip() else f"{prefix}-{fallback}"


def _ranges(ranges) -> tuple[dict[str, int], ...] | None:
    if ranges is None:
        return None
    out = []
    for item in ranges:
        if not isinstance(item, Mapping):
            raise ValueError("ranges must contain mappings")
        s, d, n = int(item["src_offset"]), int(item["dst_offset"]), int(item["bytes"])
        if s < 0 or d < 0:
            raise ValueError("range offsets must be non-negative")
        if n <= 0:
            raise ValueError("range bytes must be positive")
        out.append({"src_offset": s, "dst_offset": d, "bytes": n})
    return tuple(out)


__all__ = ["DaemonScheduler", "SchedulingDecision", "scheduling_decision_leases",
           "scheduling_decision_stats", "plan_stats", "path_summary", "parse_mode",
           "resolved_mode", "profile_payload", "runtime_state_metadata"]
