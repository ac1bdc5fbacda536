"""Worker helper core: authorize -> validate ticket -> stage -> bind -> execute
-> check bytes -> report -> release/clean up -> release staging.

Lifecycle and failure semantics follow turbobus/worker/helper.py:
every stage failure ends in a recorded ``final_state``
(``authorization_failed``, ``status_failed``, ``cleanup_failed``,
``complete`` or ``failed``, :884-1026); tickets must come from the daemon
(issuer ``turbobus-daemon``, positive plan generation, a transfer id,
:1320-1339) and must match the decision, buffers, relays and ranges
(:1275-1481); completed bytes must equal the plan's (:1163-1209); cleanup is
multi-lease aware (:602-800).  The execution step runs the WHOLE ticketed
plan (direct and relay lanes) on the worker's persistent engine.
"""

from __future__ import annotations

from ..planner_types import assignment_chunks

from dataclasses import asdict, dataclass, field
from enum import Enum
from collections.abc import Mapping
from typing import Any, Iterable

from ..schema import (BufferRegistration, DaemonResponse, ExecutionTicket, SchedulingDecision,
                      TransferStatusState, WorkerDataPlaneCompletion, WorkerDataPlaneRequest,
                      WorkerTransferAuthorization, WorkerTransferAuthorizationRequest)
from .resources import WorkerDataPlaneResourceBinder, WorkerDataPlaneResourceError
from .staging_pool import WorkerStagingPool, WorkerStagingSlot

TICKET_ISSUER = "turbobus-daemon"


class WorkerTransferState(str, Enum):
    FAILED = "failed"
    COMPLETE = "complete"


class WorkerAuthorizationError(RuntimeError):
    pass


class WorkerStatusReportError(RuntimeError):
    pass


class WorkerCleanupError(RuntimeError):
    pass


# ---- plan walking -------------------------------------------------------------------------------

def _assignments(plan: Mapping[str, Any]):
    for a in plan.get("assignments", ()) or ():
        if not isinstance(a, Mapping):
            raise ValueError("daemon plan assignment must be an object")
        p = a.get("path")
        if not isinstance(p, Mapping):
            raise ValueError("daemon plan assignment path must be an object")
        yield a, p


def _chunks(a: Mapping[str, Any]):
    try:
        chunks = assignment_chunks(a)
    except ValueError as exc:
        raise ValueError(f"daemon plan chunk is invalid: {exc}") from None
    for c in chunks:
        yield {"src_offset": int(c["src_offset"]), "dst_offset": int(c["dst_offset"]), "bytes": int(c["bytes"])}


def planned_relays(plan: Mapping[str, Any]) -> tuple[int, ...]:
    out = []
    for _a, p in _assignments(plan):
        if str(p.get("kind", "")).lower() == "relay":
            r = int(p.get("relay_device", -1))
            if r not in out:
                out.append(r)
    return tuple(out)


def relay_ranges_for(ticket: ExecutionTicket, relays: Iterable[int]) -> tuple[dict[str, int], ...]:
    auth = {int(r) for r in relays}
    if not auth:
        raise ValueError("ticket relay_gpus must not be empty")
    out = []
    for a, p in _assignments(ticket.plan):
        if str(p.get("kind", "")).lower() != "relay" or int(p.get("relay_device", -1)) not in auth:
            continue
        if str(p.get("direction", "")).lower() != ticket.direction:
            raise ValueError("ticket plan direction does not match ticket")
        out.extend(_chunks(a))
    if not out:
        raise ValueError("ticket plan has no authorized relay chunks")
    if sum(r["bytes"] for r in out) > ticket.total_bytes:
        raise ValueError("ticket relay ranges exceed ticket total bytes")
    return tuple(out)


def plan_total_bytes(plan: Mapping[str, Any]) -> int:
    return sum(c["bytes"] for a, _p in _assignments(plan) for c in _chunks(a))


# ---- ticket validation ----------------------------------------------------------------------------

def validate_daemon_ticket(ticket: ExecutionTicket, plan_generation: object | None = None) -> None:
    if not isinstance(ticket, ExecutionTicket):
        raise TypeError("ticket must be an ExecutionTicket")
    md = ticket.metadata
    if md.get("issuer") != TICKET_ISSUER:
        raise ValueError(f"execution ticket must be issued by {TICKET_ISSUER}")
    gen = md.get("plan_generation")
    if gen is None:
        raise ValueError("execution ticket missing plan_generation")
    if int(gen) <= 0:
        raise ValueError("execution ticket plan_generation must be positive")
    if plan_generation is not None and int(plan_generation) != int(gen):
        raise ValueError("execution ticket plan_generation is stale")
    tid = md.get("transfer_id")
    if tid is None or not str(tid).strip():
        raise ValueError("execution ticket missing transfer_id")


def _check_ticket_buffers(ticket: ExecutionTicket, src: BufferRegistration, dst: BufferRegistration) -> None:
    if not isinstance(src, BufferRegistration) or not isinstance(dst, BufferRegistration):
        raise TypeError("src_buffer and dst_buffer must be BufferRegistration")
    if src.buffer_id != ticket.source_buffer_id:
        raise ValueError("ticket source buffer does not match worker buffer")
    if dst.buffer_id != ticket.destination_buffer_id:
        raise ValueError("ticket destination buffer does not match worker buffer")
    if src.job_id != ticket.job_id or dst.job_id != ticket.job_id:
        raise ValueError("ticket job does not match worker buffers")


def _check_ticket_decision(ticket: ExecutionTicket, d: SchedulingDecision, plan_generation) -> None:
    for attr in ("decision_id", "intent_id", "topology_snapshot_id", "job_id", "session_id"):
        if getattr(ticket, attr) != getattr(d, attr):
            raise ValueError(f"ticket {attr} does not match scheduling decision")
    if dict(ticket.plan) != dict(d.plan):
        raise ValueError("ticket plan does not match scheduling decision")
    dg = (d.metadata or {}).get("plan_generation") if hasattr(d, "metadata") else None
    if dg is not None and int(dg) != int(ticket.metadata.get("plan_generation", 0)):
        raise ValueError("ticket plan_generation does not match scheduling decision")


def _resolve_relays(ticket: ExecutionTicket, relay_gpu, relay_gpus) -> tuple[int, ...]:
    planned = planned_relays(ticket.plan)
    if not planned:
        raise ValueError("worker ticket requires at least one relay path")
    req = None
    if relay_gpus is not None:
        req = tuple(int(r) for r in relay_gpus)
        if not req:
            raise ValueError("worker ticket relay_gpus must not be empty")
    if relay_gpu is not None:
        if req is None:
            req = (int(relay_gpu),)
        elif int(relay_gpu) not in req:
            raise ValueError("ticket relay does not match requested relay_gpus")
    if req is None:
        return planned
    if set(req) - set(planned):
        raise ValueError("ticket relay does not match daemon plan")
    return req


def _resolve_leases(ticket: ExecutionTicket, lease_id, lease_ids) -> tuple[str, ...]:
    req = None
    if lease_ids is not None:
        req = tuple(str(x) for x in lease_ids)
        if not req or any(not x.strip() for x in req):
            raise ValueError("worker ticket lease_ids must be non-empty")
    if lease_id is not None:
        if req is None:
            req = (str(lease_id),)
        elif str(lease_id) not in req:
            raise ValueError("worker lease_id does not match requested lease_ids")
    have = tuple(ticket.lease_ids)
    if not have:
        raise ValueError("worker ticket requires at least one lease id")
    if req is None:
        return have
    if set(req) - set(have):
        raise ValueError("worker lease_id does not match ticket")
    return req


def _buffer(payload) -> BufferRegistration:
    if not isinstance(payload, Mapping):
        raise ValueError("buffer payload must be a mapping")
    return BufferRegistration(**{k: payload[k] for k in ("buffer_id", "job_id", "kind", "size_bytes")},
                              device_index=payload.get("device_index"), address=payload.get("address"),
                              pinned=bool(payload.get("pinned", False)),
                              handle_type=payload.get("handle_type", "registered_buffer"),
                              metadata=dict(payload.get("metadata") or {}))


# ---- request / result ----------------------------------------------------------------------------

@dataclass(frozen=True)
class WorkerTransferRequest:
    authorization: WorkerTransferAuthorization
    ticket: ExecutionTicket
    data_plane: WorkerDataPlaneRequest | None = None

    @classmethod
    def from_authorization_payload(cls, payload: Mapping[str, object]) -> "WorkerTransferRequest":
        if not isinstance(payload, Mapping):
            raise ValueError("authorization payload must be a mapping")
        if payload.get("ticket") is None:
            raise ValueError("daemon worker authorization response must include execution ticket")
        return cls.from_execution_ticket_payload(payload)

    @classmethod
    def from_execution_ticket_payload(cls, payload: Mapping[str, object]) -> "WorkerTransferRequest":
        if not isinstance(payload, Mapping) or not isinstance(payload.get("ticket"), Mapping):
            raise ValueError("execution ticket payload must include ticket")
        dec = payload.get("decision")
        return cls.from_execution_ticket(
            ExecutionTicket(**dict(payload["ticket"])), src_buffer=_buffer(payload["src_buffer"]),
            dst_buffer=_buffer(payload["dst_buffer"]), relay_gpu=payload.get("relay_gpu"),
            relay_gpus=payload.get("relay_gpus"), lease_id=payload.get("lease_id"),
            lease_ids=payload.get("lease_ids"), transfer_id=payload.get("transfer_id"),
            decision=None if dec is None else SchedulingDecision(**dict(dec)),
            plan_generation=payload.get("plan_generation"))

    @classmethod
    def from_authorization(cls, authorization: WorkerTransferAuthorization) -> "WorkerTransferRequest":
        raise ValueError("worker transfer requests must be built from daemon-issued ExecutionTicket objects")

    @classmethod
    def from_execution_ticket(cls, ticket: ExecutionTicket, *, src_buffer: BufferRegistration,
                              dst_buffer: BufferRegistration, relay_gpu: int | None = None,
                              relay_gpus: Iterable[int] | None = None, lease_id: str | None = None,
                              lease_ids: Iterable[str] | None = None, transfer_id: str | None = None,
                              decision: SchedulingDecision | None = None,
                              plan_generation: object | None = None) -> "WorkerTransferRequest":
        _check_ticket_buffers(ticket, src_buffer, dst_buffer)
        validate_daemon_ticket(ticket, plan_generation)
        if decision is not None:
            _check_ticket_decision(ticket, decision, plan_generation)
        relays = _resolve_relays(ticket, relay_gpu, relay_gpus)
        primary = int(relay_gpu) if relay_gpu is not None else relays[0]
        if primary not in relays:
            raise ValueError("ticket relay does not match daemon plan")
        leases = _resolve_leases(ticket, lease_id, lease_ids)
        primary_lease = str(lease_id) if lease_id is not None else leases[0]
        tid = str(transfer_id) if transfer_id is not None else str(
            ticket.metadata.get("transfer_id") or ticket.ticket_id)
        auth = WorkerTransferAuthorization(
            transfer_id=tid, lease_id=primary_lease, session_id=ticket.session_id, job_id=ticket.job_id,
            src_buffer=src_buffer, dst_buffer=dst_buffer, direction=ticket.direction,
            ranges=relay_ranges_for(ticket, relays), relay_gpu=primary, plan=dict(ticket.plan))
        dp = WorkerDataPlaneRequest.from_authorization(auth, metadata={
            "relay_gpus": relays, "lease_ids": leases, "primary_relay_gpu": primary,
            "primary_lease_id": primary_lease,
            "relay_ranges_by_gpu": {str(r): relay_ranges_for(ticket, (r,)) for r in relays}})
        return cls(authorization=auth, ticket=ticket, data_plane=dp)

    def __post_init__(self) -> None:
        a = self.authorization
        if not isinstance(a, WorkerTransferAuthorization):
            raise TypeError("authorization must be a WorkerTransferAuthorization")
        dp = self.data_plane if self.data_plane is not None else WorkerDataPlaneRequest.from_authorization(a)
        if not isinstance(dp, WorkerDataPlaneRequest):
            raise TypeError("data_plane must be a WorkerDataPlaneRequest")
        pairs = (("transfer_id", dp.transfer_id, a.transfer_id), ("lease_id", dp.lease_id, a.lease_id),
                 ("session_id", dp.session_id, a.session_id), ("job_id", dp.job_id, a.job_id),
                 ("relay", dp.relay_gpu, a.relay_gpu), ("direction", dp.direction, a.direction),
                 ("src handle", dp.src_handle.buffer_id, a.src_buffer.buffer_id),
                 ("dst handle", dp.dst_handle.buffer_id, a.dst_buffer.buffer_id),
                 ("ranges", dp.ranges, a.ranges), ("plan", dp.plan, a.plan))
        for what, x, y in pairs:
            if x != y:
                raise ValueError(f"data-plane {what} does not match authorization")
        if not isinstance(self.ticket, ExecutionTicket):
            raise TypeError("ticket must be an ExecutionTicket")
        validate_daemon_ticket(self.ticket)
        t = self.ticket
        for what, x, y in (("job", t.job_id, a.job_id), ("session", t.session_id, a.session_id),
                           ("source buffer", t.source_buffer_id, a.src_buffer.buffer_id),
                           ("destination buffer", t.destination_buffer_id, a.dst_buffer.buffer_id),
                           ("direction", t.direction, a.direction), ("plan", dict(t.plan), a.plan)):
            if x != y:
                raise ValueError(f"ticket {what} does not match worker authorization")
        relays = tuple(int(r) for r in dp.metadata.get("relay_gpus", (a.relay_gpu,)))
        if a.relay_gpu not in relays:
            raise ValueError("ticket relay does not match worker authorization")
        if relay_ranges_for(t, relays) != a.ranges:
            raise ValueError("ticket ranges do not match worker authorization")
        object.__setattr__(self, "data_plane", dp)

    @property
    def transfer_id(self) -> str:
        return self.authorization.transfer_id

    @property
    def relay_gpus(self) -> tuple[int, ...]:
        return tuple(int(r) for r in self.data_plane.metadata.get("relay_gpus", (self.data_plane.relay_gpu,)))

    @property
    def lease_ids(self) -> tuple[str, ...]:
        ids = tuple(str(x) for x in self.data_plane.metadata.get("lease_ids", (self.authorization.lease_id,)))
        if not ids:
            raise ValueError("worker request has no lease ids")
        if self.authorization.lease_id not in ids:
            raise ValueError("worker request primary lease is not authorized")
        return ids

    def as_dict(self) -> dict[str, object]:
        return {"authorization": asdict(self.authorization), "data_plane": asdict(self.data_plane),
                "ticket": asdict(self.ticket)}


@dataclass(frozen=True)
class WorkerTransferResult:
    transfer_id: str
    state: WorkerTransferState
    error: str | None = None
    bytes_completed: int = 0
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not str(self.transfer_id).strip():
            raise ValueError("transfer_id must be non-empty")
        if int(self.bytes_completed) < 0:
            raise ValueError("bytes_completed must be non-negative")
        object.__setattr__(self, "transfer_id", str(self.transfer_id))
        object.__setattr__(self, "state", WorkerTransferState(self.state))
        object.__setattr__(self, "bytes_completed", int(self.bytes_completed))
        if self.error is not None:
            object.__setattr__(self, "error", str(self.error))
        object.__setattr__(self, "metadata", dict(self.metadata))

    def as_dict(self) -> dict[str, object]:
        return {"transfer_id": self.transfer_id, "state": self.state.value, "error": self.error,
                "bytes_completed": self.bytes_completed, "metadata": dict(self.metadata)}

    def data_plane_completion(self, lease_id: str) -> WorkerDataPlaneCompletion:
        u = status_update_for(self)
        return WorkerDataPlaneCompletion(transfer_id=self.transfer_id, lease_id=lease_id, state=u["state"],
                                         bytes_completed=self.bytes_completed,
                                         error=u["error"] if u["state"] == "failed" else None,
                                         metadata=dict(self.metadata))


def status_update_for(result: WorkerTransferResult) -> dict[str, object]:
    state = TransferStatusState.COMPLETE if result.state is WorkerTransferState.COMPLETE else TransferStatusState.FAILED
    err = result.error
    if state is TransferStatusState.FAILED and err is None:
        err = "worker transfer failed"
    return {"transfer_id": result.transfer_id, "state": state.value, "bytes_completed": result.bytes_completed,
            "error": err}


def _failed(request: WorkerTransferRequest, slot: WorkerStagingSlot | None, error: str) -> WorkerTransferResult:
    md = {"executor": "worker", "relay_gpu": request.data_plane.relay_gpu}
    if slot is not None:
        md["staging_slot_id"] = slot.slot_id
    return WorkerTransferResult(request.transfer_id, WorkerTransferState.FAILED, error=error, metadata=md)


def check_completion_bytes(request: WorkerTransferRequest, result: WorkerTransferResult) -> WorkerTransferResult:
    if result.state is not WorkerTransferState.COMPLETE:
        return result
    want = plan_total_bytes(request.data_plane.plan)
    if want <= 0:
        raise ValueError("daemon worker plan has no bytes to complete")
    if result.bytes_completed == want:
        return result
    return WorkerTransferResult(result.transfer_id, WorkerTransferState.FAILED,
                                error=f"worker completed {result.bytes_completed} bytes, plan has {want}",
                                bytes_completed=result.bytes_completed, metadata=result.metadata)


def require_daemon_worker_plan(request: WorkerTransferRequest) -> None:
    dp = request.data_plane
    if not dp.plan:
        raise ValueError("daemon worker authorization did not include a transfer plan")
    if not list(dp.plan.get("assignments", ()) or ()):
        raise ValueError("daemon worker authorization plan has no assignments")
    target_h = dp.dst_handle if dp.direction == "h2d" else dp.src_handle
    if target_h.device_index is None:
        raise ValueError("worker target handle requires a CUDA device index")
    target = int(target_h.device_index)
    relays = set(request.relay_gpus)
    total, rr = 0, []
    for a, p in _assignments(dp.plan):
        kind = str(p.get("kind", "")).lower()
        if kind not in ("direct", "relay"):
            raise ValueError("daemon plan path must be direct or relay")
        if str(p.get("direction", "")).lower() != dp.direction:
            raise ValueError("daemon plan direction does not match worker request")
        if int(p.get("target_device", target)) != target:
            raise ValueError("daemon plan target does not match worker device")
        if not bool(p.get("enabled", True)):
            raise ValueError("daemon plan path is disabled")
        if kind == "relay" and int(p.get("relay_device", -1)) not in relays:
            raise ValueError("daemon plan relay is not authorized by worker ticket")
        for c in _chunks(a):
            total += c["bytes"]
            if kind == "relay":
                rr.append(c)
    if total <= 0:
        raise ValueError("daemon plan has no assigned bytes")
    if int(dp.plan.get("total_bytes", total)) != total:
        raise ValueError("daemon plan total bytes do not match assigned chunks")
    if not rr:
        raise ValueError("daemon plan has no authorized relay chunks")
    if tuple(rr) != dp.ranges:
        raise ValueError("authorized ranges do not match daemon plan")


def cleanup_target(kind: str, lease_id: str, session_id: str) -> str:
    k = str(kind).lower()
    if k == "reservation":
        return str(lease_id)
    if k == "session":
        return str(session_id)
    raise ValueError("worker cleanup target must be reservation or session")


# ---- lifecycle records and envelopes -----------------------------------------------------------------

@dataclass(frozen=True)
class WorkerTransferLifecycleRecord:
    authorization_request: WorkerTransferAuthorizationRequest
    worker_request: WorkerTransferRequest | None = None
    staging_slot: WorkerStagingSlot | None = None
    staging_release: WorkerStagingSlot | None = None
    result: WorkerTransferResult | None = None
    status_update: Mapping[str, object] | None = None
    status_response: DaemonResponse | None = None
    cleanup_target_kind: str | None = None
    cleanup_target_id: str | None = None
    cleanup_response: DaemonResponse | None = None
    final_state: str = "created"
    error: str | None = None

    def __post_init__(self) -> None:
        checks = (("authorization_request", WorkerTransferAuthorizationRequest, False),
                  ("worker_request", WorkerTransferRequest, True), ("staging_slot", WorkerStagingSlot, True),
                  ("staging_release", WorkerStagingSlot, True), ("result", WorkerTransferResult, True),
                  ("status_response", DaemonResponse, True), ("cleanup_response", DaemonResponse, True))
        for name, typ, optional in checks:
            v = getattr(self, name)
            if (v is None and not optional) or (v is not None and not isinstance(v, typ)):
                raise TypeError(f"{name} must be a {typ.__name__}")
        if self.status_update is not None:
            if not isinstance(self.status_update, Mapping):
                raise TypeError("status_update must be a mapping")
            object.__setattr__(self, "status_update", dict(self.status_update))
        if not str(self.final_state).strip():
            raise ValueError("final_state must be non-empty")
        object.__setattr__(self, "final_state", str(self.final_state))
        for name in ("cleanup_target_kind", "cleanup_target_id", "error"):
            if getattr(self, name) is not None:
                object.__setattr__(self, name, str(getattr(self, name)))

    @property
    def lease_ids(self) -> tuple[str, ...]:
        return self.worker_request.lease_ids if self.worker_request is not None else (
            self.authorization_request.lease_id,)

    @property
    def transfer_id(self) -> str:
        return self.worker_request.transfer_id if self.worker_request is not None else \
            self.authorization_request.transfer_id

    @property
    def lease_id(self) -> str:
        return self.worker_request.authorization.lease_id if self.worker_request is not None else \
            self.authorization_request.lease_id

    def as_dict(self) -> dict[str, object]:
        tgt = None
        if self.cleanup_target_kind is not None or self.cleanup_target_id is not None:
            tgt = {"target_kind": self.cleanup_target_kind, "target_id": self.cleanup_target_id}
        return {
            "authorization_request": asdict(self.authorization_request),
            "worker_request": None if self.worker_request is None else self.worker_request.as_dict(),
            "staging_slot": None if self.staging_slot is None else self.staging_slot.as_dict(),
            "staging_release": None if self.staging_release is None else self.staging_release.as_dict(),
            "result": None if self.result is None else self.result.as_dict(),
            "status_update": None if self.status_update is None else dict(self.status_update),
            "status_response": None if self.status_response is None else asdict(self.status_response),
            "cleanup_target": tgt,
            "cleanup_response": None if self.cleanup_response is None else asdict(self.cleanup_response),
            "lease_ids": self.lease_ids, "final_state": self.final_state, "error": self.error,
        }

    def completion_envelope(self) -> "WorkerDataPlaneCompletionEnvelope":
        return WorkerDataPlaneCompletionEnvelope.from_lifecycle(self)


_MAPPING_FIELDS = ("staging_slot", "worker_result", "daemon_status_update", "daemon_status_response",
                   "daemon_cleanup_response", "staging_release")


@dataclass(frozen=True)
class WorkerDataPlaneCompletionEnvelope:
    ok: bool
    transfer_id: str | None = None
    lease_id: str | None = None
    lease_ids: tuple[str, ...] = ()
    final_state: str | None = None
    staging_slot: Mapping[str, object] | None = None
    worker_result: Mapping[str, object] | None = None
    daemon_status_update: Mapping[str, object] | None = None
    daemon_status_response: Mapping[str, object] | None = None
    daemon_cleanup_response: Mapping[str, object] | None = None
    staging_release: Mapping[str, object] | None = None
    error: str | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "ok", bool(self.ok))
        for name in _MAPPING_FIELDS:
            v = getattr(self, name)
            if v is None:
                continue
            if not isinstance(v, Mapping):
                raise TypeError(f"{name} must be a mapping")
            object.__setattr__(self, name, dict(v))
        for name in ("transfer_id", "lease_id", "final_state", "error"):
            if getattr(self, name) is not None:
                object.__setattr__(self, name, str(getattr(self, name)))
        object.__setattr__(self, "lease_ids", tuple(str(x) for x in self.lease_ids))
        if self.lease_ids and self.lease_id is not None and self.lease_id not in self.lease_ids:
            raise ValueError("lease_id must be included in lease_ids")

    @classmethod
    def from_lifecycle(cls, lifecycle: WorkerTransferLifecycleRecord) -> "WorkerDataPlaneCompletionEnvelope":
        lc = lifecycle
        if not isinstance(lc, WorkerTransferLifecycleRecord):
            raise TypeError("lifecycle must be a WorkerTransferLifecycleRecord")
        d = lc.as_dict()
        return cls(ok=True, transfer_id=lc.transfer_id, lease_id=lc.lease_id, lease_ids=lc.lease_ids,
                   final_state=lc.final_state, staging_slot=d["staging_slot"], worker_result=d["result"],
                   daemon_status_update=d["status_update"], daemon_status_response=d["status_response"],
                   daemon_cleanup_response=d["cleanup_response"], staging_release=d["staging_release"],
                   error=lc.error)

    def as_dict(self) -> dict[str, object]:
        out = {"ok": self.ok, "transfer_id": self.transfer_id, "lease_id": self.lease_id,
               "lease_ids": self.lease_ids, "final_state": self.final_state, "error": self.error}
        for name in _MAPPING_FIELDS:
            v = getattr(self, name)
            out[name] = None if v is None else dict(v)
        return out


@dataclass(frozen=True)
class WorkerServiceRequestEnvelope:
    payload: Mapping[str, object]
    cleanup_target_kind: str = "reservation"

    def __post_init__(self) -> None:
        if not isinstance(self.payload, Mapping):
            raise ValueError("worker service payload must be a mapping")
        k = str(self.cleanup_target_kind)
        if k not in ("reservation", "session"):
            raise ValueError("cleanup_target_kind must be reservation or session")
        object.__setattr__(self, "payload", dict(self.payload))
        object.__setattr__(self, "cleanup_target_kind", k)

    def as_dict(self) -> dict[str, object]:
        return {"payload": dict(self.payload), "cleanup_target_kind": self.cleanup_target_kind}


@dataclass(frozen=True)
class WorkerServiceResponseEnvelope:
    ok: bool
    completion: Mapping[str, object] | None = None
    error: str | None = None
    final_state: str | None = None

    def __post_init__(self) -> None:
        if self.completion is not None and not isinstance(self.completion, Mapping):
            raise TypeError("completion must be a mapping")
        object.__setattr__(self, "ok", bool(self.ok))
        if self.completion is not None:
            object.__setattr__(self, "completion", dict(self.completion))
        for name in ("error", "final_state"):
            if getattr(self, name) is not None:
                object.__setattr__(self, name, str(getattr(self, name)))

    @classmethod
    def from_lifecycle(cls, lifecycle: WorkerTransferLifecycleRecord) -> "WorkerServiceResponseEnvelope":
        return cls(ok=True, completion=lifecycle.completion_envelope().as_dict(), final_state=lifecycle.final_state,
                   error=lifecycle.error)

    @classmethod
    def from_error(cls, error: str) -> "WorkerServiceResponseEnvelope":
        return cls(ok=False, error=str(error))

    def as_dict(self) -> dict[str, object]:
        return {"ok": self.ok, "completion": None if self.completion is None else dict(self.completion),
                "error": self.error, "final_state": self.final_state}


# ---- daemon-facing steps ---------------------------------------------------------------------------

class WorkerTransferAuthorizer:
    def __init__(self, daemon_client) -> None:
        self.daemon_client = daemon_client

    def authorize(self, request: WorkerTransferAuthorizationRequest) -> WorkerTransferRequest:
        resp: DaemonResponse = self.daemon_client.authorize_worker_transfer(request)
        if not resp.ok:
            raise WorkerAuthorizationError(resp.error or "worker transfer authorization failed")
        try:
            wr = WorkerTransferRequest.from_authorization_payload(resp.payload)
            require_daemon_worker_plan(wr)
            return wr
        except (KeyError, TypeError, ValueError) as exc:
            raise WorkerAuthorizationError(f"invalid worker authorization response: {exc}") from exc


class WorkerTransferStatusReporter:
    def __init__(self, daemon_client) -> None:
        self.daemon_client = daemon_client

    def report(self, result: WorkerTransferResult) -> DaemonResponse:
        if not isinstance(result, WorkerTransferResult):
            raise TypeError("result must be a WorkerTransferResult")
        u = status_update_for(result)
        resp: DaemonResponse = self.daemon_client.transfer_status(u["transfer_id"], state=u["state"],
                                                                  bytes_completed=u["bytes_completed"],
                                                                  error=u["error"])
        if not resp.ok:
            raise WorkerStatusReportError(resp.error or "worker transfer status report failed")
        return resp


class WorkerTransferCleanupCoordinator:
    def __init__(self, daemon_client) -> None:
        self.daemon_client = daemon_client

    def cleanup_authorization_failure(self, request: WorkerTransferAuthorizationRequest,
                                      target_kind: str = "reservation",
                                      reason: str = "worker_authorization_failed",
                                      force: bool = True) -> DaemonResponse:
        if not isinstance(request, WorkerTransferAuthorizationRequest):
            raise TypeError("request must be a WorkerTransferAuthorizationRequest")
        return self._cleanup(target_kind, cleanup_target(target_kind, request.lease_id, request.session_id),
                             reason, force)

    def cleanup_execution_failure(self, request: WorkerTransferRequest, result: WorkerTransferResult,
                                  target_kind: str = "reservation", reason: str | None = None,
                                  force: bool = True) -> DaemonResponse:
        if not isinstance(request, WorkerTransferRequest) or not isinstance(result, WorkerTransferResult):
            raise TypeError("request/result must be WorkerTransferRequest/WorkerTransferResult")
        a = request.authorization
        reason = reason or f"worker_{result.state.value}"
        if target_kind == "session":
            return self._cleanup(target_kind, a.session_id, reason, force)
        leases = request.lease_ids
        if result.state is WorkerTransferState.COMPLETE:
            if len(leases) == 1:
                release = getattr(self.daemon_client, "release_transfer", None)
                if not callable(release):
                    raise WorkerCleanupError("daemon client cannot release completed worker transfer")
                resp = release(a.lease_id)
                if not resp.ok:
                    raise WorkerCleanupError(resp.error or "worker completion release failed")
                return resp
            return self._each_lease(leases, target_kind, reason or "worker_complete", force, release=True)
        if len(leases) == 1:
            return self._cleanup(target_kind, cleanup_target(target_kind, a.lease_id, a.session_id), reason, force)
        return self._each_lease(leases, target_kind, reason, force, release=False)

    def cleanup_status_report_failure(self, request: WorkerTransferRequest, target_kind: str = "reservation",
                                      reason: str = "worker_status_report_failed",
                                      force: bool = True) -> DaemonResponse:
        if not isinstance(request, WorkerTransferRequest):
            raise TypeError("request must be a WorkerTransferRequest")
        a = request.authorization
        if target_kind == "session" or len(request.lease_ids) == 1:
            return self._cleanup(target_kind, cleanup_target(target_kind, a.lease_id, a.session_id), reason, force)
        return self._each_lease(request.lease_ids, target_kind, reason, force, release=False)

    def _cleanup(self, kind: str, target_id: str, reason: str, force: bool) -> DaemonResponse:
        resp: DaemonResponse = self.daemon_client.cleanup(target_kind=kind, target_id=target_id, reason=reason,
                                                          force=force)
        if not resp.ok:
            raise WorkerCleanupError(resp.error or "worker cleanup failed")
        return resp

    def _each_lease(self, leases: tuple[str, ...], kind: str, reason: str, force: bool,
                    release: bool) -> DaemonResponse:
        fn = getattr(self.daemon_client, "release_transfer" if release else "cleanup", None)
        if not callable(fn):
            raise WorkerCleanupError("daemon client cannot " + ("release completed" if release else "clean")
                                     + " worker transfer")
        responses, released, errors = [], [], []
        for lid in leases:
            resp = fn(lid) if release else fn(target_kind=kind, target_id=lid, reason=reason, force=force)
            responses.append(asdict(resp))
            if resp.ok:
                pl = resp.payload if isinstance(resp.payload, Mapping) else {}
                released.append(str(pl.get("reservation_id", lid)))
            else:
                errors.append(f"{lid}: {resp.error or 'worker cleanup failed'}")
        if errors:
            raise WorkerCleanupError("; ".join(errors))
        return DaemonResponse(ok=True, payload={
            "reservation_id": leases[0], "lease_ids": leases, "released_reservation_ids": tuple(released),
            "lease_responses": tuple(responses), "cleanup_kind": kind, "reason": reason,
            "cleanup_mode": "release" if release else "cleanup"})


def _default_executor():
    from .cuda_executor import CudaWorkerExecutor

    return CudaWorkerExecutor()


def _execute(executor, binder, request: WorkerTransferRequest, slot: WorkerStagingSlot) -> WorkerTransferResult:
    bound = getattr(executor, "execute_bound", None)
    if binder is not None and callable(bound):
        try:
            with binder.bind(request.data_plane) as res:
                return bound(request, slot, res)
        except WorkerDataPlaneResourceError as exc:
            return _failed(request, slot, str(exc))
    return executor.execute(request, slot)


class WorkerTransferClient:
    """Runs authorized transfers: ``submit`` (execute), ``submit_and_report``,
    ``submit_report_and_cleanup`` and the recorded
    ``submit_report_cleanup_lifecycle``."""

    def __init__(self, daemon_client, executor: object | None = None,
                 status_reporter: WorkerTransferStatusReporter | None = None,
                 cleanup_coordinator: WorkerTransferCleanupCoordinator | None = None,
                 staging_pool: WorkerStagingPool | None = None,
                 resource_binder: WorkerDataPlaneResourceBinder | None = None) -> None:
        if executor is None:
            executor = _default_executor()
            resource_binder = resource_binder or WorkerDataPlaneResourceBinder()
        self.authorizer = WorkerTransferAuthorizer(daemon_client)
        self.executor = executor
        self.status_reporter = status_reporter or WorkerTransferStatusReporter(daemon_client)
        self.cleanup_coordinator = cleanup_coordinator or WorkerTransferCleanupCoordinator(daemon_client)
        self.staging_pool = staging_pool or WorkerStagingPool()
        self.resource_binder = resource_binder

    def authorize(self, request: WorkerTransferAuthorizationRequest) -> WorkerTransferRequest:
        return self.authorizer.authorize(request)

    def _run(self, wr: WorkerTransferRequest, slot: WorkerStagingSlot) -> WorkerTransferResult:
        try:
            return check_completion_bytes(wr, _execute(self.executor, self.resource_binder, wr, slot))
        except Exception as exc:  # noqa: BLE001 - every executor failure becomes a failed result
            return _failed(wr, slot, str(exc))

    def submit(self, request: WorkerTransferAuthorizationRequest) -> WorkerTransferResult:
        wr = self.authorize(request)
        slot = self.staging_pool.allocate(wr.data_plane)
        try:
            return self._run(wr, slot)
        finally:
            self.staging_pool.release(slot.slot_id, wr.data_plane)

    def submit_and_report(self, request: WorkerTransferAuthorizationRequest) -> WorkerTransferResult:
        result = self.submit(request)
        self.status_reporter.report(result)
        return result

    def submit_report_and_cleanup(self, request: WorkerTransferAuthorizationRequest,
                                  cleanup_target_kind: str = "reservation") -> WorkerTransferResult:
        lc = self.submit_report_cleanup_lifecycle(request, cleanup_target_kind=cleanup_target_kind)
        errs = {"authorization_failed": WorkerAuthorizationError, "status_failed": WorkerStatusReportError,
                "cleanup_failed": WorkerCleanupError}
        if lc.final_state in errs:
            raise errs[lc.final_state](lc.error or lc.final_state.replace("_", " "))
        if lc.result is None:
            raise RuntimeError("worker lifecycle completed without a result")
        return lc.result

    def submit_report_cleanup_lifecycle(self, request: WorkerTransferAuthorizationRequest,
                                        cleanup_target_kind: str = "reservation") -> WorkerTransferLifecycleRecord:
        kind = cleanup_target_kind
        try:
            wr = self.authorize(request)
        except WorkerAuthorizationError as exc:
            tgt = cleanup_target(kind, request.lease_id, request.session_id)
            try:
                cr = self.cleanup_coordinator.cleanup_authorization_failure(request, target_kind=kind)
            except WorkerCleanupError as cexc:
                return WorkerTransferLifecycleRecord(request, cleanup_target_kind=kind, cleanup_target_id=tgt,
                                                     final_state="cleanup_failed", error=str(cexc))
            return WorkerTransferLifecycleRecord(request, cleanup_target_kind=kind, cleanup_target_id=tgt,
                                                 cleanup_response=cr, final_state="authorization_failed",
                                                 error=str(exc))
        a = wr.authorization
        slot = self.staging_pool.allocate(wr.data_plane)
        result = self._run(wr, slot)
        update = status_update_for(result)
        common = dict(authorization_request=request, worker_request=wr, staging_slot=slot, result=result,
                      status_update=update, cleanup_target_kind=kind)
        try:
            sr = self.status_reporter.report(result)
        except WorkerStatusReportError as exc:
            rel = self.staging_pool.release(slot.slot_id, wr.data_plane)
            tgt = cleanup_target(kind, a.lease_id, a.session_id)
            try:
                cr = self.cleanup_coordinator.cleanup_status_report_failure(wr, target_kind=kind)
            except WorkerCleanupError as cexc:
                return WorkerTransferLifecycleRecord(**common, staging_release=rel, cleanup_target_id=tgt,
                                                     final_state="cleanup_failed", error=str(cexc))
            return WorkerTransferLifecycleRecord(**common, staging_release=rel, cleanup_target_id=tgt,
                                                 cleanup_response=cr, final_state="status_failed", error=str(exc))
        tgt = a.lease_id if result.state is WorkerTransferState.COMPLETE else cleanup_target(kind, a.lease_id,
                                                                                             a.session_id)
        try:
            cr = self.cleanup_coordinator.cleanup_execution_failure(wr, result, target_kind=kind)
        except WorkerCleanupError as exc:
            rel = self.staging_pool.release(slot.slot_id, wr.data_plane)
            return WorkerTransferLifecycleRecord(**common, staging_release=rel, status_response=sr,
                                                 cleanup_target_id=tgt, final_state="cleanup_failed",
                                                 error=str(exc))
        rel = self.staging_pool.release(slot.slot_id, wr.data_plane)
        return WorkerTransferLifecycleRecord(**common, staging_release=rel, status_response=sr,
                                             cleanup_target_id=tgt, cleanup_response=cr,
                                             final_state=result.state.value, error=result.error)


class WorkerTransferService:
    """Envelope-level entry point of the worker helper."""

    def __init__(self, daemon_client=None, transfer_client: WorkerTransferClient | None = None, **client_kw) -> None:
        if transfer_client is None:
            if daemon_client is None:
                raise ValueError("daemon_client or transfer_client is required")
            transfer_client = WorkerTransferClient(daemon_client, **client_kw)
        self.transfer_client = transfer_client

    def handle_lifecycle(self, request: WorkerTransferAuthorizationRequest,
                         cleanup_target_kind: str = "reservation") -> WorkerTransferLifecycleRecord:
        if not isinstance(request, WorkerTransferAuthorizationRequest):
            raise TypeError("request must be a WorkerTransferAuthorizationRequest")
        return self.transfer_client.submit_report_cleanup_lifecycle(request, cleanup_target_kind=cleanup_target_kind)

    def parse_authorization_request(self, payload: Mapping[str, object]) -> WorkerTransferAuthorizationRequest:
        return parse_worker_authorization_request_payload(payload)

    def handle_envelope(self, envelope) -> WorkerServiceResponseEnvelope:
        try:
            env = envelope if isinstance(envelope, WorkerServiceRequestEnvelope) else WorkerServiceRequestEnvelope(
                **dict(envelope))
            req = self.parse_authorization_request(env.payload)
            return WorkerServiceResponseEnvelope.from_lifecycle(
                self.handle_lifecycle(req, cleanup_target_kind=env.cleanup_target_kind))
        except Exception as exc:  # noqa: BLE001 - every failure becomes an error envelope
            return WorkerServiceResponseEnvelope.from_error(str(exc))

    def handle_envelope_payload(self, envelope: Mapping[str, object]) -> dict[str, object]:
        return self.handle_envelope(envelope).as_dict()


def parse_worker_authorization_request_payload(payload: Mapping[str, object]) -> WorkerTransferAuthorizationRequest:
    if not isinstance(payload, Mapping):
        raise ValueError("worker authorization payload must be a mapping")
    body = payload.get("authorization", payload)
    if not isinstance(body, Mapping):
        raise ValueError("worker authorization payload must be a mapping")
    try:
        return WorkerTransferAuthorizationRequest(
            transfer_id=body["transfer_id"], lease_id=body["lease_id"], token=body["token"],
            session_id=body["session_id"], job_id=body["job_id"], src_buffer_id=body["src_buffer_id"],
            dst_buffer_id=body["dst_buffer_id"], direction=body["direction"],
            ranges=tuple(body.get("ranges", ()) or ()), relay_gpu=body.get("relay_gpu"))
    except KeyError as exc:
        raise ValueError(f"missing worker authorization field: {exc.args[0]}") from exc


__all__ = [
    "TICKET_ISSUER", "WorkerAuthorizationError", "WorkerCleanupError", "WorkerDataPlaneCompletion",
    "WorkerDataPlaneCompletionEnvelope", "WorkerDataPlaneRequest", "WorkerServiceRequestEnvelope",
    "WorkerServiceResponseEnvelope", "WorkerStatusReportError", "WorkerTransferAuthorizer",
    "WorkerTransferCleanupCoordinator", "WorkerTransferClient", "WorkerTransferLifecycleRecord",
    "WorkerTransferRequest", "WorkerTransferResult", "WorkerTransferService", "WorkerTransferState",
    "WorkerTransferStatusReporter", "check_completion_bytes", "parse_worker_authorization_request_payload",
    "plan_total_bytes", "relay_ranges_for", "require_daemon_worker_plan", "status_update_for",
    "validate_daemon_ticket",
]
