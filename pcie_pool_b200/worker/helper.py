"""Worker helper: the life of one daemon-ticketed transfer inside a worker.

::

    authorize ──► plan check ──► staging slot ──► bind + run the plan ──► byte check
        │                                                                     │
        ▼                                                                     ▼
    cleanup ◄──────────────────── cleanup / release ◄──────────────── status report
    (authorization_failed)        (complete | failed | cleanup_failed)    (status_failed)

    the staging slot is released on every path that took one

What is contract, kept so that TurboBus workers, daemons and logs interoperate
(turbobus/worker/helper.py): the public class and function names, the ticket
rules (issuer ``turbobus-daemon``, a positive and current plan generation, a
transfer id; the ticket agrees with its decision, buffers, relays, leases and
ranges), the completed-bytes rule, the cleanup targets (a reservation or the
session), the lifecycle's ``final_state`` values and the envelope fields.

How it is built here:

* ``TicketPlan`` reads a daemon plan once into lanes (kind, relay, direction,
  target, enabled, chunks); every later question (the relays, a relay's
  chunks, the total) is answered from that view.
* Agreement checks are tables of ``(what, got, want)`` rows run by
  ``_agree``; each message names what disagreed.
* ``_Lifecycle`` is a step machine: each step returns the next step or a
  final state, and the record is assembled once at the end.  The staging slot
  is released by the machine itself, whatever step ended the run.
* ``cleanup_calls`` turns an outcome into the list of daemon calls a cleanup
  needs (release per lease after success, cleanup per lease or of the session
  after failure); the coordinator only executes that list.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import asdict, dataclass, field
from enum import Enum
from typing import Any, Callable, Iterable

from ..planner_types import assignment_chunks
from ..schema import (BufferRegistration, DaemonResponse, ExecutionTicket, SchedulingDecision,
                      TransferStatusState, WorkerDataPlaneCompletion, WorkerDataPlaneRequest,
                      WorkerTransferAuthorization, WorkerTransferAuthorizationRequest)
from .resources import WorkerDataPlaneResourceBinder, WorkerDataPlaneResourceError
from .staging_pool import WorkerStagingPool, WorkerStagingSlot

TICKET_ISSUER = "turbobus-daemon"
CLEANUP_KINDS = ("reservation", "session")


class WorkerTransferState(str, Enum):
    FAILED = "failed"
    COMPLETE = "complete"


class WorkerAuthorizationError(RuntimeError):
    """The daemon refused the transfer, or its answer failed a check."""


class WorkerStatusReportError(RuntimeError):
    """The daemon refused the worker's status report."""


class WorkerCleanupError(RuntimeError):
    """A release or cleanup call was refused (every failing lease is named)."""


# ---- the plan, read once ----------------------------------------------------------------------------

@dataclass(frozen=True)
class PlanLane:
    kind: str
    relay: int
    direction: str
    target: int | None
    enabled: bool
    chunks: tuple[dict, ...]

    @property
    def bytes(self) -> int:
        return sum(c["bytes"] for c in self.chunks)


class TicketPlan:
    """A daemon plan (``{"assignments": [{"path": ..., "chunks"|"runs": ...}]}``)
    as a list of ``PlanLane``; malformed assignments raise ``ValueError``."""

    def __init__(self, plan: Mapping[str, Any]) -> None:
        if not isinstance(plan, Mapping):
            raise ValueError("a daemon plan must be a mapping")
        lanes = []
        for a in plan.get("assignments", ()) or ():
            path = a.get("path") if isinstance(a, Mapping) else None
            if not isinstance(path, Mapping):
                raise ValueError("each daemon plan assignment must be a mapping with a path mapping")
            try:
                raw = assignment_chunks(a)
            except ValueError as exc:
                raise ValueError(f"daemon plan chunk is malformed: {exc}") from None
            chunks = tuple({"src_offset": int(c["src_offset"]), "dst_offset": int(c["dst_offset"]),
                            "bytes": int(c["bytes"])} for c in raw)
            tgt = path.get("target_device")
            lanes.append(PlanLane(kind=str(path.get("kind", "")).lower(), relay=int(path.get("relay_device", -1)),
                                  direction=str(path.get("direction", "")).lower(),
                                  target=None if tgt is None else int(tgt),
                                  enabled=bool(path.get("enabled", True)), chunks=chunks))
        self.lanes: tuple[PlanLane, ...] = tuple(lanes)
        self.declared_total = plan.get("total_bytes")

    @property
    def relays(self) -> tuple[int, ...]:
        """Relay devices in plan order, each once."""
        return tuple(dict.fromkeys(l.relay for l in self.lanes if l.kind == "relay"))

    @property
    def total(self) -> int:
        return sum(l.bytes for l in self.lanes)

    def relay_chunks(self, relays: Iterable[int], direction: str | None = None) -> tuple[dict, ...]:
        """The chunks of the relay lanes of ``relays``, in plan order; with
        ``direction``, a relay lane of another direction raises."""
        want = {int(r) for r in relays}
        out = []
        for l in self.lanes:
            if l.kind != "relay" or l.relay not in want:
                continue
            if direction is not None and l.direction != direction:
                raise ValueError(f"relay {l.relay}'s lane direction {l.direction or '?'} differs from the "
                                 f"ticket's {direction}")
            out.extend(l.chunks)
        return tuple(out)


def planned_relays(plan: Mapping[str, Any]) -> tuple[int, ...]:
    return TicketPlan(plan).relays


def plan_total_bytes(plan: Mapping[str, Any]) -> int:
    return TicketPlan(plan).total


def relay_ranges_for(ticket: ExecutionTicket, relays: Iterable[int]) -> tuple[dict[str, int], ...]:
    """The byte ranges ``relays`` carry under ``ticket``'s plan."""
    relays = tuple(relays)
    if not relays:
        raise ValueError("relay_gpus is empty: a ticket's relay ranges need at least one relay")
    out = TicketPlan(ticket.plan).relay_chunks(relays, ticket.direction)
    if not out:
        raise ValueError(f"the ticket's plan gives relays {list(relays)} no chunks")
    if sum(r["bytes"] for r in out) > ticket.total_bytes:
        raise ValueError("the ticket's relay ranges add up to more than its total bytes")
    return out


# ---- agreement checks -------------------------------------------------------------------------------

def _agree(rows: Iterable[tuple[str, object, object]], template: str) -> None:
    """Raise ``ValueError(template.format(what))`` for the first row whose
    ``got`` differs from ``want``."""
    for what, got, want in rows:
        if got != want:
            raise ValueError(template.format(what))


def validate_daemon_ticket(ticket: ExecutionTicket, plan_generation: object | None = None) -> None:
    """A ticket the worker may act on: issued by the daemon, for a transfer,
    at a positive plan generation that is the current one when given."""
    if not isinstance(ticket, ExecutionTicket):
        raise TypeError(f"validate_daemon_ticket needs an ExecutionTicket, got {type(ticket).__name__}")
    md = ticket.metadata
    if md.get("issuer") != TICKET_ISSUER:
        raise ValueError(f"ticket was not issued by {TICKET_ISSUER} (issuer {md.get('issuer')!r})")
    gen = md.get("plan_generation")
    if gen is None:
        raise ValueError("ticket has no plan_generation")
    if int(gen) <= 0:
        raise ValueError(f"ticket plan_generation must be a positive integer, not {gen}")
    if plan_generation is not None and int(plan_generation) != int(gen):
        raise ValueError(f"ticket plan_generation {gen} is stale: the daemon is at {plan_generation}")
    if not str(md.get("transfer_id") or "").strip():
        raise ValueError("ticket names no transfer_id")


def _check_buffers(ticket: ExecutionTicket, src: BufferRegistration, dst: BufferRegistration) -> None:
    if not isinstance(src, BufferRegistration) or not isinstance(dst, BufferRegistration):
        raise TypeError("src_buffer and dst_buffer must be BufferRegistration records")
    _agree((("source buffer", src.buffer_id, ticket.source_buffer_id),
            ("destination buffer", dst.buffer_id, ticket.destination_buffer_id),
            ("source buffer's job", src.job_id, ticket.job_id),
            ("destination buffer's job", dst.job_id, ticket.job_id)), "ticket {} differs from the worker's")


def _check_decision(ticket: ExecutionTicket, d: SchedulingDecision) -> None:
    rows = [(a, getattr(ticket, a), getattr(d, a))
            for a in ("decision_id", "intent_id", "topology_snapshot_id", "job_id", "session_id")]
    rows.append(("plan", dict(ticket.plan), dict(d.plan)))
    dg = (getattr(d, "metadata", None) or {}).get("plan_generation")
    if dg is not None:
        rows.append(("plan_generation", int(ticket.metadata.get("plan_generation", 0)), int(dg)))
    _agree(rows, "ticket {} differs from the scheduling decision")


def _pick(requested_many, requested_one, available: tuple, label: str, cast: Callable) -> tuple:
    """The subset of ``available`` a payload asks for (``label`` + ``s`` and
    ``label``), defaulting to all of it."""
    chosen = None
    if requested_many is not None:
        chosen = tuple(cast(x) for x in requested_many)
        if not chosen or any(not str(x).strip() for x in chosen):
            raise ValueError(f"{label}s is empty or holds a blank entry")
    if requested_one is not None:
        one = cast(requested_one)
        if chosen is None:
            chosen = (one,)
        elif one not in chosen:
            raise ValueError(f"{label} {one!r} is not one of the requested {label}s")
    if chosen is None:
        return available
    extra = set(chosen) - set(available)
    if extra:
        raise ValueError(f"{label}s {sorted(extra)} are not in the daemon plan's ticket")
    return chosen


def _buffer(payload) -> BufferRegistration:
    if not isinstance(payload, Mapping):
        raise ValueError("a buffer record must be a mapping")
    return BufferRegistration(**{k: payload[k] for k in ("buffer_id", "job_id", "kind", "size_bytes")},
                              device_index=payload.get("device_index"), address=payload.get("address"),
                              pinned=bool(payload.get("pinned", False)),
                              handle_type=payload.get("handle_type", "registered_buffer"),
                              metadata=dict(payload.get("metadata") or {}))


# ---- the ticketed request -----------------------------------------------------------------------------

@dataclass(frozen=True)
class WorkerTransferRequest:
    """A daemon ticket turned into what the worker executes: the
    authorization (primary relay and lease) and the data-plane request (all
    relays and leases the worker serves, their ranges by relay)."""

    authorization: WorkerTransferAuthorization
    ticket: ExecutionTicket
    data_plane: WorkerDataPlaneRequest | None = None

    @classmethod
    def from_authorization_payload(cls, payload: Mapping[str, object]) -> "WorkerTransferRequest":
        if not isinstance(payload, Mapping):
            raise ValueError("the daemon's authorization answer is not a mapping")
        if payload.get("ticket") is None:
            raise ValueError("the daemon's authorization answer carries no execution ticket")
        return cls.from_execution_ticket_payload(payload)

    @classmethod
    def from_execution_ticket_payload(cls, payload: Mapping[str, object]) -> "WorkerTransferRequest":
        if not isinstance(payload, Mapping) or not isinstance(payload.get("ticket"), Mapping):
            raise ValueError("an execution ticket payload needs a ticket mapping")
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
        raise ValueError("a worker request is built from the daemon's ExecutionTicket, not from a bare authorization")

    @classmethod
    def from_execution_ticket(cls, ticket: ExecutionTicket, *, src_buffer: BufferRegistration,
                              dst_buffer: BufferRegistration, relay_gpu: int | None = None,
                              relay_gpus: Iterable[int] | None = None, lease_id: str | None = None,
                              lease_ids: Iterable[str] | None = None, transfer_id: str | None = None,
                              decision: SchedulingDecision | None = None,
                              plan_generation: object | None = None) -> "WorkerTransferRequest":
        _check_buffers(ticket, src_buffer, dst_buffer)
        validate_daemon_ticket(ticket, plan_generation)
        if decision is not None:
            _check_decision(ticket, decision)
        plan = TicketPlan(ticket.plan)
        if not plan.relays:
            raise ValueError("the daemon plan has no relay lane for a worker to serve")
        relays = _pick(relay_gpus, relay_gpu, plan.relays, "relay_gpu", int)
        if not ticket.lease_ids:
            raise ValueError("the ticket holds no lease id")
        leases = _pick(lease_ids, lease_id, tuple(ticket.lease_ids), "lease_id", str)
        primary = int(relay_gpu) if relay_gpu is not None else relays[0]
        primary_lease = str(lease_id) if lease_id is not None else leases[0]
        tid = str(transfer_id if transfer_id is not None else ticket.metadata.get("transfer_id") or ticket.ticket_id)
        auth = WorkerTransferAuthorization(
            transfer_id=tid, lease_id=primary_lease, session_id=ticket.session_id, job_id=ticket.job_id,
            src_buffer=src_buffer, dst_buffer=dst_buffer, direction=ticket.direction,
            ranges=relay_ranges_for(ticket, relays), relay_gpu=primary, plan=dict(ticket.plan))
        by_relay = {str(r): relay_ranges_for(ticket, (r,)) for r in relays}
        dp = WorkerDataPlaneRequest.from_authorization(auth, metadata={
            "relay_gpus": relays, "lease_ids": leases, "primary_relay_gpu": primary,
            "primary_lease_id": primary_lease, "relay_ranges_by_gpu": by_relay})
        return cls(authorization=auth, ticket=ticket, data_plane=dp)

    def __post_init__(self) -> None:
        a = self.authorization
        if not isinstance(a, WorkerTransferAuthorization):
            raise TypeError("authorization must be a WorkerTransferAuthorization")
        dp = self.data_plane if self.data_plane is not None else WorkerDataPlaneRequest.from_authorization(a)
        if not isinstance(dp, WorkerDataPlaneRequest):
            raise TypeError("data_plane must be a WorkerDataPlaneRequest")
        _agree((("transfer_id", dp.transfer_id, a.transfer_id), ("lease_id", dp.lease_id, a.lease_id),
                ("session_id", dp.session_id, a.session_id), ("job_id", dp.job_id, a.job_id),
                ("relay", dp.relay_gpu, a.relay_gpu), ("direction", dp.direction, a.direction),
                ("src handle", dp.src_handle.buffer_id, a.src_buffer.buffer_id),
                ("dst handle", dp.dst_handle.buffer_id, a.dst_buffer.buffer_id),
                ("ranges", dp.ranges, a.ranges), ("plan", dp.plan, a.plan)),
               "data-plane request's {} disagrees with the authorization")
        t = self.ticket
        if not isinstance(t, ExecutionTicket):
            raise TypeError("ticket must be an ExecutionTicket")
        validate_daemon_ticket(t)
        _agree((("job", t.job_id, a.job_id), ("session", t.session_id, a.session_id),
                ("source buffer", t.source_buffer_id, a.src_buffer.buffer_id),
                ("destination buffer", t.destination_buffer_id, a.dst_buffer.buffer_id),
                ("direction", t.direction, a.direction), ("plan", dict(t.plan), a.plan)),
               "ticket's {} disagrees with the authorization")
        relays = tuple(int(r) for r in dp.metadata.get("relay_gpus", (a.relay_gpu,)))
        if a.relay_gpu not in relays:
            raise ValueError(f"authorized relay {a.relay_gpu} is not among the request's relays {list(relays)}")
        if relay_ranges_for(t, relays) != a.ranges:
            raise ValueError("ticket's relay ranges disagree with the authorization")
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
            raise ValueError("the request holds no lease id")
        if self.authorization.lease_id not in ids:
            raise ValueError(f"primary lease {self.authorization.lease_id!r} is not one of the request's leases")
        return ids

    def as_dict(self) -> dict[str, object]:
        return {"authorization": asdict(self.authorization), "data_plane": asdict(self.data_plane),
                "ticket": asdict(self.ticket)}


def require_daemon_worker_plan(request: WorkerTransferRequest) -> None:
    """Checks of the ticketed plan before a staging slot is taken: lanes are
    direct or relay, of the request's direction, target and relays, enabled,
    add up to the declared total, and the relay chunks are the authorized
    ranges."""
    dp = request.data_plane
    if not dp.plan or not list(dp.plan.get("assignments", ()) or ()):
        raise ValueError("the authorization carries no relay path: its plan has no assignments")
    target_h = dp.dst_handle if dp.direction == "h2d" else dp.src_handle
    if target_h.device_index is None:
        raise ValueError("the worker's target handle has no CUDA device index")
    target = int(target_h.device_index)
    plan = TicketPlan(dp.plan)
    allowed = set(request.relay_gpus)
    for lane in plan.lanes:
        if lane.kind not in ("direct", "relay"):
            raise ValueError(f"daemon plan lane of kind {lane.kind!r}: only direct and relay lanes exist")
        if lane.direction != dp.direction:
            raise ValueError(f"daemon plan lane direction {lane.direction or '?'} differs from the "
                             f"request's {dp.direction}")
        if lane.target is not None and lane.target != target:
            raise ValueError(f"daemon plan lane targets GPU {lane.target}, the worker's handle GPU {target}")
        if not lane.enabled:
            raise ValueError("daemon plan lane is disabled")
        if lane.kind == "relay" and lane.relay not in allowed:
            raise ValueError(f"daemon plan relay {lane.relay} is not authorized by the ticket")
    total = plan.total
    if total <= 0:
        raise ValueError("daemon plan assigns no bytes")
    if int(plan.declared_total if plan.declared_total is not None else total) != total:
        raise ValueError(f"daemon plan total_bytes {plan.declared_total} is not the sum of its chunks ({total})")
    relay_chunks = plan.relay_chunks(allowed)
    if not relay_chunks:
        raise ValueError("daemon plan gives the authorized relays no chunks")
    if relay_chunks != dp.ranges:
        raise ValueError("authorized ranges are not the plan's relay chunks")


# ---- results --------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class WorkerTransferResult:
    transfer_id: str
    state: WorkerTransferState
    error: str | None = None
    bytes_completed: int = 0
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not str(self.transfer_id).strip():
            raise ValueError("a result needs a transfer_id")
        if int(self.bytes_completed) < 0:
            raise ValueError("bytes_completed cannot be negative")
        object.__setattr__(self, "transfer_id", str(self.transfer_id))
        object.__setattr__(self, "state", WorkerTransferState(self.state))
        object.__setattr__(self, "bytes_completed", int(self.bytes_completed))
        object.__setattr__(self, "error", None if self.error is None else str(self.error))
        object.__setattr__(self, "metadata", dict(self.metadata))

    @property
    def complete(self) -> bool:
        return self.state is WorkerTransferState.COMPLETE

    def as_dict(self) -> dict[str, object]:
        return {"transfer_id": self.transfer_id, "state": self.state.value, "error": self.error,
                "bytes_completed": self.bytes_completed, "metadata": dict(self.metadata)}

    def data_plane_completion(self, lease_id: str) -> WorkerDataPlaneCompletion:
        u = status_update_for(self)
        return WorkerDataPlaneCompletion(transfer_id=self.transfer_id, lease_id=lease_id, state=u["state"],
                                         bytes_completed=self.bytes_completed,
                                         error=None if self.complete else u["error"], metadata=dict(self.metadata))


def status_update_for(result: WorkerTransferResult) -> dict[str, object]:
    """The daemon status report of a result (a failure always has an error)."""
    if result.complete:
        return {"transfer_id": result.transfer_id, "state": TransferStatusState.COMPLETE.value,
                "bytes_completed": result.bytes_completed, "error": result.error}
    return {"transfer_id": result.transfer_id, "state": TransferStatusState.FAILED.value,
            "bytes_completed": result.bytes_completed, "error": result.error or "worker transfer failed"}


def failed_result(request: WorkerTransferRequest, slot: WorkerStagingSlot | None, error: str) -> WorkerTransferResult:
    md: dict[str, object] = {"executor": "worker", "relay_gpu": request.data_plane.relay_gpu}
    if slot is not None:
        md["staging_slot_id"] = slot.slot_id
    return WorkerTransferResult(request.transfer_id, WorkerTransferState.FAILED, error=error, metadata=md)


_failed = failed_result


def check_completion_bytes(request: WorkerTransferRequest, result: WorkerTransferResult) -> WorkerTransferResult:
    """A complete result must have moved exactly the plan's bytes; otherwise
    it becomes a failed one."""
    if not result.complete:
        return result
    want = plan_total_bytes(request.data_plane.plan)
    if want <= 0:
        raise ValueError("the worker's plan has no bytes to complete")
    if result.bytes_completed == want:
        return result
    return WorkerTransferResult(result.transfer_id, WorkerTransferState.FAILED,
                                error=f"executor reported {result.bytes_completed} bytes, the plan moves {want}",
                                bytes_completed=result.bytes_completed, metadata=result.metadata)


# ---- cleanup as data ------------------------------------------------------------------------------------

def cleanup_target(kind: str, lease_id: str, session_id: str) -> str:
    k = str(kind).lower()
    if k not in CLEANUP_KINDS:
        raise ValueError(f"cleanup target kind {kind!r}: it must be reservation or session")
    return str(lease_id) if k == "reservation" else str(session_id)


@dataclass(frozen=True)
class DaemonCall:
    """One release (``target_kind`` None) or cleanup the daemon is asked for."""

    target_id: str
    target_kind: str | None = None
    reason: str = ""
    force: bool = True


def cleanup_calls(leases: tuple[str, ...], session_id: str, kind: str, reason: str, force: bool,
                  release: bool) -> list[DaemonCall]:
    """The daemon calls that end a transfer: a release per lease after
    success; otherwise a cleanup per lease, or one of the session."""
    cleanup_target(kind, leases[0] if leases else "", session_id)  # validates the kind
    if release:
        return [DaemonCall(lid) for lid in leases]
    if kind == "session":
        return [DaemonCall(str(session_id), "session", reason, force)]
    return [DaemonCall(lid, "reservation", reason, force) for lid in leases]


# ---- lifecycle record and envelopes ---------------------------------------------------------------------

def _opt_str(obj, *names: str) -> None:
    for n in names:
        v = getattr(obj, n)
        if v is not None:
            object.__setattr__(obj, n, str(v))


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

    _TYPES = {"worker_request": WorkerTransferRequest, "staging_slot": WorkerStagingSlot,
              "staging_release": WorkerStagingSlot, "result": WorkerTransferResult,
              "status_response": DaemonResponse, "cleanup_response": DaemonResponse}

    def __post_init__(self) -> None:
        if not isinstance(self.authorization_request, WorkerTransferAuthorizationRequest):
            raise TypeError("authorization_request must be a WorkerTransferAuthorizationRequest")
        for name, typ in self._TYPES.items():
            v = getattr(self, name)
            if v is not None and not isinstance(v, typ):
                raise TypeError(f"{name} must be a {typ.__name__} or None")
        if self.status_update is not None:
            if not isinstance(self.status_update, Mapping):
                raise TypeError("status_update must be a mapping")
            object.__setattr__(self, "status_update", dict(self.status_update))
        if not str(self.final_state).strip():
            raise ValueError("final_state cannot be blank")
        _opt_str(self, "final_state", "cleanup_target_kind", "cleanup_target_id", "error")

    @property
    def lease_ids(self) -> tuple[str, ...]:
        if self.worker_request is not None:
            return self.worker_request.lease_ids
        return (self.authorization_request.lease_id,)

    @property
    def transfer_id(self) -> str:
        src = self.worker_request or self.authorization_request
        return src.transfer_id

    @property
    def lease_id(self) -> str:
        if self.worker_request is not None:
            return self.worker_request.authorization.lease_id
        return self.authorization_request.lease_id

    def as_dict(self) -> dict[str, object]:
        def d(x):
            return None if x is None else (x.as_dict() if hasattr(x, "as_dict") else asdict(x))

        tgt = None
        if self.cleanup_target_kind is not None or self.cleanup_target_id is not None:
            tgt = {"target_kind": self.cleanup_target_kind, "target_id": self.cleanup_target_id}
        return {"authorization_request": asdict(self.authorization_request),
                "worker_request": d(self.worker_request), "staging_slot": d(self.staging_slot),
                "staging_release": d(self.staging_release), "result": d(self.result),
                "status_update": None if self.status_update is None else dict(self.status_update),
                "status_response": d(self.status_response), "cleanup_target": tgt,
                "cleanup_response": d(self.cleanup_response), "lease_ids": self.lease_ids,
                "final_state": self.final_state, "error": self.error}

    def completion_envelope(self) -> "WorkerDataPlaneCompletionEnvelope":
        return WorkerDataPlaneCompletionEnvelope.from_lifecycle(self)


# record field -> completion-envelope field
_ENVELOPE_FROM_RECORD = {"staging_slot": "staging_slot", "result": "worker_result",
                         "status_update": "daemon_status_update", "status_response": "daemon_status_response",
                         "cleanup_response": "daemon_cleanup_response", "staging_release": "staging_release"}
_MAPPING_FIELDS = tuple(_ENVELOPE_FROM_RECORD.values())


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
            if v is not None and not isinstance(v, Mapping):
                raise TypeError(f"{name} must be a mapping or None")
            if v is not None:
                object.__setattr__(self, name, dict(v))
        _opt_str(self, "transfer_id", "lease_id", "final_state", "error")
        object.__setattr__(self, "lease_ids", tuple(str(x) for x in self.lease_ids))
        if self.lease_ids and self.lease_id is not None and self.lease_id not in self.lease_ids:
            raise ValueError(f"lease_id {self.lease_id!r} is not in lease_ids")

    @classmethod
    def from_lifecycle(cls, lifecycle: WorkerTransferLifecycleRecord) -> "WorkerDataPlaneCompletionEnvelope":
        if not isinstance(lifecycle, WorkerTransferLifecycleRecord):
            raise TypeError("lifecycle must be a WorkerTransferLifecycleRecord")
        rec = lifecycle.as_dict()
        return cls(ok=True, transfer_id=lifecycle.transfer_id, lease_id=lifecycle.lease_id,
                   lease_ids=lifecycle.lease_ids, final_state=lifecycle.final_state, error=lifecycle.error,
                   **{env: rec[src] for src, env in _ENVELOPE_FROM_RECORD.items()})

    def as_dict(self) -> dict[str, object]:
        out: dict[str, object] = {"ok": self.ok, "transfer_id": self.transfer_id, "lease_id": self.lease_id,
                                  "lease_ids": self.lease_ids, "final_state": self.final_state, "error": self.error}
        out.update({n: None if getattr(self, n) is None else dict(getattr(self, n)) for n in _MAPPING_FIELDS})
        return out


@dataclass(frozen=True)
class WorkerServiceRequestEnvelope:
    payload: Mapping[str, object]
    cleanup_target_kind: str = "reservation"

    def __post_init__(self) -> None:
        if not isinstance(self.payload, Mapping):
            raise ValueError("the worker service payload must be a mapping")
        k = str(self.cleanup_target_kind)
        if k not in CLEANUP_KINDS:
            raise ValueError(f"cleanup_target_kind {k!r}: it must be reservation or session")
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
            raise TypeError("completion must be a mapping or None")
        object.__setattr__(self, "ok", bool(self.ok))
        if self.completion is not None:
            object.__setattr__(self, "completion", dict(self.completion))
        _opt_str(self, "error", "final_state")

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


# ---- daemon-facing steps ------------------------------------------------------------------------------

class WorkerTransferAuthorizer:
    """Asks the daemon for the ticket and checks it into a request."""

    def __init__(self, daemon_client) -> None:
        self.daemon_client = daemon_client

    def authorize(self, request: WorkerTransferAuthorizationRequest) -> WorkerTransferRequest:
        resp: DaemonResponse = self.daemon_client.authorize_worker_transfer(request)
        if not resp.ok:
            raise WorkerAuthorizationError(resp.error or "the daemon refused the worker transfer")
        try:
            wr = WorkerTransferRequest.from_authorization_payload(resp.payload)
            require_daemon_worker_plan(wr)
        except (KeyError, TypeError, ValueError) as exc:
            raise WorkerAuthorizationError(f"the daemon's authorization failed a check: {exc}") from exc
        return wr


class WorkerTransferStatusReporter:
    def __init__(self, daemon_client) -> None:
        self.daemon_client = daemon_client

    def report(self, result: WorkerTransferResult) -> DaemonResponse:
        if not isinstance(result, WorkerTransferResult):
            raise TypeError("report() takes a WorkerTransferResult")
        u = status_update_for(result)
        resp: DaemonResponse = self.daemon_client.transfer_status(u["transfer_id"], state=u["state"],
                                                                  bytes_completed=u["bytes_completed"],
                                                                  error=u["error"])
        if not resp.ok:
            raise WorkerStatusReportError(resp.error or "the daemon refused the status report")
        return resp


class WorkerTransferCleanupCoordinator:
    """Runs ``cleanup_calls``: one daemon call per entry, every entry tried,
    every refusal named in one ``WorkerCleanupError``."""

    def __init__(self, daemon_client) -> None:
        self.daemon_client = daemon_client

    def cleanup_authorization_failure(self, request: WorkerTransferAuthorizationRequest,
                                      target_kind: str = "reservation",
                                      reason: str = "worker_authorization_failed",
                                      force: bool = True) -> DaemonResponse:
        if not isinstance(request, WorkerTransferAuthorizationRequest):
            raise TypeError("request must be a WorkerTransferAuthorizationRequest")
        target = cleanup_target(target_kind, request.lease_id, request.session_id)
        return self._run([DaemonCall(target, str(target_kind).lower(), reason, force)], single=True)

    def cleanup_execution_failure(self, request: WorkerTransferRequest, result: WorkerTransferResult,
                                  target_kind: str = "reservation", reason: str | None = None,
                                  force: bool = True) -> DaemonResponse:
        if not isinstance(request, WorkerTransferRequest) or not isinstance(result, WorkerTransferResult):
            raise TypeError("cleanup_execution_failure takes a WorkerTransferRequest and a WorkerTransferResult")
        release = result.complete and target_kind != "session"
        reason = reason or f"worker_{result.state.value}"
        calls = cleanup_calls(request.lease_ids, request.authorization.session_id, target_kind, reason, force,
                              release=release)
        return self._run(calls, single=len(calls) == 1)

    def cleanup_status_report_failure(self, request: WorkerTransferRequest, target_kind: str = "reservation",
                                      reason: str = "worker_status_report_failed",
                                      force: bool = True) -> DaemonResponse:
        if not isinstance(request, WorkerTransferRequest):
            raise TypeError("request must be a WorkerTransferRequest")
        calls = cleanup_calls(request.lease_ids, request.authorization.session_id, target_kind, reason, force,
                              release=False)
        return self._run(calls, single=len(calls) == 1)

    def _call(self, c: DaemonCall) -> DaemonResponse:
        if c.target_kind is None:
            fn = getattr(self.daemon_client, "release_transfer", None)
            if not callable(fn):
                raise WorkerCleanupError("this daemon client cannot release a completed transfer")
            return fn(c.target_id)
        fn = getattr(self.daemon_client, "cleanup", None)
        if not callable(fn):
            raise WorkerCleanupError("this daemon client cannot clean up a transfer")
        return fn(target_kind=c.target_kind, target_id=c.target_id, reason=c.reason, force=c.force)

    def _run(self, calls: list[DaemonCall], single: bool) -> DaemonResponse:
        if single:
            resp = self._call(calls[0])
            if not resp.ok:
                what = "release" if calls[0].target_kind is None else "cleanup"
                raise WorkerCleanupError(resp.error or f"the daemon refused the {what}")
            return resp
        responses, done, refused = [], [], []
        for c in calls:
            resp = self._call(c)
            responses.append(asdict(resp))
            if resp.ok:
                pl = resp.payload if isinstance(resp.payload, Mapping) else {}
                done.append(str(pl.get("reservation_id", c.target_id)))
            else:
                refused.append(f"{c.target_id}: {resp.error or 'refused'}")
        if refused:
            raise WorkerCleanupError("; ".join(refused))
        release = calls[0].target_kind is None
        leases = tuple(c.target_id for c in calls)
        return DaemonResponse(ok=True, payload={
            "reservation_id": leases[0], "lease_ids": leases, "released_reservation_ids": tuple(done),
            "lease_responses": tuple(responses), "cleanup_kind": calls[0].target_kind or "reservation",
            "reason": calls[0].reason or "worker_complete", "cleanup_mode": "release" if release else "cleanup"})


# ---- the lifecycle machine ------------------------------------------------------------------------------

def _default_executor():
    from .cuda_executor import CudaWorkerExecutor

    return CudaWorkerExecutor()


class _Lifecycle:
    """One run of ``submit_report_cleanup_lifecycle``.  Steps are methods
    returning the next step, or None once ``final`` is set; the record is
    built from the attributes collected on the way."""

    def __init__(self, client: "WorkerTransferClient", request: WorkerTransferAuthorizationRequest,
                 kind: str) -> None:
        self.c, self.request, self.kind = client, request, kind
        self.wr: WorkerTransferRequest | None = None
        self.slot = self.release = self.result = None
        self.update = self.status = self.cleanup = None
        self.target_id: str | None = None
        self.final, self.error = "created", None

    def run(self) -> WorkerTransferLifecycleRecord:
        step = self.authorize
        try:
            while step is not None:
                step = step()
        finally:
            if self.slot is not None and self.release is None:
                self.release = self.c.staging_pool.release(self.slot.slot_id, self.wr.data_plane)
        return WorkerTransferLifecycleRecord(
            self.request, worker_request=self.wr, staging_slot=self.slot, staging_release=self.release,
            result=self.result, status_update=self.update, status_response=self.status,
            cleanup_target_kind=self.kind, cleanup_target_id=self.target_id, cleanup_response=self.cleanup,
            final_state=self.final, error=self.error)

    def _end(self, final: str, error: str | None) -> None:
        self.final, self.error = final, error

    def authorize(self):
        try:
            self.wr = self.c.authorize(self.request)
            return self.execute
        except WorkerAuthorizationError as exc:
            self.target_id = cleanup_target(self.kind, self.request.lease_id, self.request.session_id)
            try:
                self.cleanup = self.c.cleanup_coordinator.cleanup_authorization_failure(self.request,
                                                                                       target_kind=self.kind)
                self._end("authorization_failed", str(exc))
            except WorkerCleanupError as cexc:
                self._end("cleanup_failed", str(cexc))
            return None

    def execute(self):
        self.slot = self.c.staging_pool.allocate(self.wr.data_plane)
        self.result = self.c._run(self.wr, self.slot)
        self.update = status_update_for(self.result)
        return self.report

    def report(self):
        a = self.wr.authorization
        try:
            self.status = self.c.status_reporter.report(self.result)
        except WorkerStatusReportError as exc:
            self.release = self.c.staging_pool.release(self.slot.slot_id, self.wr.data_plane)
            self.target_id = cleanup_target(self.kind, a.lease_id, a.session_id)
            try:
                self.cleanup = self.c.cleanup_coordinator.cleanup_status_report_failure(self.wr,
                                                                                       target_kind=self.kind)
                self._end("status_failed", str(exc))
            except WorkerCleanupError as cexc:
                self._end("cleanup_failed", str(cexc))
            return None
        return self.finish

    def finish(self):
        a = self.wr.authorization
        self.target_id = a.lease_id if self.result.complete else cleanup_target(self.kind, a.lease_id,
                                                                                  a.session_id)
        try:
            self.cleanup = self.c.cleanup_coordinator.cleanup_execution_failure(self.wr, self.result,
                                                                               target_kind=self.kind)
        except WorkerCleanupError as exc:
            self._end("cleanup_failed", str(exc))
            return None
        self._end(self.result.state.value, self.result.error)
        return None


class WorkerTransferClient:
    """Runs authorized transfers: ``submit`` (execute only),
    ``submit_and_report``, ``submit_report_and_cleanup`` and the recorded
    ``submit_report_cleanup_lifecycle``."""

    _RAISE_FOR = {"authorization_failed": WorkerAuthorizationError, "status_failed": WorkerStatusReportError,
                  "cleanup_failed": WorkerCleanupError}

    def __init__(self, daemon_client, executor: object | None = None,
                 status_reporter: WorkerTransferStatusReporter | None = None,
                 cleanup_coordinator: WorkerTransferCleanupCoordinator | None = None,
                 staging_pool: WorkerStagingPool | None = None,
                 resource_binder: WorkerDataPlaneResourceBinder | None = None) -> None:
        if executor is None:  # the default executor binds through the default binder
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

    def _execute(self, wr: WorkerTransferRequest, slot: WorkerStagingSlot) -> WorkerTransferResult:
        bound = getattr(self.executor, "execute_bound", None)
        if self.resource_binder is None or not callable(bound):
            return self.executor.execute(wr, slot)
        try:
            with self.resource_binder.bind(wr.data_plane) as res:
                return bound(wr, slot, res)
        except WorkerDataPlaneResourceError as exc:
            return failed_result(wr, slot, str(exc))

    def _run(self, wr: WorkerTransferRequest, slot: WorkerStagingSlot) -> WorkerTransferResult:
        try:
            return check_completion_bytes(wr, self._execute(wr, slot))
        except Exception as exc:  # noqa: BLE001 - an executor failure is a failed result
            return failed_result(wr, slot, str(exc))

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
        err = self._RAISE_FOR.get(lc.final_state)
        if err is not None:
            raise err(lc.error or lc.final_state.replace("_", " "))
        if lc.result is None:
            raise RuntimeError("the worker lifecycle ended without a result")
        return lc.result

    def submit_report_cleanup_lifecycle(self, request: WorkerTransferAuthorizationRequest,
                                        cleanup_target_kind: str = "reservation") -> WorkerTransferLifecycleRecord:
        return _Lifecycle(self, request, cleanup_target_kind).run()


class WorkerTransferService:
    """Envelope-level entry point of the worker helper."""

    def __init__(self, daemon_client=None, transfer_client: WorkerTransferClient | None = None, **client_kw) -> None:
        if transfer_client is None:
            if daemon_client is None:
                raise ValueError("WorkerTransferService needs a daemon_client or transfer_client")
            transfer_client = WorkerTransferClient(daemon_client, **client_kw)
        self.transfer_client = transfer_client

    def handle_lifecycle(self, request: WorkerTransferAuthorizationRequest,
                         cleanup_target_kind: str = "reservation") -> WorkerTransferLifecycleRecord:
        if not isinstance(request, WorkerTransferAuthorizationRequest):
            raise TypeError("handle_lifecycle takes a WorkerTransferAuthorizationRequest")
        return self.transfer_client.submit_report_cleanup_lifecycle(request, cleanup_target_kind=cleanup_target_kind)

    def parse_authorization_request(self, payload: Mapping[str, object]) -> WorkerTransferAuthorizationRequest:
        return parse_worker_authorization_request_payload(payload)

    def handle_envelope(self, envelope) -> WorkerServiceResponseEnvelope:
        try:
            env = envelope if isinstance(envelope, WorkerServiceRequestEnvelope) else \
                WorkerServiceRequestEnvelope(**dict(envelope))
            lc = self.handle_lifecycle(self.parse_authorization_request(env.payload),
                                       cleanup_target_kind=env.cleanup_target_kind)
            return WorkerServiceResponseEnvelope.from_lifecycle(lc)
        except Exception as exc:  # noqa: BLE001 - any failure answers as an error envelope
            return WorkerServiceResponseEnvelope.from_error(str(exc))

    def handle_envelope_payload(self, envelope: Mapping[str, object]) -> dict[str, object]:
        return self.handle_envelope(envelope).as_dict()


_AUTH_FIELDS = ("transfer_id", "lease_id", "token", "session_id", "job_id", "src_buffer_id", "dst_buffer_id",
                "direction")


def parse_worker_authorization_request_payload(payload: Mapping[str, object]) -> WorkerTransferAuthorizationRequest:
    """``{...}`` or ``{"authorization": {...}}`` -> the request record."""
    body = payload.get("authorization", payload) if isinstance(payload, Mapping) else None
    if not isinstance(body, Mapping):
        raise ValueError("a worker authorization payload must be a mapping")
    missing = [k for k in _AUTH_FIELDS if k not in body]
    if missing:
        raise ValueError(f"missing worker authorization field: {missing[0]}")
    return WorkerTransferAuthorizationRequest(**{k: body[k] for k in _AUTH_FIELDS},
                                              ranges=tuple(body.get("ranges", ()) or ()),
                                              relay_gpu=body.get("relay_gpu"))


__all__ = [
    "CLEANUP_KINDS", "DaemonCall", "PlanLane", "TICKET_ISSUER", "TicketPlan", "WorkerAuthorizationError",
    "WorkerCleanupError", "WorkerDataPlaneCompletion", "WorkerDataPlaneCompletionEnvelope", "WorkerDataPlaneRequest",
    "WorkerServiceRequestEnvelope", "WorkerServiceResponseEnvelope", "WorkerStatusReportError",
    "WorkerTransferAuthorizer", "WorkerTransferCleanupCoordinator", "WorkerTransferClient",
    "WorkerTransferLifecycleRecord", "WorkerTransferRequest", "WorkerTransferResult", "WorkerTransferService",
    "WorkerTransferState", "WorkerTransferStatusReporter", "check_completion_bytes", "cleanup_calls",
    "cleanup_target", "failed_result", "parse_worker_authorization_request_payload", "plan_total_bytes",
    "planned_relays", "relay_ranges_for", "require_daemon_worker_plan", "status_update_for",
    "validate_daemon_ticket",
]
