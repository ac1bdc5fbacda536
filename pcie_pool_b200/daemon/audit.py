"""Audit records: one per relay authorization, completion, failure, mismatch
or cleanup.  The 29-field record shape is the reference's
(turbobus/daemon/server.py:2630-2670) so evidence tooling reads both."""

from __future__ import annotations

import time
from typing import Any

from ..schema import TransferStatusState

AUDIT_FIELDS = (
    "audit_id", "event_type", "created_at", "transfer_id", "decision_id", "ticket_id",
    "topology_snapshot_id", "lease_id", "session_id", "job_id", "user_id", "process_id",
    "container_id", "relay_gpu", "direction", "bytes_total", "bytes_completed",
    "duration_seconds", "state", "reason", "failure_reason", "cleanup_kind", "cleanup_target_id",
    "source_buffer_id", "destination_buffer_id", "buffer_ids", "staging_record_id",
)


def _first(*vals):
    for v in vals:
        if v is not None:
            return v
    return None


def build_audit_record(st, *, event_type: str, transfer_id: str | None = None, reservation=None,
                       lease=None, staging_record: dict | None = None, ticket=None,
                       state: TransferStatusState | str | None = None, reason: str | None = None,
                       failure_reason: str | None = None, cleanup_kind: str | None = None,
                       cleanup_target_id: str | None = None, session_id: str | None = None,
                       bytes_completed: int | None = None, now: float | None = None) -> dict[str, Any]:
    """Resolve every field from the most specific object available
    (reservation > lease > staging record > ticket > transfer status)."""
    created = float(time.time() if now is None else now)
    sr = staging_record or {}
    tid = transfer_id if transfer_id is not None else sr.get("transfer_id")
    tid = None if tid is None else str(tid)
    status = None if tid is None else st.statuses.get(tid)
    decision = None if tid is None else st.decisions.get(tid)
    ticket_id = ticket.ticket_id if ticket is not None else (None if tid is None else st.transfer_tickets.get(tid))
    if ticket is None and ticket_id is not None:
        ticket = st.tickets.get(ticket_id)
    lease_id = _first(None if lease is None else lease.lease_id,
                      None if reservation is None else reservation.reservation_id, sr.get("lease_id"))
    if lease is None and lease_id is not None:
        lease = st.leases.get(lease_id)
    sess = _first(session_id, None if status is None else status.session_id,
                  None if lease is None else lease.session_id,
                  None if reservation is None else reservation.session_id, sr.get("session_id"))
    job_id = _first(None if status is None else status.job_id, None if lease is None else lease.job_id,
                    sr.get("job_id"), None if decision is None else decision.job_id)
    job = None if job_id is None else st.jobs.get(job_id)
    if lease is not None:
        buffer_ids = tuple(lease.buffer_ids)
    elif sr:
        buffer_ids = tuple(str(b) for b in sr.get("buffer_ids", ()))
    elif ticket is not None:
        buffer_ids = (ticket.source_buffer_id, ticket.destination_buffer_id)
    else:
        buffer_ids = ()
    relay = _first(None if reservation is None else reservation.relay_gpu,
                   None if lease is None else lease.relay_gpu,
                   None if sr.get("relay_gpu") is None else int(sr["relay_gpu"]))
    direction = _first(None if reservation is None else reservation.direction, sr.get("direction"),
                       None if ticket is None else ticket.direction)
    if reservation is not None:
        total = int(reservation.bytes)
    elif sr:
        total = int(sr.get("requested_bytes", 0) or 0)
    else:
        total = 0 if status is None else int(status.bytes_total)
    done = int(bytes_completed) if bytes_completed is not None else (
        int(status.bytes_completed) if status is not None else 0)
    if reservation is not None and total:
        done = min(done, total)
    started = float(sr.get("created_at", 0.0) or 0.0) if sr else (
        float(decision.issued_at) if decision is not None else None)
    rec = {
        "audit_id": f"audit-{len(st.audit) + 1}",
        "event_type": str(event_type),
        "created_at": created,
        "transfer_id": tid,
        "decision_id": None if decision is None else decision.decision_id,
        "ticket_id": ticket_id,
        "topology_snapshot_id": None if decision is None else decision.topology_snapshot_id,
        "lease_id": lease_id,
        "session_id": None if sess is None else str(sess),
        "job_id": job_id,
        "user_id": None if job is None else job.user_id,
        "process_id": None if job is None else job.process_id,
        "container_id": None if job is None else job.container_id,
        "relay_gpu": relay,
        "direction": direction,
        "bytes_total": total,
        "bytes_completed": done,
        "duration_seconds": max(0.0, created - started) if started else None,
        "state": state.value if isinstance(state, TransferStatusState) else (None if state is None else str(state)),
        "reason": reason,
        "failure_reason": failure_reason,
        "cleanup_kind": cleanup_kind,
        "cleanup_target_id": cleanup_target_id,
        "source_buffer_id": None if ticket is None else ticket.source_buffer_id,
        "destination_buffer_id": None if ticket is None else ticket.destination_buffer_id,
        "buffer_ids": buffer_ids,
        "staging_record_id": sr.get("staging_record_id") if sr else None,
    }
    st.audit.append(rec)
    return rec
