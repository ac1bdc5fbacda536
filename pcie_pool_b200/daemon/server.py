"""The per-node daemon: the authority over sessions, jobs, buffers, relay
leases, plans, admissions, tickets, transfer statuses, staging records, the
audit log and the bandwidth-profile cache.

Semantics follow the reference daemon (turbobus/daemon/server.py) so existing
clients and workers interoperate: the same 23 request types, payload keys,
error strings, lease/plan TTLs (30 s), plan generations, admission states
(admitted / delayed / expired), cleanup cascade and audit records.  What is
new here:

* intents are *executed*: with an ``executor`` attached, every admitted
  intent is handed to the data plane and its receipt turns ``complete`` (or
  ``failed``) with measured per-lane statistics and ``completed_at``
  (the reference only plans them);
* delayed admissions are re-evaluated automatically when relay capacity is
  released, instead of waiting for an explicit RESCHEDULE_TRANSFER;
* ``wait_transfer_receipt`` blocks on a condition variable instead of a
  10 ms polling loop;
* the profile cache can persist to a JSON file across daemon restarts;
* the socket server serves connections concurrently (one thread each).
"""

from __future__ import annotations

import json
import os
import threading
from collections import deque
import time
import uuid
from dataclasses import dataclass, field
from collections.abc import Mapping
from typing import Any, Callable, Iterable

from ..scheduler import DaemonScheduler, scheduling_decision_leases, scheduling_decision_stats
from ..schema import contract_asdict as asdict
from ..utils.log import logger
from ..schema import (BufferRegistration, CleanupRequest, DaemonRequest, DaemonResponse,
                      ExecutionTicket, JobIdentity, LeaseToken, PeerIdentity, RelayQuota, RequestType,
                      SchedulingDecision, Session, TERMINAL_STATES, TransferIntent, TransferReceipt,
                      TransferReservation, TransferStatus, TransferStatusState,
                      WorkerTransferAuthorization, WorkerTransferAuthorizationRequest, byte_ranges)
from ..planner_types import assignment_bytes, assignment_chunk_count, assignment_has_chunks, assignment_spans
from ..topology import TopologyProvider
from .audit import build_audit_record
from .landing import LandingSpec, validate_landing
from .wire import reserve_socket

ADMITTED = "admitted"
DELAYED = "delayed"
EXPIRED = "expired"
PLAN_TTL_SECONDS = 30.0
TICKET_ISSUER = "turbobus-daemon"
_LOG = logger("daemon")
TOPOLOGY_UNAVAILABLE = "topology provider is required; synthetic topology is test fixture only"
PROFILE_STORE_FORMAT = "pcie_pool_b200.profile_cache.v1"


def ok(**payload) -> DaemonResponse:
    return DaemonResponse(ok=True, payload=payload)


def fail(error: str, **payload) -> DaemonResponse:
    return DaemonResponse(ok=False, payload=payload, error=error)


def removed_summary() -> dict[str, int]:
    return {"jobs": 0, "buffers": 0, "sessions": 0, "reservations": 0, "staging_records": 0,
            "transfers": 0}


def merge_removed(into: dict | None, src: dict | None) -> dict | None:
    if into is not None and src:
        for k, v in src.items():
            into[k] = int(into.get(k, 0)) + int(v)
    return into


@dataclass
class DaemonState:
    jobs: dict[str, JobIdentity] = field(default_factory=dict)
    job_peers: dict[str, PeerIdentity] = field(default_factory=dict)
    session_peers: dict[str, PeerIdentity] = field(default_factory=dict)
    buffers: dict[str, BufferRegistration] = field(default_factory=dict)
    buffer_fds: dict[str, int] = field(default_factory=dict)  # daemon-owned VMM descriptors
    sessions: dict[str, Session] = field(default_factory=dict)
    reservations: dict[str, TransferReservation] = field(default_factory=dict)
    reservation_transfer: dict[str, str] = field(default_factory=dict)
    intents: dict[str, TransferIntent] = field(default_factory=dict)
    intent_transfer: dict[str, str] = field(default_factory=dict)
    queue: dict[str, None] = field(default_factory=dict)    # transfer ids in submit order (ordered set)
    live: dict[str, None] = field(default_factory=dict)     # the non-terminal ones among them
    terminal_order: deque = field(default_factory=deque)    # terminal ids, oldest first (history trim)
    ticket_ids: dict[str, list[str]] = field(default_factory=dict)  # transfer id -> every ticket issued
    queue_records: dict[str, dict[str, Any]] = field(default_factory=dict)
    version: int = 0
    plan_requests: dict[str, dict[str, Any]] = field(default_factory=dict)
    generations: dict[str, int] = field(default_factory=dict)
    plan_expiry: dict[str, float] = field(default_factory=dict)
    admissions: dict[str, dict[str, Any]] = field(default_factory=dict)
    lease_generation: dict[str, int] = field(default_factory=dict)
    plans: dict[str, dict[str, Any]] = field(default_factory=dict)
    decisions: dict[str, SchedulingDecision] = field(default_factory=dict)
    tickets: dict[str, ExecutionTicket] = field(default_factory=dict)
    transfer_tickets: dict[str, str] = field(default_factory=dict)
    leases: dict[str, LeaseToken] = field(default_factory=dict)
    statuses: dict[str, TransferStatus] = field(default_factory=dict)
    staging: dict[str, dict[str, Any]] = field(default_factory=dict)
    audit: list[dict[str, Any]] = field(default_factory=list)
    conn_sessions: set[str] = field(default_factory=set)
    conn_session_conn: dict[str, str] = field(default_factory=dict)
    cleanup_events: list[CleanupRequest] = field(default_factory=list)
    system_cleanup_events: list[CleanupRequest] = field(default_factory=list)
    profiles: dict[str, dict[str, Any]] = field(default_factory=dict)
    measured: dict[str, dict[str, Any]] = field(default_factory=dict)
    completed_at: dict[str, float] = field(default_factory=dict)
    target_seen: dict[int, float] = field(default_factory=dict)  # device -> last time it was a target


class TurboBusDaemon:
    """Resource-control daemon (the node's PCIe-pool authority)."""

    def __init__(self, relay_gpus: Iterable[int], max_sessions_per_relay: int = 1,
                 max_inflight_chunks_per_relay: int = 8, session_timeout_seconds: float = 0.0,
                 profile_max_age_seconds: float = 0.0,
                 topology_provider: TopologyProvider | None = None, *,
                 scheduler: DaemonScheduler | None = None, executor=None,
                 profile_store_path: str | None = None,
                 clock: Callable[[], float] = time.time, link_hold_seconds: float = 1.0,
                 history_limit: int = 10000, audit_limit: int = 100000, lane_feedback: bool = True,
                 uplink_rates: Mapping[int, float] | None = None, lend_ratio: float = 1.25) -> None:
        self._lock = threading.RLock()
        self._changed = threading.Condition(self._lock)
        self._st = DaemonState()
        self._scheduler = scheduler or DaemonScheduler()
        self._topology = topology_provider
        self._session_timeout = max(0.0, float(session_timeout_seconds))
        self._profile_max_age = max(0.0, float(profile_max_age_seconds))
        # A GPU that was the target of a transfer within this window is not
        # lent as a relay: in multi-tenant training every GPU moves its own
        # shard each step, and relaying through it only queues another job's
        # chunks in front of that GPU's own on its link.  0 disables.
        self._link_hold = max(0.0, float(link_hold_seconds))
        # A long-running daemon keeps the records of the last ``history_limit``
        # finished transfers (receipts, statuses, plans, tickets) and the last
        # ``audit_limit`` audit records; older ones are dropped, so memory and
        # the per-request bookkeeping stay bounded.
        self._history_limit = max(1, int(history_limit))
        self._audit_limit = max(1, int(audit_limit))
        self._clock = clock
        self._quotas = {g: RelayQuota(relay_gpu=g, max_sessions=int(max_sessions_per_relay),
                                      max_inflight_chunks=int(max_inflight_chunks_per_relay))
                        for g in norm_relays(relay_gpus)}
        # Per-lane rates measured by the data plane, per (target, direction,
        # landing op): a fused op loads the lanes differently from the plain
        # copies a profile probes (the target's own landing kernel shares its
        # SMs and HBM with every relay's), so each op's split converges to all
        # lanes finishing together.  They refine the profile's concurrent
        # lane rates once every lane of the profile has been measured.
        from ..parallel.balance import LaneBalancer

        self._feedback = LaneBalancer(alpha=0.5) if lane_feedback else None
        self._published: dict[tuple[int, str], tuple[object, dict, dict]] = {}
        # Lending across contention groups (off unless rates are given): a GPU
        # whose link is busy with its own traffic, or held for it, may still
        # relay for a target whose measured concurrent rate (all links busy)
        # is lower by ``lend_ratio`` or more -- a GPU in a more contended
        # uplink group.  The busy GPU's own uplink group has the headroom the
        # borrower's lacks; the lane feedback then sizes the borrowed lanes.
        self._uplink_rates: dict[int, float] = {}
        self._lend_ratio = max(1.0, float(lend_ratio))
        if uplink_rates:
            self.set_uplink_rates(uplink_rates)
        self._executor = None
        self._profile_store = profile_store_path
        if profile_store_path:
            self._load_profiles(profile_store_path)
        if executor is not None:
            self.attach_executor(executor)

    def set_uplink_rates(self, rates: Mapping[int, float] | None) -> None:
        """Per-GPU host->device rate measured with every link busy
        (``topology.uplink_probe.probe_rates(...)["concurrent"]``); None or
        empty turns lending across contention groups off."""
        with self._lock:
            self._uplink_rates = {int(g): float(r) for g, r in (rates or {}).items() if float(r) > 0.0}

    def _lendable(self, target: int) -> frozenset[int]:
        """Busy or held GPUs that may still relay for ``target`` (see
        ``set_uplink_rates``)."""
        rates = self._uplink_rates
        mine = rates.get(int(target))
        if not rates or mine is None:
            return frozenset()
        return frozenset(g for g, r in rates.items() if g != int(target) and r >= self._lend_ratio * mine)

    # ---- accessors -------------------------------------------------------------------
    @property
    def relay_gpus(self) -> tuple[int, ...]:
        return tuple(sorted(self._quotas))

    @property
    def topology_provider(self) -> TopologyProvider | None:
        return self._topology

    def attach_executor(self, executor) -> None:
        """Hand admitted intents to ``executor.submit(daemon, transfer_id, ticket)``."""
        self._executor = executor
        bind = getattr(executor, "bind", None)
        if callable(bind):
            bind(self)

    def _now(self) -> float:
        return float(self._clock())

    # ---- topology / discovery --------------------------------------------------------
    def get_inventory(self) -> DaemonResponse:
        if self._topology is None:
            return fail(TOPOLOGY_UNAVAILABLE)
        inv = self._topology.snapshot()
        return ok(inventory=inv.as_dict(), topology_snapshot=asdict(inv.to_topology_snapshot()))

    def invalidate_topology(self) -> DaemonResponse:
        if self._topology is None:
            return fail(TOPOLOGY_UNAVAILABLE)
        inval = getattr(self._topology, "invalidate", None)
        if not callable(inval):
            return fail("topology provider does not support invalidation")
        try:
            inval()
        except NotImplementedError:
            return fail("topology provider does not support invalidation")
        inv = self._topology.snapshot()
        return ok(topology_snapshot_id=inv.topology_snapshot_id(), topology_version=inv.version,
                  inventory_source=inv.source, inventory_discovered_at=inv.discovered_at,
                  inventory=inv.as_dict(), topology_snapshot=asdict(inv.to_topology_snapshot()))

    def discover_relays(self, target_gpu: int | None = None,
                        requested_relays: Iterable[int] | None = None) -> DaemonResponse:
        now = self._now()
        with self._lock:
            self._reap(now)
            if self._topology is None:
                return fail(TOPOLOGY_UNAVAILABLE)
            inv = self._topology.snapshot()
            cands = tuple(sorted(self._quotas)) if requested_relays is None else tuple(norm_relays(requested_relays))
            disc = self._discovery(inv, None if target_gpu is None else int(target_gpu), cands)
            if target_gpu is not None:
                # every eligible relay, in the order that spreads lanes over
                # sockets, root complexes and switches (take a prefix)
                disc["recommended_relays"] = inv.spread_relays(int(target_gpu),
                                                               [g for g in cands if g in self._quotas], len(cands))
            return ok(relay_discovery=disc)

    def choose_relays(self, target_gpu: int, count: int, candidates: Iterable[int] | None = None) -> list[int]:
        """``count`` relays for lanes into ``target_gpu``, spread over PCIe
        uplinks (topology: socket, root complex, switch), among the relays
        this daemon lends."""
        with self._lock:
            if self._topology is None:
                raise ValueError(TOPOLOGY_UNAVAILABLE)
            inv = self._topology.snapshot()
            cands = sorted(self._quotas) if candidates is None else [g for g in norm_relays(candidates)
                                                                     if g in self._quotas]
            return inv.spread_relays(int(target_gpu), cands, int(count))

    # ---- sessions / jobs / buffers -----------------------------------------------------
    def register_session(self, target_gpu: int, requested_relays: Iterable[int],
                         max_inflight_chunks: int = 8, peer_identity: PeerIdentity | None = None,
                         connection_scoped: bool = False, connection_id: str | None = None) -> DaemonResponse:
        relays = norm_relays(requested_relays)
        inflight = int(max_inflight_chunks)
        if inflight <= 0:
            return fail("max_inflight_chunks must be positive")
        now = self._now()
        with self._lock:
            self._reap(now)
            bad = [g for g in relays if g not in self._quotas or not self._quotas[g].can_attach()]
            if bad:
                return fail(f"relay GPUs are unavailable: {bad}")
            sid = str(uuid.uuid4())
            s = Session(session_id=sid, target_gpu=int(target_gpu), relay_gpus=relays,
                        max_inflight_chunks=inflight, created_at=now, last_seen=now)
            self._st.sessions[sid] = s
            if peer_identity is not None:
                self._st.session_peers[sid] = peer_identity
            if connection_scoped:
                self._st.conn_sessions.add(sid)
                if connection_id is not None:
                    self._st.conn_session_conn[sid] = str(connection_id)
            for g in relays:
                self._quotas[g].sessions.add(sid)
            payload: dict[str, Any] = {"session": asdict(s)}
            if peer_identity is not None:
                payload["peer_identity"] = asdict(peer_identity)
            if connection_scoped:
                payload["connection_scoped"] = True
            return DaemonResponse(ok=True, payload=payload)

    def register_job(self, job_id: str, user_id: str | None = None, session_id: str | None = None,
                     container_id: str | None = None, process_id: int | None = None,
                     weight: float = 1.0, peer_identity: PeerIdentity | None = None) -> DaemonResponse:
        try:
            user_id, process_id, container_id = bind_job_to_peer(user_id, process_id, container_id,
                                                                 peer_identity)
        except ValueError as exc:
            return fail(str(exc))
        job = JobIdentity(job_id=job_id, user_id=user_id, session_id=session_id,
                          container_id=container_id, process_id=process_id, weight=weight)
        with self._lock:
            if job.session_id is not None and job.session_id not in self._st.sessions:
                return fail("unknown session")
            try:
                same_owner(self._st.session_peers.get(job.session_id) if job.session_id else None,
                           peer_identity, "session")
            except ValueError as exc:
                return fail(str(exc))
            self._st.jobs[job.job_id] = job
            if peer_identity is not None:
                self._st.job_peers[job.job_id] = peer_identity
            payload: dict[str, Any] = {"job": asdict(job)}
            if peer_identity is not None:
                payload["peer_identity"] = asdict(peer_identity)
            return DaemonResponse(ok=True, payload=payload)

    def register_buffer(self, buffer_id: str, job_id: str, kind: str, size_bytes: int,
                        device_index: int | None = None, address: int | None = None,
                        pinned: bool = False, handle_type: str = "registered_buffer",
                        metadata: dict | None = None,
                        peer_identity: PeerIdentity | None = None, fds: list[int] | None = None) -> DaemonResponse:
        md = dict(metadata or {})
        owned_fd = None
        if str(handle_type).lower() == "cuda_vmm_fd":
            # keep a duplicate of the exporter's descriptor for as long as the
            # buffer stays registered (the executor imports and maps it)
            if fds:
                if len(fds) != 1:
                    return fail("a cuda_vmm_fd buffer takes exactly one descriptor")
                owned_fd = os.dup(int(fds[0]))
            elif "vmm_fd" in md:  # in-process caller: its own descriptor number
                owned_fd = os.dup(int(md["vmm_fd"]))
            else:
                return fail("a cuda_vmm_fd buffer needs its descriptor attached")
            md["vmm_fd"] = owned_fd
        try:
            buf = BufferRegistration(buffer_id=buffer_id, job_id=job_id, kind=kind, size_bytes=size_bytes,
                                     device_index=device_index, address=address, pinned=pinned,
                                     handle_type=handle_type, metadata=md)
        except (TypeError, ValueError):
            if owned_fd is not None:
                os.close(owned_fd)
            raise
        with self._lock:
            self._reap(self._now())
            if buf.job_id not in self._st.jobs:
                return fail("unknown job")
            try:
                self._peer_owns_job(buf.job_id, peer_identity)
            except ValueError as exc:
                return fail(str(exc))
            if self._buffer_leases(buf.buffer_id):
                if owned_fd is not None:
                    os.close(owned_fd)
                return fail("buffer has active lease")
            self._drop_buffer(buf.buffer_id)
            self._st.buffers[buf.buffer_id] = buf
            if owned_fd is not None:
                self._st.buffer_fds[buf.buffer_id] = owned_fd
            return ok(buffer=asdict(buf))

    def _drop_buffer(self, buffer_id: str):
        """Forget a registration and close the descriptor the daemon kept for it."""
        fd = self._st.buffer_fds.pop(str(buffer_id), None)
        if fd is not None:
            try:
                os.close(fd)
            except OSError:
                pass
        return self._st.buffers.pop(str(buffer_id), None)

    # ---- cleanup -----------------------------------------------------------------------
    def cleanup(self, target_kind: str, target_id: str, reason: str, force: bool = False) -> DaemonResponse:
        req = CleanupRequest(target_kind=target_kind, target_id=target_id, reason=reason, force=force)
        with self._lock:
            removed = removed_summary()
            kind, tid = req.target_kind, req.target_id
            if kind == "job":
                if tid not in self._st.jobs and not req.force:
                    return fail("unknown job")
                merge_removed(removed, self._cleanup_job(tid, req.reason))
            elif kind == "buffer":
                if tid not in self._st.buffers and not req.force:
                    return fail("unknown buffer")
                transfers = self._transfers_for_buffer(tid)
                for lid in self._buffer_leases(tid):
                    merge_removed(removed, self._release_counted(lid, TransferStatusState.CANCELED, req.reason))
                if self._drop_buffer(tid) is not None:
                    removed["buffers"] += 1
                for t in transfers:
                    if self._cancel_if_active(t, req.reason):
                        removed["transfers"] += 1
            elif kind == "session":
                if self._close_session(tid, req.reason, removed) is None and not req.force:
                    return fail("unknown session")
            elif kind == "reservation":
                rel = self._release_counted(tid, TransferStatusState.CANCELED, req.reason)
                if rel["reservations"] == 0 and rel["staging_records"] == 0 and not req.force:
                    return fail("unknown reservation")
                merge_removed(removed, rel)
            else:
                return fail("unsupported cleanup target")
            self._st.cleanup_events.append(req)
            self._changed.notify_all()
            self._readmit_delayed()
            return ok(cleanup=asdict(req), removed=removed)

    def close_session(self, session_id: str) -> DaemonResponse:
        with self._lock:
            self._reap_sessions(self._now())
            removed = removed_summary()
            if self._close_session(session_id, "session_closed", removed) is None:
                return fail("unknown session")
            self._changed.notify_all()
            self._readmit_delayed()
            return ok(session_id=session_id, removed=removed)

    # ---- manual reservations -------------------------------------------------------------
    def reserve_transfer(self, session_id: str, relay_gpu: int, chunks: int, bytes_: int = 0,
                         direction: str = "unknown") -> DaemonResponse:
        chunks, relay, nbytes = int(chunks), int(relay_gpu), int(bytes_)
        d = str(direction).lower()
        if chunks <= 0:
            return fail("chunks must be positive")
        if nbytes < 0:
            return fail("bytes must be non-negative")
        if d not in ("h2d", "d2h", "unknown"):
            return fail("direction must be h2d, d2h, or unknown")
        now = self._now()
        with self._lock:
            self._reap(now)
            s = self._st.sessions.get(session_id)
            if s is None or not s.active:
                return fail("unknown session")
            if relay not in s.relay_gpus:
                return fail("relay GPU is not assigned to this session")
            if chunks > s.max_inflight_chunks:
                return fail("reservation exceeds session chunk limit")
            if s.active_chunks + chunks > s.max_inflight_chunks:
                return fail("session chunk quota is unavailable")
            q = self._quotas.get(relay)
            if q is None or not q.can_reserve(chunks):
                return fail("relay chunk quota is unavailable")
            r = TransferReservation(reservation_id=str(uuid.uuid4()), session_id=session_id,
                                    relay_gpu=relay, chunks=chunks, bytes=nbytes, direction=d)
            self._st.reservations[r.reservation_id] = r
            tok = LeaseToken(lease_id=r.reservation_id, session_id=session_id, relay_gpu=relay,
                             token=str(uuid.uuid4()), issued_at=now, expires_at=0.0)
            self._st.leases[tok.lease_id] = tok
            s.active_chunks += chunks
            q.active_chunks += chunks
            self._touch(session_id, now)
            return ok(reservation=asdict(r), lease_token=asdict(tok))

    def release_transfer(self, reservation_id: str) -> DaemonResponse:
        with self._lock:
            rid = str(reservation_id)
            tid = self._st.reservation_transfer.get(rid)
            if tid is not None:
                st = self._st.statuses.get(tid)
                if st is None:
                    return fail("unknown transfer")
                if st.state is not TransferStatusState.COMPLETE:
                    return fail("transfer is not complete")
            if self._release(rid) is None:
                return fail("unknown reservation")
            self._changed.notify_all()
            self._readmit_delayed()
            return ok(reservation_id=reservation_id)

    # ---- transfer status --------------------------------------------------------------------
    def transfer_status(self, transfer_id: str, state: str | None = None,
                        bytes_completed: int | None = None, error: str | None = None) -> DaemonResponse:
        with self._lock:
            resp = self._transfer_status(str(transfer_id), state, bytes_completed, error)
            self._changed.notify_all()
            if resp.ok and state is not None and TransferStatusState(state) in TERMINAL_STATES:
                self._readmit_delayed()
            return resp

    def _transfer_status(self, tid: str, state, nbytes, error) -> DaemonResponse:
        cur = self._st.statuses.get(tid)
        if cur is None:
            return fail("unknown transfer")
        if state is None and nbytes is None and error is None:
            return ok(status=asdict(cur))
        try:
            want = cur.state if state is None else TransferStatusState(state)
        except ValueError as exc:
            return fail(str(exc))
        if cur.state in TERMINAL_STATES:
            same = want == cur.state and (nbytes is None or _as_int(nbytes) == cur.bytes_completed) \
                and (error is None or error == cur.error)
            return ok(status=asdict(cur)) if same else fail("terminal transfer status cannot be updated")
        try:
            new = TransferStatus(transfer_id=cur.transfer_id, job_id=cur.job_id, state=want,
                                 bytes_total=cur.bytes_total,
                                 bytes_completed=cur.bytes_completed if nbytes is None else int(nbytes),
                                 session_id=cur.session_id, error=cur.error if error is None else error)
        except ValueError as exc:
            if want is TransferStatusState.COMPLETE:
                # A completion that does not account for every byte fails the
                # transfer and releases what it held.
                msg = str(exc)
                failed = self._terminal(tid, TransferStatusState.FAILED, msg)
                self._audit_transfer("detected_mismatch", tid, TransferStatusState.FAILED,
                                     reason="transfer_status_mismatch", failure_reason=msg)
                removed = self._release_for_transfer(tid, TransferStatusState.FAILED, "transfer_status_mismatch")
                self._refresh_record(tid)
                return fail(msg, status=asdict(failed), removed=removed)
            return fail(str(exc))
        self._st.statuses[tid] = new
        if new.state in TERMINAL_STATES:
            self._st.completed_at.setdefault(tid, self._now())
        self._refresh_record(tid)
        removed = removed_summary()
        if new.state is TransferStatusState.COMPLETE:
            self._audit_transfer("worker_completion", tid, new.state, bytes_completed=new.bytes_completed)
        elif new.state in (TransferStatusState.FAILED, TransferStatusState.CANCELED):
            failed = new.state is TransferStatusState.FAILED
            why = new.error or ("worker_failed" if failed else "transfer_canceled")
            self._audit_transfer("worker_failure" if failed else "transfer_canceled", tid, new.state,
                                 reason=why, failure_reason=why, bytes_completed=new.bytes_completed)
            merge_removed(removed, self._release_for_transfer(tid, new.state, why))
        return ok(status=asdict(new), removed=removed)

    # ---- intents ------------------------------------------------------------------------------
    def submit_transfer_intent(self, intent: TransferIntent,
                               peer_identity: PeerIdentity | None = None) -> DaemonResponse:
        if not isinstance(intent, TransferIntent):
            return fail("intent must be a TransferIntent")
        try:
            chunk = intent_chunk_bytes(intent)
            spec = LandingSpec.from_metadata(intent.metadata)
        except (TypeError, ValueError) as exc:
            return fail(str(exc))
        if spec is not None and spec.op != "copy":
            with self._lock:
                try:
                    self._validate_landing(intent, spec, chunk, peer_identity)
                except ValueError as exc:
                    return fail(str(exc))
        with self._lock:
            existing = self._st.intent_transfer.get(intent.intent_id)
            if existing is not None:
                # Idempotent resubmission of the same intent.
                if self._st.intents.get(intent.intent_id) != intent:
                    return fail("intent_id already belongs to a different transfer intent")
                try:
                    self._validate_buffers((intent.source_buffer_id, intent.destination_buffer_id),
                                           intent.job_id, intent.session_id, peer_identity)
                    receipt = self._receipt(intent.intent_id)
                except ValueError as exc:
                    return fail(str(exc))
                tk = self._st.transfer_tickets.get(existing)
                return ok(receipt=asdict(receipt), transfer_id=existing,
                          ticket=None if tk is None else asdict(self._st.tickets[tk]))
        planned = self.plan_transfer(
            session_id=intent.session_id, total_bytes=intent.total_bytes, chunk_bytes=chunk,
            mode="auto", direction=intent.direction, job_id=intent.job_id,
            buffer_ids=[intent.source_buffer_id, intent.destination_buffer_id], ranges=intent.ranges,
            intent_id=intent.intent_id, workload_kind=intent.workload_kind.value,
            priority=intent.priority, peer_identity=peer_identity, allow_delayed_admission=True,
            _for_intent=True)
        if not planned.ok:
            return planned
        tid = str(planned.payload["transfer_id"])
        now = self._now()
        with self._lock:
            decision = self._st.decisions.get(tid)
            if decision is None:
                return fail("scheduling decision is unavailable")
            self._st.intents[intent.intent_id] = intent
            self._st.intent_transfer[intent.intent_id] = tid
            ticket = None
            if self._st.admissions.get(tid, {}).get("state") == ADMITTED:
                ticket = self._intent_ticket(intent, tid, decision, now)
                self._store_ticket(tid, ticket)
            self._refresh_record(tid, now)
            receipt = self._receipt(intent.intent_id)
            resp = ok(receipt=asdict(receipt), transfer_id=tid, decision=asdict(decision),
                      ticket=None if ticket is None else asdict(ticket),
                      admission=planned.payload.get("admission", {}),
                      plan_generation=planned.payload.get("plan_generation", 0),
                      plan_expires_at=planned.payload.get("plan_expires_at"),
                      reservations=planned.payload.get("reservations", []),
                      lease_tokens=planned.payload.get("lease_tokens", []),
                      planning=planned.payload.get("planning", {}))
            if ticket is not None:
                self._dispatch(tid, ticket)
            return resp

    def _validate_landing(self, intent: TransferIntent, spec: LandingSpec, chunk: int, peer) -> None:
        """A fused-op intent may only touch buffers its job registered: the
        spec's kv buffers are checked for ownership (authenticated peer) and
        every unit / tensor it addresses for bounds (daemon/landing.py)."""
        S = self._st
        h2d = intent.direction == "h2d"
        host_id, dev_id = ((intent.source_buffer_id, intent.destination_buffer_id) if h2d
                           else (intent.destination_buffer_id, intent.source_buffer_id))
        host, dev = S.buffers.get(host_id), S.buffers.get(dev_id)
        if host is None or dev is None:
            raise ValueError("unknown buffer")
        for bid in spec.buffer_ids():
            self._peer_owns_buffer(bid, peer)
        validate_landing(spec, direction=intent.direction, job_id=intent.job_id, device_buffer=dev,
                         host_buffer=host, ranges=intent.ranges, total_bytes=intent.total_bytes,
                         chunk_bytes=chunk, buffers=S.buffers)

    def landing_buffers(self, intent: TransferIntent | None) -> dict[str, BufferRegistration]:
        """Registrations of the extra device buffers a fused-op intent names
        (the executor resolves their addresses)."""
        if intent is None:
            return {}
        try:
            spec = LandingSpec.from_metadata(intent.metadata)
        except ValueError:
            return {}
        if spec is None:
            return {}
        with self._lock:
            return {b: self._st.buffers[b] for b in spec.buffer_ids() if b in self._st.buffers}

    def wait_transfer_receipt(self, intent_id: str, timeout_seconds: float | None = None) -> DaemonResponse:
        iid = str(intent_id)
        timeout = 0.0 if timeout_seconds is None else max(0.0, float(timeout_seconds))
        deadline = time.monotonic() + timeout
        with self._lock:
            while True:
                # the receipt is built once, when it is answered; a wake-up
                # before the transfer ends only looks at its state
                tid = self._st.intent_transfer.get(iid)
                st = self._st.statuses.get(tid) if tid is not None else None
                left = deadline - time.monotonic()
                if st is None or st.state in TERMINAL_STATES or timeout_seconds is None or left <= 0:
                    try:
                        return ok(receipt=asdict(self._receipt(iid)))
                    except ValueError as exc:
                        return fail(str(exc))
                self._changed.wait(timeout=min(left, 0.5))

    # ---- leases -----------------------------------------------------------------------------
    def validate_lease(self, lease_id: str, token: str, session_id: str | None = None,
                       relay_gpu: int | None = None, job_id: str | None = None,
                       buffer_ids: Iterable[str] | None = None, now: float | None = None,
                       peer_identity: PeerIdentity | None = None) -> DaemonResponse:
        at = self._now() if now is None else float(now)
        with self._lock:
            self._reap_sessions(at)
            lease = self._st.leases.get(str(lease_id))
            if lease is None:
                return fail("unknown lease")
            if lease.token != str(token):
                return fail("invalid lease token")
            if session_id is not None and lease.session_id != str(session_id):
                return fail("lease session mismatch")
            if relay_gpu is not None and lease.relay_gpu != int(relay_gpu):
                return fail("lease relay mismatch")
            if job_id is not None and lease.job_id != str(job_id):
                return fail("lease job mismatch")
            owner = lease.job_id if lease.job_id is not None else job_id
            try:
                if owner is not None:
                    self._peer_owns_job(str(owner), peer_identity)
                if buffer_ids is not None:
                    req = tuple(str(b) for b in buffer_ids)
                    if req != lease.buffer_ids:
                        return fail("lease buffer mismatch")
                    for b in req:
                        buf = self._st.buffers.get(b)
                        if buf is None:
                            return fail("unknown buffer")
                        if lease.job_id is not None and buf.job_id != lease.job_id:
                            return fail("lease buffer owner mismatch")
                        self._peer_owns_buffer(b, peer_identity)
            except ValueError as exc:
                return fail(str(exc))
            if lease.expires_at and at > lease.expires_at:
                self._expire_lease(lease.lease_id)
                return fail("lease expired")
            if lease.lease_id not in self._st.reservations:
                return fail("lease is not active")
            tid = self._st.reservation_transfer.get(lease.lease_id)
            if tid is not None:
                tk = self._st.tickets.get(self._st.transfer_tickets.get(tid, ""))
                if tk is not None and at > tk.expires_at:
                    return fail("execution ticket expired")
                err = self._admission_error(tid, lease.lease_id, at)
                if err is not None:
                    return fail(err)
                st = self._st.statuses.get(tid)
                if st is not None and st.state in TERMINAL_STATES:
                    return fail("transfer is terminal")
            return ok(lease_token=asdict(lease))

    def authorize_worker_transfer(self, request: WorkerTransferAuthorizationRequest,
                                  peer_identity: PeerIdentity | None = None) -> DaemonResponse:
        now = self._now()
        with self._lock:
            self._reap_sessions(now)
            return self._authorize(request, peer_identity, now)

    def _authorize(self, req: WorkerTransferAuthorizationRequest, peer, now: float) -> DaemonResponse:
        S = self._st
        st = S.statuses.get(req.transfer_id)
        if st is None:
            return fail("unknown transfer")
        if st.session_id != req.session_id:
            return fail("transfer session mismatch")
        if st.job_id != req.job_id:
            return fail("transfer job mismatch")
        try:
            self._peer_owns_job(req.job_id, peer)
        except ValueError as exc:
            return fail(str(exc))
        if st.state in TERMINAL_STATES:
            return fail("transfer is terminal")
        lease = S.leases.get(req.lease_id)
        if lease is None:
            return fail("unknown lease")
        for bad, msg in ((lease.token != req.token, "invalid lease token"),
                         (lease.session_id != req.session_id, "lease session mismatch"),
                         (lease.job_id != req.job_id, "lease job mismatch"),
                         (req.relay_gpu is not None and lease.relay_gpu != req.relay_gpu, "lease relay mismatch")):
            if bad:
                return fail(msg)
        if lease.expires_at and now > lease.expires_at:
            self._expire_lease(lease.lease_id)
            return fail("lease expired")
        if lease.lease_id not in S.reservations:
            return fail("lease is not active")
        err = self._admission_error(req.transfer_id, lease.lease_id, now)
        if err is not None:
            return fail(err)
        if S.reservations[lease.lease_id].direction not in ("unknown", req.direction):
            return fail("reservation direction mismatch")
        plan = S.plans.get(req.transfer_id)
        if plan is None:
            return fail("transfer plan is unavailable")
        try:
            related = self._worker_leases(req, lease)
        except ValueError as exc:
            return fail(str(exc))
        if len(related) > 1:
            err = self._admission_error(req.transfer_id, None, now)
            if err is not None:
                return fail(err)
            for other in related:
                if other.lease_id == lease.lease_id:
                    continue
                err = self._admission_error(req.transfer_id, other.lease_id, now)
                if err is not None:
                    return fail(err)
                if other.expires_at and now > other.expires_at:
                    self._expire_lease(other.lease_id)
                    return fail("lease expired")
                for bad, msg in ((other.lease_id not in S.reservations, "lease is not active"),
                                 (other.session_id != req.session_id, "lease session mismatch"),
                                 (other.job_id != req.job_id, "lease job mismatch"),
                                 (other.buffer_ids != lease.buffer_ids, "lease buffer mismatch")):
                    if bad:
                        return fail(msg)
            adm_ids = {str(x) for x in S.admissions.get(req.transfer_id, {}).get("lease_ids", ()) or ()}
            if adm_ids and adm_ids != {l.lease_id for l in related}:
                return fail("worker lease set mismatch")
        try:
            ranges = relay_ranges(plan, tuple(l.relay_gpu for l in related), req.direction)
        except ValueError as exc:
            return fail(str(exc))
        if req.ranges and req.ranges != ranges:
            return fail("worker ranges do not match daemon plan")
        reserved = sum(int(S.reservations[l.lease_id].bytes) for l in related if l.lease_id in S.reservations)
        if sum(r["bytes"] for r in ranges) > reserved:
            return fail("authorization exceeds reservation bytes")
        if (req.src_buffer_id, req.dst_buffer_id) != lease.buffer_ids:
            return fail("lease buffer mismatch")
        src, dst = S.buffers.get(req.src_buffer_id), S.buffers.get(req.dst_buffer_id)
        if src is None or dst is None:
            return fail("unknown buffer")
        try:
            self._peer_owns_buffer(src.buffer_id, peer)
            self._peer_owns_buffer(dst.buffer_id, peer)
        except ValueError as exc:
            return fail(str(exc))
        auth = WorkerTransferAuthorization(transfer_id=req.transfer_id, lease_id=req.lease_id,
                                           session_id=req.session_id, job_id=req.job_id,
                                           src_buffer=src, dst_buffer=dst, direction=req.direction,
                                           ranges=ranges, relay_gpu=lease.relay_gpu, plan=plan)
        decision = S.decisions.get(req.transfer_id)
        if decision is None:
            return fail("scheduling decision is unavailable")
        exp = min(float(l.expires_at or (now + PLAN_TTL_SECONDS)) for l in related)
        if exp <= now:
            return fail("lease expired")
        ticket = self._plan_ticket(req.transfer_id, decision, auth.src_buffer.buffer_id,
                                   auth.dst_buffer.buffer_id, now, exp, tuple(l.lease_id for l in related))
        self._store_ticket(req.transfer_id, ticket)
        records = {}
        for l in related:
            rr = relay_ranges(plan, l.relay_gpu, req.direction)
            records[l.lease_id] = self._staging_record(l, req.transfer_id, req.direction, rr, now)
        for l in related:
            res = S.reservations.get(l.lease_id)
            if res is not None:
                build_audit_record(S, event_type="relay_authorized", transfer_id=req.transfer_id,
                                   reservation=res, lease=l, staging_record=records[l.lease_id],
                                   ticket=ticket, state=st.state, reason="worker_authorized",
                                   bytes_completed=st.bytes_completed, now=now)
        return ok(ticket=asdict(ticket), decision=asdict(decision), src_buffer=asdict(src),
                  dst_buffer=asdict(dst), relay_gpu=lease.relay_gpu,
                  relay_gpus=tuple(l.relay_gpu for l in related), lease_id=req.lease_id,
                  lease_ids=tuple(l.lease_id for l in related), transfer_id=req.transfer_id,
                  plan_generation=S.generations.get(req.transfer_id, 0),
                  staging_record=dict(records[lease.lease_id]),
                  staging_records=[dict(records[l.lease_id]) for l in related])

    # ---- planning --------------------------------------------------------------------------------
    def plan_transfer(self, session_id: str, total_bytes: int, chunk_bytes: int, mode: str = "pool",
                      direction: str = "h2d", job_id: str | None = None,
                      buffer_ids: Iterable[str] | None = None, ranges: Iterable[dict] | None = None,
                      intent_id: str | None = None, topology_snapshot_id: str | None = None,
                      workload_kind: str = "generic", priority: int = 0,
                      peer_identity: PeerIdentity | None = None,
                      allow_delayed_admission: bool = False, _for_intent: bool = False) -> DaemonResponse:
        now = self._now()
        try:
            rs = norm_ranges(ranges)
            if rs is not None and sum(r["bytes"] for r in rs) != int(total_bytes):
                return fail("range bytes must match total_bytes")
        except (KeyError, TypeError, ValueError) as exc:
            return fail(str(exc))
        with self._lock:
            self._reap(now)
            try:
                session, decision, bids, job, elig, relays, _snap = self._decide(
                    session_id=session_id, total_bytes=total_bytes, chunk_bytes=chunk_bytes, mode=mode,
                    direction=direction, job_id=job_id, buffer_ids=buffer_ids, ranges=rs,
                    intent_id=intent_id, topology_snapshot_id=topology_snapshot_id,
                    workload_kind=workload_kind, priority=priority, peer=peer_identity, now=now,
                    defer=allow_delayed_admission)
            except ValueError as exc:
                return fail(TOPOLOGY_UNAVAILABLE) if str(exc) == TOPOLOGY_UNAVAILABLE else fail(str(exc))
            S = self._st
            tid = str(uuid.uuid4())
            S.generations[tid] = 1
            adm = self._admission(decision, session, allow_delayed_admission, now)
            reservations = []
            if adm["state"] == ADMITTED:
                reservations = self._commit_leases(session, decision, tid, bids)
                adm["lease_ids"] = tuple(r.reservation_id for r in reservations)
            status = TransferStatus(transfer_id=tid, job_id=str(job or session.session_id),
                                    state=TransferStatusState.SUBMITTED, bytes_total=int(total_bytes),
                                    bytes_completed=0, session_id=session.session_id)
            S.statuses[tid] = status
            S.plans[tid] = dict(decision.plan)
            S.decisions[tid] = decision
            S.plan_requests[tid] = {
                "session_id": session.session_id, "total_bytes": int(total_bytes),
                "chunk_bytes": int(chunk_bytes), "mode": str(mode), "direction": str(direction).lower(),
                "job_id": None if job is None else str(job), "buffer_ids": bids, "ranges": rs,
                "intent_id": None if intent_id is None else str(intent_id),
                "topology_snapshot_id": topology_snapshot_id, "workload_kind": str(workload_kind),
                "priority": int(priority)}
            S.plan_expiry[tid] = self._plan_expiry(decision, now)
            S.admissions[tid] = {**adm, "plan_generation": 1, "plan_expires_at": S.plan_expiry[tid]}
            self._record_planned(tid, status, intent_id, bids, total_bytes, chunk_bytes, rs, direction,
                                 decision, now)
            self._touch(session.session_id, now)
            if not reservations and len(bids) >= 2 and direct_only(decision):
                tk = self._plan_ticket(tid, decision, bids[0], bids[1], now, None, ())
                self._store_ticket(tid, tk)
            if _for_intent:  # submit_transfer_intent answers with its own record of the decision
                return DaemonResponse(ok=True, payload=self._intent_planned_payload(tid, session, relays, elig,
                                                                                  reservations))
            return DaemonResponse(ok=True, payload=self._planned_payload(tid, decision, status, session,
                                                                         relays, elig, reservations))

    def reschedule_transfer(self, transfer_id: str, now: float | None = None) -> DaemonResponse:
        at = self._now() if now is None else float(now)
        with self._lock:
            resp = self._reschedule(str(transfer_id), at)
            self._changed.notify_all()
            return resp

    def _reschedule(self, tid: str, at: float) -> DaemonResponse:
        S = self._st
        self._reap(at)
        st = S.statuses.get(tid)
        if st is None:
            return fail("unknown transfer")
        if st.state in TERMINAL_STATES:
            return fail("transfer is terminal")
        req = S.plan_requests.get(tid)
        if req is None:
            return fail("transfer plan request is unavailable")
        self._release_for_transfer(tid, TransferStatusState.CANCELED, "reschedule", mark_terminal=False)
        try:
            session, decision, bids, _job, elig, relays, _snap = self._decide(
                session_id=str(req["session_id"]), total_bytes=int(req["total_bytes"]),
                chunk_bytes=int(req["chunk_bytes"]), mode=str(req["mode"]), direction=str(req["direction"]),
                job_id=req.get("job_id"), buffer_ids=req.get("buffer_ids"), ranges=req.get("ranges"),
                intent_id=req.get("intent_id"), topology_snapshot_id=req.get("topology_snapshot_id"),
                workload_kind=str(req.get("workload_kind", "generic")),
                priority=int(req.get("priority", 0) or 0), peer=None, now=at, defer=True,
                exclude=tid)
        except ValueError as exc:
            return fail(str(exc))
        gen = int(S.generations.get(tid, 0)) + 1
        S.generations[tid] = gen
        S.plans[tid] = dict(decision.plan)
        S.decisions[tid] = decision
        S.plan_expiry[tid] = self._plan_expiry(decision, at)
        adm = self._admission(decision, session, True, at, exclude=tid)
        reservations = []
        if adm["state"] == ADMITTED:
            reservations = self._commit_leases(session, decision, tid, bids)
            adm["lease_ids"] = tuple(r.reservation_id for r in reservations)
        S.admissions[tid] = {**adm, "plan_generation": gen, "plan_expires_at": S.plan_expiry[tid],
                             "rescheduled_at": float(at)}
        S.tickets.pop(S.transfer_tickets.pop(tid, ""), None)
        iid = req.get("intent_id")
        intent = None if iid is None else S.intents.get(str(iid))
        ticket = None
        if intent is not None and adm["state"] == ADMITTED:
            ticket = self._intent_ticket(intent, tid, decision, at)
            self._store_ticket(tid, ticket)
        self._refresh_record(tid, at)
        self._touch(session.session_id, at)
        payload = self._planned_payload(tid, decision, st, session, relays, elig, reservations)
        if ticket is not None:
            self._dispatch(tid, ticket)
        return DaemonResponse(ok=True, payload=payload)

    # ---- profiles ----------------------------------------------------------------------------------
    def get_profile(self, target_gpu: int, relay_gpus: Iterable[int]) -> DaemonResponse:
        key = profile_key(target_gpu, relay_gpus)
        with self._lock:
            self._purge_profiles(self._now())
            e = self._st.profiles.get(key)
            return ok(profile=dict(e) if e else None)

    def put_profile(self, target_gpu: int, relay_gpus: Iterable[int], profile: dict,
                    profile_bytes: int = 0, updated_at: float | None = None) -> DaemonResponse:
        target = int(target_gpu)
        relays = norm_relays(relay_gpus)
        try:
            norm = normalize_profile(profile, target)
        except (TypeError, ValueError) as exc:
            return fail(str(exc))
        entry = {"target_gpu": target, "relay_gpus": relays, "profile_bytes": int(profile_bytes),
                 "updated_at": float(self._now() if updated_at is None else updated_at), "profile": norm}
        with self._lock:
            self._purge_profiles(self._now())
            self._st.profiles[profile_key(target, relays)] = entry
            stored = self._save_profiles()
        if stored is not None:
            return ok(profile=dict(entry), profile_store_error=stored)
        return ok(profile=dict(entry))

    def invalidate_profile(self, target_gpu: int, relay_gpus: Iterable[int]) -> DaemonResponse:
        key = profile_key(target_gpu, relay_gpus)
        with self._lock:
            gone = self._st.profiles.pop(key, None)
            stored = self._save_profiles()
        extra = {} if stored is None else {"profile_store_error": stored}
        return ok(profile_key=key, removed=gone is not None, **extra)

    def _save_profiles(self) -> str | None:
        """Write the profile cache through to disk (temp file, fsync, atomic
        rename).  The in-memory cache stays authoritative: a failed write is
        logged and returned as a message, never raised, so a full or
        read-only disk cannot turn a profile update into a daemon error."""
        if not self._profile_store:
            return None
        tmp = f"{self._profile_store}.tmp"
        try:
            with open(tmp, "w", encoding="utf-8") as fh:
                json.dump({"format": PROFILE_STORE_FORMAT, "profiles": self._st.profiles}, fh, sort_keys=True)
                fh.flush()
                os.fsync(fh.fileno())
            os.replace(tmp, self._profile_store)
        except OSError as exc:
            msg = f"profile store not written: {exc}"
            _LOG.warning("profile_store_write_failed", path=self._profile_store, error=str(exc))
            return msg
        return None

    def _load_profiles(self, path: str) -> None:
        try:
            with open(path, encoding="utf-8") as fh:
                data = json.load(fh)
        except (OSError, ValueError):
            return
        if isinstance(data, dict) and data.get("format") == PROFILE_STORE_FORMAT:
            for key, entry in (data.get("profiles") or {}).items():
                if isinstance(entry, dict) and isinstance(entry.get("profile"), dict):
                    self._st.profiles[str(key)] = entry

    # ---- reaping / describe -----------------------------------------------------------------------
    def reap_stale_sessions(self, now: float | None = None) -> list[str]:
        with self._lock:
            out = self._reap_sessions(self._now() if now is None else float(now))
            self._changed.notify_all()
            return out

    def reap_expired_leases(self, now: float | None = None) -> list[str]:
        with self._lock:
            out = self._reap_leases(self._now() if now is None else float(now))
            self._changed.notify_all()
            return out

    def describe(self) -> DaemonResponse:
        with self._lock:
            now = self._now()
            self._reap(now)
            S = self._st
            return ok(
                jobs={k: asdict(v) for k, v in S.jobs.items()},
                job_peer_identities={k: asdict(v) for k, v in S.job_peers.items()},
                buffers={k: asdict(v) for k, v in S.buffers.items()},
                sessions={k: asdict(v) for k, v in S.sessions.items()},
                session_peer_identities={k: asdict(v) for k, v in S.session_peers.items()},
                reservations={k: asdict(v) for k, v in S.reservations.items()},
                staging_records={k: dict(v) for k, v in S.staging.items()},
                audit_records=[dict(r) for r in S.audit],
                connection_scoped_sessions=sorted(S.conn_sessions),
                transfer_statuses={k: asdict(v) for k, v in S.statuses.items()},
                transfer_queue=[dict(S.queue_records[t]) for t in S.queue if t in S.queue_records],
                runtime_resource_state=self._runtime_state(now),
                cleanup_events=[asdict(c) for c in S.cleanup_events],
                system_cleanup_events=[asdict(c) for c in S.system_cleanup_events],
                relay_quotas={k: {"relay_gpu": q.relay_gpu, "max_sessions": q.max_sessions,
                                  "max_inflight_chunks": q.max_inflight_chunks,
                                  "active_chunks": q.active_chunks, "sessions": sorted(q.sessions)}
                              for k, q in self._quotas.items()},
                profile_cache={k: dict(v) for k, v in S.profiles.items()},
                measured_transfers={k: dict(v) for k, v in S.measured.items()})

    # ---- executor callbacks -------------------------------------------------------------------------
    def executor_started(self, transfer_id: str) -> None:
        with self._lock:
            st = self._st.statuses.get(transfer_id)
            if st is not None and st.state is TransferStatusState.SUBMITTED:
                self._transfer_status(transfer_id, TransferStatusState.RUNNING.value, None, None)
                self._changed.notify_all()

    def executor_finished(self, transfer_id: str, *, ok_: bool, bytes_completed: int,
                          error: str | None = None, measured: dict | None = None) -> None:
        """Record the data plane's outcome: status, measured stats, leases."""
        m = measured or {}
        if ok_ and self._feedback is not None:
            self._observe_lanes(m)
        if ok_:
            _LOG.info("transfer_complete", transfer_id=transfer_id, bytes=int(bytes_completed),
                      cuda_ms=float(m.get("cuda_ms", 0.0) or 0.0), gb_per_s=float(m.get("gb_per_s", 0.0) or 0.0),
                      lanes=len(m.get("path_stats", ()) or ()), fallback=m.get("fallback_reason", ""))
        else:
            _LOG.warning("transfer_failed", transfer_id=transfer_id, bytes=int(bytes_completed), error=error or "")
        with self._lock:
            if measured:
                self._st.measured[transfer_id] = dict(measured)
            st = self._st.statuses.get(transfer_id)
            if st is None or st.state in TERMINAL_STATES:
                self._changed.notify_all()
                return
            if ok_:
                self._transfer_status(transfer_id, TransferStatusState.COMPLETE.value, bytes_completed, None)
                self._release_for_transfer(transfer_id, TransferStatusState.COMPLETE, None)
            else:
                self._transfer_status(transfer_id, TransferStatusState.FAILED.value,
                                      min(int(bytes_completed), st.bytes_total), error or "data plane failed")
            self._changed.notify_all()
            self._readmit_delayed()

    def _observe_lanes(self, m: Mapping) -> None:
        stats = m.get("path_stats") or ()
        if not stats or m.get("failover"):
            return
        rates: dict[int, float] = {}
        for p in stats:
            if not isinstance(p, Mapping) or float(p.get("cuda_ms", 0.0) or 0.0) <= 0.0:
                return
            dev = int(p["target_device"]) if int(p.get("relay_device", -1)) < 0 else int(p["relay_device"])
            rates[dev] = float(p.get("gib_per_second", 0.0) or 0.0)
        first = stats[0]
        key = f"{first.get('direction', 'h2d')}:{m.get('landing_op', 'copy')}"
        self._feedback.observe_rates(int(first.get("target_device", 0)), key, rates)

    def _refined_profile(self, entry, target: int, direction: str, intent) -> Mapping | None:
        """``entry`` with its concurrent ``direction`` lane rates replaced by
        the rates measured for this intent's landing op, when every lane of
        the profile has one; otherwise ``entry`` itself."""
        from ..scheduler.daemon import profile_payload

        payload = profile_payload(entry)
        if payload is None or self._feedback is None:
            return entry
        spec = LandingSpec.from_metadata(intent.metadata) if intent is not None else None
        key = (int(target), f"{direction}:{spec.op if spec is not None else 'copy'}")
        rates = self._feedback.rates(*key)
        if not rates:
            return entry
        # Publish new rates only when a lane moved by more than 4 %: the
        # split does not jitter with every measurement, and a repeated intent
        # shape keeps hitting the scheduler's plan cache.
        pub = self._published.get(key)
        if pub is not None and pub[0] is payload and set(pub[1]) == set(rates) and all(
                abs(rates[d] - pub[1][d]) <= 0.04 * pub[1][d] for d in rates):
            return pub[2]
        conc = dict(payload.get("concurrent") or {})
        block = conc.get(direction)
        lanes = ([int(x) for x in block["lanes"]] if isinstance(block, Mapping) and block.get("lanes") else
                 [int(payload.get("target_device", target))] +
                 [int(r["relay_device"]) for r in payload.get("relays", ()) or () if isinstance(r, Mapping)])
        if not all(d in rates for d in lanes):
            return entry
        conc[direction] = {**(dict(block) if isinstance(block, Mapping) else {}), "lanes": lanes,
                           "lane_gibps": {str(d): rates[d] for d in lanes}, "source": "measured lane feedback"}
        refined = {**payload, "concurrent": conc}
        self._published[key] = (payload, dict(rates), refined)
        return refined

    def _dispatch(self, tid: str, ticket: ExecutionTicket) -> None:
        if self._executor is None:
            return
        S = self._st
        src = S.buffers.get(ticket.source_buffer_id)
        dst = S.buffers.get(ticket.destination_buffer_id)
        intent = S.intents.get(ticket.intent_id)
        self._executor.submit(self, tid, ticket, src, dst, intent)

    def _readmit_delayed(self) -> None:
        """Re-plan delayed intents now that capacity may have been freed."""
        S = self._st
        for tid in list(S.live):
            adm = S.admissions.get(tid, {})
            st = S.statuses.get(tid)
            if adm.get("state") != DELAYED or st is None or st.state in TERMINAL_STATES:
                continue
            if not S.plan_requests.get(tid, {}).get("intent_id"):
                continue
            self._reschedule(tid, self._now())

    # ---- wire -------------------------------------------------------------------------------------
    def handle_request(self, request: DaemonRequest, connection_id: str | None = None,
                       fds: list[int] | None = None) -> DaemonResponse:
        """``fds``: descriptors that arrived with the request (valid in this
        process until the call returns; the daemon keeps duplicates)."""
        try:
            return self._dispatch_request(request, connection_id, fds or [])
        except (KeyError, TypeError, ValueError, OSError) as exc:
            return fail(f"invalid request: {exc}")

    def handle_wire_message(self, data: bytes | str, peer_identity: PeerIdentity | None = None,
                            connection_id: str | None = None, fds: list[int] | None = None) -> DaemonResponse:
        try:
            text = data.decode("utf-8") if isinstance(data, bytes) else str(data)
            obj = json.loads(text)
            if not isinstance(obj, dict):
                raise ValueError("request must be a JSON object")
            payload = obj.get("payload", {})
            if not isinstance(payload, dict):
                raise ValueError("payload must be a JSON object")
            req = DaemonRequest(request_type=RequestType(obj["request_type"]),
                                session_id=obj.get("session_id"), payload=payload,
                                peer_identity=peer_identity)
        except Exception as exc:  # noqa: BLE001 - every malformed message gets an error reply
            return fail(f"invalid request: {exc}")
        # a descriptor number in the JSON would name one of the daemon's own
        # files: over the socket only attached descriptors count
        md = payload.get("metadata") if isinstance(payload.get("metadata"), dict) else None
        if md is not None and "vmm_fd" in md:
            return fail("vmm_fd cannot be given in the request; attach the descriptor instead")
        return self.handle_request(req, connection_id=connection_id, fds=fds)

    def close_connection(self, peer_identity: PeerIdentity | None, connection_id: str | None,
                         reason: str = "socket_disconnect") -> dict[str, int]:
        with self._lock:
            removed = removed_summary()
            if peer_identity is None:
                return removed
            for sid in sorted(self._st.conn_sessions):
                if connection_id is not None and self._st.conn_session_conn.get(sid) != str(connection_id):
                    continue
                if not same_connection(self._st.session_peers.get(sid), peer_identity):
                    continue
                self._close_session(sid, reason, removed)
            self._changed.notify_all()
            return removed

    def serve_forever(self, socket_path: str, stop_event: threading.Event | None = None,
                      ready_event: threading.Event | None = None) -> None:
        from .wire import serve_unix

        serve_unix(self, socket_path, stop_event=stop_event, ready_event=ready_event)

    def _dispatch_request(self, r: DaemonRequest, conn_id: str | None, fds: list[int] | None = None) -> DaemonResponse:
        p = r.payload
        T = RequestType
        t = r.request_type
        if t == T.REGISTER_JOB:
            return self.register_job(job_id=str(p["job_id"]), user_id=p.get("user_id"),
                                     session_id=p.get("session_id"), container_id=p.get("container_id"),
                                     process_id=p.get("process_id"), weight=float(p.get("weight", 1.0)),
                                     peer_identity=r.peer_identity)
        if t == T.REGISTER_BUFFER:
            return self.register_buffer(
                buffer_id=str(p["buffer_id"]), job_id=str(p["job_id"]), kind=str(p.get("kind", "cpu_pinned")),
                size_bytes=int(p.get("size_bytes", 0)), device_index=p.get("device_index"),
                address=p.get("address"), pinned=bool(p.get("pinned", False)),
                handle_type=str(p.get("handle_type", "registered_buffer")), metadata=p.get("metadata") or {},
                peer_identity=r.peer_identity, fds=fds)
        if t == T.GET_INVENTORY:
            return self.get_inventory()
        if t == T.DISCOVER_RELAYS:
            tg = p.get("target_gpu")
            return self.discover_relays(None if tg is None else int(tg), p.get("relay_gpus"))
        if t == T.REAP_EXPIRED_LEASES:
            exp = self.reap_expired_leases(now=p.get("now"))
            return ok(expired_lease_ids=exp, expired_count=len(exp))
        if t == T.REGISTER_SESSION:
            return self.register_session(target_gpu=int(p["target_gpu"]), requested_relays=p.get("relay_gpus", []),
                                         max_inflight_chunks=int(p.get("max_inflight_chunks", 8)),
                                         peer_identity=r.peer_identity,
                                         connection_scoped=bool(p.get("connection_scoped", False)),
                                         connection_id=conn_id)
        if t == T.CLOSE_SESSION:
            if r.session_id is None:
                return fail("session_id is required")
            return self.close_session(r.session_id)
        if t in (T.RESERVE_TRANSFER, T.ISSUE_LEASE):
            if r.session_id is None:
                return fail("session_id is required")
            return self.reserve_transfer(session_id=r.session_id, relay_gpu=int(p["relay_gpu"]),
                                         chunks=int(p.get("chunks", 1)), bytes_=int(p.get("bytes", 0)),
                                         direction=str(p.get("direction", "unknown")))
        if t == T.PLAN_TRANSFER:
            if r.session_id is None:
                return fail("session_id is required")
            return self.plan_transfer(
                session_id=r.session_id, total_bytes=int(p.get("total_bytes", p.get("bytes", 0))),
                chunk_bytes=int(p.get("chunk_bytes", 16 * 1024 * 1024)), mode=str(p.get("mode", "pool")),
                direction=str(p.get("direction", "h2d")),
                job_id=str(p["job_id"]) if "job_id" in p else None, buffer_ids=p.get("buffer_ids"),
                ranges=p.get("ranges"), intent_id=p.get("intent_id"),
                topology_snapshot_id=p.get("topology_snapshot_id"),
                workload_kind=str(p.get("workload_kind", "generic")), priority=int(p.get("priority", 0)),
                peer_identity=r.peer_identity)
        if t == T.SUBMIT_TRANSFER_INTENT:
            ip = p.get("intent")
            if not isinstance(ip, dict):
                return fail("intent is required")
            return self.submit_transfer_intent(TransferIntent(**ip), peer_identity=r.peer_identity)
        if t == T.WAIT_TRANSFER_RECEIPT:
            return self.wait_transfer_receipt(str(p["intent_id"]), p.get("timeout_seconds"))
        if t == T.RESCHEDULE_TRANSFER:
            return self.reschedule_transfer(str(p["transfer_id"]), now=p.get("now"))
        if t == T.RELEASE_TRANSFER:
            rid = p.get("reservation_id")
            return fail("reservation_id is required") if rid is None else self.release_transfer(str(rid))
        if t == T.TRANSFER_STATUS:
            return self.transfer_status(str(p["transfer_id"]), p.get("state"), p.get("bytes_completed"),
                                        p.get("error"))
        if t == T.VALIDATE_LEASE:
            return self.validate_lease(lease_id=str(p["lease_id"]), token=str(p["token"]),
                                       session_id=p.get("session_id"), relay_gpu=p.get("relay_gpu"),
                                       job_id=p.get("job_id"), buffer_ids=p.get("buffer_ids"),
                                       peer_identity=r.peer_identity)
        if t == T.AUTHORIZE_WORKER_TRANSFER:
            return self.authorize_worker_transfer(WorkerTransferAuthorizationRequest(**p),
                                                  peer_identity=r.peer_identity)
        if t == T.CLEANUP:
            return self.cleanup(str(p["target_kind"]), str(p["target_id"]), str(p.get("reason", "manual")),
                                bool(p.get("force", False)))
        if t == T.INVALIDATE_PROFILE:
            return self.invalidate_profile(int(p["target_gpu"]), p.get("relay_gpus", []))
        if t == T.INVALIDATE_TOPOLOGY:
            return self.invalidate_topology()
        if t == T.GET_PROFILE:
            return self.get_profile(int(p["target_gpu"]), p.get("relay_gpus", []))
        if t == T.PUT_PROFILE:
            try:
                return self.put_profile(int(p["target_gpu"]), p.get("relay_gpus", []), p.get("profile", {}),
                                        int(p.get("profile_bytes", 0)), p.get("updated_at"))
            except Exception as exc:  # noqa: BLE001 - reported to the client
                return fail(str(exc))
        if t == T.PROFILE:
            return self.describe()
        return fail(f"unsupported request: {t}")

    # ================================================================================================
    # internals (caller holds the lock)
    # ================================================================================================
    def _reap(self, now: float) -> None:
        self._reap_sessions(now)
        self._reap_leases(now)
        self._purge_profiles(now)

    def _touch(self, sid: str, now: float | None = None) -> None:
        s = self._st.sessions.get(sid)
        if s is not None:
            s.last_seen = self._now() if now is None else float(now)

    def _reap_sessions(self, now: float) -> list[str]:
        if self._session_timeout <= 0.0:
            return []
        dead = [sid for sid, s in self._st.sessions.items()
                if s.active and s.last_seen > 0.0 and now - s.last_seen > self._session_timeout]
        for sid in dead:
            self._close_session(sid, "stale_session_timeout", None)
        return dead

    def _reap_leases(self, now: float) -> list[str]:
        dead = [lid for lid, l in self._st.leases.items() if l.expires_at and float(now) > l.expires_at]
        for lid in dead:
            self._expire_lease(lid)
        return dead

    def _purge_profiles(self, now: float) -> list[str]:
        if self._profile_max_age <= 0.0:
            return []
        dead = [k for k, e in self._st.profiles.items()
                if now - float(e.get("updated_at", 0.0) or 0.0) > self._profile_max_age]
        for k in dead:
            self._st.profiles.pop(k, None)
        return dead

    def _expire_lease(self, lid: str):
        res = self._release(lid, TransferStatusState.CANCELED, "lease_expired")
        if res is None:
            self._st.leases.pop(lid, None)
        return res

    def _peer_owns_job(self, job_id: str, peer: PeerIdentity | None) -> None:
        if peer is None or not peer.authenticated:
            return
        if self._st.jobs.get(str(job_id)) is None:
            raise ValueError("unknown job")
        owner = self._st.job_peers.get(str(job_id))
        if owner is None:
            raise ValueError("job owner identity is unavailable")
        same_owner(owner, peer, "job")

    def _peer_owns_buffer(self, buffer_id: str, peer: PeerIdentity | None) -> None:
        if peer is None or not peer.authenticated:
            return
        buf = self._st.buffers.get(str(buffer_id))
        if buf is None:
            raise ValueError("unknown buffer")
        try:
            self._peer_owns_job(buf.job_id, peer)
        except ValueError as exc:
            if str(exc) == "job owner does not match authenticated peer":
                raise ValueError("buffer owner does not match authenticated peer") from exc
            raise

    def _validate_buffers(self, buffer_ids, job_id, session_id, peer) -> tuple[tuple[str, ...], str | None]:
        if buffer_ids is None:
            return (), None
        ids = tuple(str(b) for b in buffer_ids)
        if not ids:
            return (), None
        if any(not b.strip() for b in ids):
            raise ValueError("buffer_ids must be non-empty")
        if len(set(ids)) != len(ids):
            raise ValueError("buffer_ids must be unique")
        owner = None if job_id is None else str(job_id)
        for b in ids:
            buf = self._st.buffers.get(b)
            if buf is None:
                raise ValueError(f"unknown buffer: {b}")
            owner = owner or buf.job_id
            if buf.job_id != owner:
                raise ValueError("buffer owner does not match job")
            self._peer_owns_buffer(b, peer)
        job = self._st.jobs.get(str(owner))
        if job is None:
            raise ValueError("unknown job")
        if job.session_id != session_id:
            raise ValueError("job session does not match transfer session")
        self._peer_owns_job(str(owner), peer)
        return ids, str(owner)

    def _buffer_leases(self, buffer_id: str) -> tuple[str, ...]:
        return tuple(lid for lid, l in sorted(self._st.leases.items())
                     if lid in self._st.reservations and str(buffer_id) in l.buffer_ids)

    def _decide(self, *, session_id, total_bytes, chunk_bytes, mode, direction, job_id, buffer_ids, ranges,
                intent_id, topology_snapshot_id, workload_kind, priority, peer, now, defer, exclude=None):
        S = self._st
        session = S.sessions.get(str(session_id))
        if session is None or not session.active:
            raise ValueError("unknown session")
        bids, owner = self._validate_buffers(buffer_ids, job_id, session.session_id, peer)
        if bids == () and job_id is not None:
            self._peer_owns_job(str(job_id), peer)
        if self._topology is None:
            raise ValueError(TOPOLOGY_UNAVAILABLE)
        snap = topology_snapshot_id or self._topology.snapshot().topology_snapshot_id()
        job = owner if owner is not None else job_id
        intent = None if intent_id is None else S.intents.get(str(intent_id))
        elig = self._eligibility(session.target_gpu, session.relay_gpus)
        relays = tuple(e["relay_gpu"] for e in elig["eligible_relays"])
        entry = S.profiles.get(profile_key(session.target_gpu, relays))
        if entry is None and relays != tuple(session.relay_gpus):
            entry = S.profiles.get(profile_key(session.target_gpu, session.relay_gpus))
        plan_session = session if relays == tuple(session.relay_gpus) else Session(
            session_id=session.session_id, target_gpu=session.target_gpu, relay_gpus=list(relays),
            max_inflight_chunks=session.max_inflight_chunks, active_chunks=session.active_chunks,
            active=session.active, created_at=session.created_at, last_seen=session.last_seen,
            closed_at=session.closed_at)
        entry = self._refined_profile(entry, session.target_gpu, str(direction).lower(), intent)
        state = self._runtime_state(now, active_only=True)
        if exclude is not None:
            state = state_without_transfer(state, str(exclude))
        lend = self._lendable(session.target_gpu)
        if lend:
            state = {**state, "lendable_relays": sorted(lend)}
        decision = self._scheduler.plan_transfer(
            session=plan_session, profile_entry=entry, relay_quotas=self._quotas, runtime_state=state,
            total_bytes=total_bytes, chunk_bytes=chunk_bytes,
            ranges=None if ranges is None else tuple(dict(r) for r in ranges), mode=mode,
            direction=direction, workload_kind=workload_kind if intent is None else intent.workload_kind,
            priority=priority if intent is None else intent.priority, now=now, job_id=job,
            intent_id=intent_id, topology_snapshot_id=snap, defer_relay_admission=defer)
        return session, decision, bids, job, elig, relays, snap

    def _eligibility(self, target: int, relays, inventory=None) -> dict[str, Any]:
        inv = inventory or self._topology.snapshot()
        e = inv.relay_eligibility(int(target), relays)
        good, filtered = [], list(e["filtered_relays"])
        for item in e["eligible_relays"]:
            g = int(item["relay_gpu"])
            if g in self._quotas:
                good.append({"relay_gpu": g, "reason": "eligible"})
            else:
                filtered.append({"relay_gpu": g, "reason": "relay not configured"})
        return {**e, "eligible_relays": good, "filtered_relays": filtered}

    def _admission(self, decision, session: Session, allow_delayed: bool, now: float,
                   exclude: str | None = None) -> dict[str, Any]:
        leases = scheduling_decision_leases(decision)
        if not leases:
            return {"state": ADMITTED, "reason": "direct_or_fallback_plan", "requested_lease_count": 0,
                    "requested_chunks": 0, "lease_ids": (), "admitted_at": float(now)}
        chunks = sum(l.chunk_limit for l in leases)
        why = self._admission_block(session, leases, exclude)
        if why is None:
            return {"state": ADMITTED, "reason": "relay_resources_available",
                    "requested_lease_count": len(leases), "requested_chunks": chunks, "lease_ids": (),
                    "admitted_at": float(now)}
        if allow_delayed:
            return {"state": DELAYED, "reason": why, "requested_lease_count": len(leases),
                    "requested_chunks": chunks, "lease_ids": (), "delayed_at": float(now)}
        return {"state": ADMITTED, "reason": "scheduler_fallback_or_rejection", "requested_lease_count": 0,
                "requested_chunks": 0, "lease_ids": (), "admitted_at": float(now)}

    def _admission_block(self, session: Session, leases, exclude: str | None = None) -> str | None:
        if session.active_chunks + sum(l.chunk_limit for l in leases) > session.max_inflight_chunks:
            return "session relay admission is delayed by chunk quota"
        state = self._runtime_state(active_only=True)
        if exclude is not None:  # a transfer being re-planned does not wait on its own old paths
            state = state_without_transfer(state, str(exclude))
        # A session's next intent in the same direction to the same target may
        # queue behind its own running transfer on the relays that session
        # already holds (the data plane runs them in submit order on those
        # lanes); another tenant's active path still blocks.
        dirs = {str(l.direction).lower() for l in leases}
        busy = busy_relays(state, queue_behind=(session.session_id, session.target_gpu, dirs))
        busy -= self._lendable(session.target_gpu)
        for l in leases:
            if l.relay_device not in session.relay_gpus:
                return "relay admission is delayed by session relay ownership"
            q = self._quotas.get(l.relay_device)
            if q is None:
                return "relay admission is delayed by missing relay quota"
            if not q.can_reserve(l.chunk_limit):
                return "relay admission is delayed by relay chunk quota"
            if int(l.relay_device) in busy:
                return "relay admission is delayed by active relay path"
        return None

    def _admission_error(self, tid: str, lease_id: str | None, now: float) -> str | None:
        adm = self._st.admissions.get(str(tid))
        if adm is None:
            return "transfer admission state is unavailable"
        if adm.get("state") == DELAYED:
            return "transfer admission is delayed"
        if adm.get("state") == EXPIRED:
            return "transfer plan expired"
        exp = self._st.plan_expiry.get(str(tid))
        if exp is not None and float(now) > float(exp):
            adm["state"] = EXPIRED
            adm["expired_at"] = float(now)
            self._refresh_record(str(tid), now)
            return "transfer plan expired"
        if lease_id is not None:
            lg = self._st.lease_generation.get(str(lease_id))
            if lg is None:
                return "lease plan generation is unavailable"
            if lg != self._st.generations.get(str(tid)):
                return "stale execution plan"
        return None

    def _plan_expiry(self, decision, now: float) -> float:
        exps = [float(l.expires_at) for l in scheduling_decision_leases(decision) if float(l.expires_at) > now]
        return min(exps) if exps else float(now) + PLAN_TTL_SECONDS

    def _commit_leases(self, session: Session, decision, tid: str | None, bids) -> list[TransferReservation]:
        out = []
        for l in scheduling_decision_leases(decision):
            r = TransferReservation(reservation_id=l.lease_id, session_id=l.session_id,
                                    relay_gpu=l.relay_device, chunks=l.chunk_limit, bytes=l.bytes_limit,
                                    direction=l.direction)
            self._st.reservations[r.reservation_id] = r
            self._st.leases[r.reservation_id] = LeaseToken(
                lease_id=r.reservation_id, session_id=r.session_id, relay_gpu=r.relay_gpu,
                token=str(uuid.uuid4()), buffer_ids=tuple(bids), job_id=l.job_id, issued_at=l.granted_at,
                expires_at=l.expires_at)
            if tid is not None:
                self._st.lease_generation[r.reservation_id] = self._st.generations.get(str(tid), 0)
                self._st.reservation_transfer[r.reservation_id] = tid
            session.active_chunks += r.chunks
            q = self._quotas.get(r.relay_gpu)
            if q is not None:
                q.active_chunks += r.chunks
            out.append(r)
        return out

    def _release(self, rid: str, final=TransferStatusState.COMPLETE, reason: str | None = None,
                 mark_terminal: bool = True) -> TransferReservation | None:
        S = self._st
        rid = str(rid)
        res = S.reservations.get(rid)
        if res is None:
            return None
        tid = S.reservation_transfer.get(rid)
        if reason is not None:
            build_audit_record(S, event_type="cleanup", transfer_id=tid, reservation=res,
                               lease=S.leases.get(rid), staging_record=S.staging.get(rid), state=final,
                               reason=reason,
                               failure_reason=reason if final in (TransferStatusState.FAILED,
                                                                  TransferStatusState.CANCELED) else None,
                               cleanup_kind="reservation", cleanup_target_id=rid)
        for d in (S.reservations, S.leases, S.lease_generation, S.staging):
            d.pop(rid, None)
        tid = S.reservation_transfer.pop(rid, None)
        s = S.sessions.get(res.session_id)
        if s is not None:
            s.active_chunks = max(0, s.active_chunks - res.chunks)
        q = self._quotas.get(res.relay_gpu)
        if q is not None:
            q.active_chunks = max(0, q.active_chunks - res.chunks)
        if tid is not None and mark_terminal:
            self._terminal_if_unblocked(tid, final)
        if reason is not None:
            S.system_cleanup_events.append(CleanupRequest("reservation", rid, reason, True))
        return res

    def _release_counted(self, rid: str, final, reason: str | None = None, mark_terminal: bool = True) -> dict:
        S = self._st
        out = removed_summary()
        tid = S.reservation_transfer.get(str(rid))
        before = None if tid is None else S.statuses.get(tid)
        had_staging = str(rid) in S.staging
        if self._release(str(rid), final, reason, mark_terminal) is not None:
            out["reservations"] += 1
        if had_staging:
            out["staging_records"] += 1
        if before is not None and before.state not in TERMINAL_STATES:
            after = S.statuses.get(before.transfer_id)
            if after is not None and after.state in TERMINAL_STATES:
                out["transfers"] += 1
        return out

    def _release_for_transfer(self, tid: str, final, reason: str | None, mark_terminal: bool = True) -> dict:
        out = removed_summary()
        for rid, t in list(self._st.reservation_transfer.items()):
            if t == str(tid):
                merge_removed(out, self._release_counted(rid, final, reason, mark_terminal))
        return out

    def _terminal_if_unblocked(self, tid: str, final) -> None:
        if any(v == tid for v in self._st.reservation_transfer.values()):
            return
        st = self._st.statuses.get(tid)
        if st is None or st.state in TERMINAL_STATES:
            return
        done = st.bytes_total if final is TransferStatusState.COMPLETE else st.bytes_completed
        self._st.statuses[tid] = TransferStatus(st.transfer_id, st.job_id, final, st.bytes_total, done,
                                                st.session_id, st.error)
        self._st.completed_at.setdefault(tid, self._now())
        self._refresh_record(tid)

    def _terminal(self, tid: str, final, error: str | None = None) -> TransferStatus:
        st = self._st.statuses.get(str(tid))
        if st is None:
            raise ValueError("unknown transfer")
        if st.state in TERMINAL_STATES:
            return st
        done = st.bytes_total if final is TransferStatusState.COMPLETE else st.bytes_completed
        new = TransferStatus(st.transfer_id, st.job_id, final, st.bytes_total, done, st.session_id,
                             st.error if error is None else error)
        self._st.statuses[new.transfer_id] = new
        self._st.completed_at.setdefault(new.transfer_id, self._now())
        self._refresh_record(new.transfer_id)
        return new

    def _cancel_if_active(self, tid: str, reason: str) -> bool:
        st = self._st.statuses.get(tid)
        if st is None or st.state in TERMINAL_STATES:
            return False
        self._terminal(tid, TransferStatusState.CANCELED, reason)
        if self._executor is not None:
            cancel = getattr(self._executor, "cancel", None)
            if callable(cancel):
                cancel(tid)
        return True

    def _close_session(self, sid: str, reason: str, removed: dict | None) -> Session | None:
        S = self._st
        s = S.sessions.pop(sid, None)
        if s is None:
            return None
        s.active = False
        s.closed_at = self._now()
        build_audit_record(S, event_type="cleanup", session_id=sid, state=TransferStatusState.CANCELED,
                           reason=reason, failure_reason=reason, cleanup_kind="session", cleanup_target_id=sid)
        S.system_cleanup_events.append(CleanupRequest("session", sid, reason, True))
        transfers = self._transfers_for_session(sid)
        for rid, res in list(S.reservations.items()):
            if res.session_id == sid:
                merge_removed(removed, self._release_counted(rid, TransferStatusState.CANCELED, reason))
        for t in transfers:
            if self._cancel_if_active(t, reason) and removed is not None:
                removed["transfers"] += 1
        for g in s.relay_gpus:
            q = self._quotas.get(g)
            if q is not None:
                q.sessions.discard(sid)
        S.conn_sessions.discard(sid)
        S.conn_session_conn.pop(sid, None)
        jobs = {j for j, job in S.jobs.items() if job.session_id == sid}
        nb = 0
        for j in jobs:
            S.jobs.pop(j, None)
            S.job_peers.pop(j, None)
        for b, buf in list(S.buffers.items()):
            if buf.job_id in jobs:
                self._drop_buffer(b)
                nb += 1
        S.session_peers.pop(sid, None)
        if removed is not None:
            removed["sessions"] += 1
            removed["jobs"] += len(jobs)
            removed["buffers"] += nb
        return s

    def _cleanup_job(self, job_id: str, reason: str) -> dict:
        S = self._st
        out = removed_summary()
        if S.jobs.pop(str(job_id), None) is not None:
            out["jobs"] += 1
        S.job_peers.pop(str(job_id), None)
        transfers = self._transfers_for_job(str(job_id))
        for rid, l in list(S.leases.items()):
            if l.job_id == str(job_id):
                merge_removed(out, self._release_counted(rid, TransferStatusState.CANCELED, reason))
        for t in transfers:
            if self._cancel_if_active(t, reason):
                out["transfers"] += 1
        for b, buf in list(S.buffers.items()):
            if buf.job_id == str(job_id):
                self._drop_buffer(b)
                out["buffers"] += 1
        return out

    def _transfers_for_job(self, job_id: str) -> tuple[str, ...]:
        S = self._st
        out = {t for t, st in S.statuses.items() if st.job_id == job_id}
        out |= {S.intent_transfer[i] for i, it in S.intents.items() if it.job_id == job_id and i in S.intent_transfer}
        out |= {S.reservation_transfer[r] for r, l in S.leases.items()
                if l.job_id == job_id and r in S.reservation_transfer}
        return tuple(sorted(out))

    def _transfers_for_session(self, sid: str) -> tuple[str, ...]:
        S = self._st
        out = {t for t, st in S.statuses.items() if st.session_id == sid}
        out |= {S.intent_transfer[i] for i, it in S.intents.items() if it.session_id == sid and i in S.intent_transfer}
        return tuple(sorted(out))

    def _transfers_for_buffer(self, bid: str) -> tuple[str, ...]:
        S = self._st
        out = {S.intent_transfer[i] for i, it in S.intents.items()
               if bid in (it.source_buffer_id, it.destination_buffer_id) and i in S.intent_transfer}
        out |= {S.reservation_transfer[r] for r, l in S.leases.items()
                if bid in l.buffer_ids and r in S.reservation_transfer}
        return tuple(sorted(out))

    def _worker_leases(self, req, primary: LeaseToken) -> tuple[LeaseToken, ...]:
        if req.ranges:
            return (primary,)
        plan = self._st.plans.get(req.transfer_id)
        if plan is None:
            return (primary,)
        relays = relay_devices(plan, req.direction)
        if not relays or primary.relay_gpu not in relays:
            return (primary,)
        related = [self._st.leases[r] for r, t in sorted(self._st.reservation_transfer.items())
                   if t == req.transfer_id and r in self._st.leases and self._st.leases[r].relay_gpu in relays]
        if primary.lease_id not in {l.lease_id for l in related}:
            related.append(primary)
        if {l.relay_gpu for l in related} != relays:
            raise ValueError("worker relay lease set mismatch")
        return tuple(sorted(related, key=lambda l: (int(l.relay_gpu), str(l.lease_id))))

    def _staging_record(self, lease: LeaseToken, tid: str, direction: str, ranges, now: float) -> dict:
        rec = {"staging_record_id": f"staging-{lease.lease_id}", "lease_id": lease.lease_id,
               "transfer_id": str(tid), "session_id": lease.session_id, "job_id": lease.job_id,
               "relay_gpu": lease.relay_gpu, "buffer_ids": lease.buffer_ids,
               "direction": str(direction).lower(), "ranges": tuple(dict(r) for r in ranges),
               "requested_bytes": sum(r["bytes"] for r in ranges), "state": "authorized",
               "created_at": float(now)}
        self._st.staging[lease.lease_id] = rec
        return rec

    def _intent_ticket(self, intent: TransferIntent, tid: str, decision, now: float) -> ExecutionTicket:
        lids = tuple(r for r, t in sorted(self._st.reservation_transfer.items()) if t == tid)
        exp = max([now + PLAN_TTL_SECONDS] + [float(self._st.leases[l].expires_at) for l in lids
                                              if l in self._st.leases and self._st.leases[l].expires_at > now])
        return self._plan_ticket(tid, decision, intent.source_buffer_id, intent.destination_buffer_id, now, exp, lids)

    def _plan_ticket(self, tid: str, decision, src: str, dst: str, now: float, expires_at: float | None,
                     lease_ids: tuple[str, ...]) -> ExecutionTicket:
        d = decision_direction(decision)
        ranges = ticket_ranges(decision.plan, d)
        exp = float(expires_at) if expires_at is not None else float(
            self._st.plan_expiry.get(str(tid), now + PLAN_TTL_SECONDS))
        if exp <= now:
            exp = now + PLAN_TTL_SECONDS
        return ExecutionTicket(
            ticket_id=f"ticket-{tid}", decision_id=decision.decision_id, intent_id=decision.intent_id,
            topology_snapshot_id=decision.topology_snapshot_id, job_id=decision.job_id,
            session_id=decision.session_id, source_buffer_id=src, destination_buffer_id=dst, direction=d,
            total_bytes=sum(r["bytes"] for r in ranges), ranges=ranges, plan=dict(decision.plan),
            issued_at=float(now), expires_at=exp, lease_ids=lease_ids,
            metadata={"issuer": TICKET_ISSUER, "transfer_id": tid,
                      "plan_generation": self._st.generations.get(str(tid), 0)})

    def _receipt(self, intent_id: str) -> TransferReceipt:
        S = self._st
        tid = S.intent_transfer.get(str(intent_id))
        if tid is None:
            raise ValueError("unknown transfer intent")
        intent = S.intents.get(str(intent_id))
        st = S.statuses.get(tid)
        decision = S.decisions.get(tid)
        if intent is None:
            raise ValueError("transfer intent is unavailable")
        if st is None:
            raise ValueError("transfer status is unavailable")
        if decision is None:
            raise ValueError("scheduling decision is unavailable")
        tk = S.tickets.get(S.transfer_tickets.get(tid, ""))
        err = st.error
        if st.state in (TransferStatusState.FAILED, TransferStatusState.CANCELED):
            err = err or f"transfer {st.state.value}"
        adm = S.admissions.get(tid, {})
        measured = S.measured.get(tid)
        md = {"transfer_id": tid, "fallback_reason": decision.fallback_reason,
              "admission_state": adm.get("state", ADMITTED), "admission_reason": adm.get("reason"),
              "plan_generation": S.generations.get(tid, 0), "plan_expires_at": S.plan_expiry.get(tid)}
        if measured:
            md["measured"] = {k: v for k, v in measured.items() if k != "path_stats"}
        done_at = S.completed_at.get(tid) if st.state in TERMINAL_STATES else None
        md["timing"] = transfer_timing(S.queue_records.get(tid) or {}, done_at)
        started = decision.issued_at
        if done_at is not None and done_at < started:
            done_at = started
        return TransferReceipt(
            receipt_id=f"receipt-{tid}", ticket_id=tk.ticket_id if tk else f"ticket-pending-{tid}",
            intent_id=intent.intent_id, decision_id=decision.decision_id,
            topology_snapshot_id=decision.topology_snapshot_id, job_id=intent.job_id,
            session_id=intent.session_id, state=st.state, bytes_total=st.bytes_total,
            bytes_completed=st.bytes_completed, started_at=started, completed_at=done_at,
            path_stats=tuple(measured["path_stats"]) if measured and measured.get("path_stats") else decision.path_summary,
            error=err, metadata=md)

    def _intent_planned_payload(self, tid, session, relays, elig, reservations) -> dict:
        """The parts of a plan answer that an intent submission passes on."""
        S = self._st
        return {"admission": dict(S.admissions.get(str(tid), {})),
                "plan_generation": S.generations.get(str(tid), 0), "plan_expires_at": S.plan_expiry.get(str(tid)),
                "transfer_id": str(tid),
                "planning": {"target_gpu": session.target_gpu, "profile_key": profile_key(session.target_gpu, relays),
                             "relay_eligibility": elig},
                "reservations": [asdict(r) for r in reservations],
                "lease_tokens": [asdict(S.leases[r.reservation_id]) for r in reservations
                                 if r.reservation_id in S.leases]}

    def _planned_payload(self, tid, decision, status, session, relays, elig, reservations) -> dict:
        S = self._st
        payload = {
            "decision": asdict(decision), "decision_id": decision.decision_id,
            "topology_snapshot_id": decision.topology_snapshot_id, "plan": dict(decision.plan),
            "path_summary": list(decision.path_summary), "stats": scheduling_decision_stats(decision).as_dict(),
            "leases": [l.as_dict() for l in scheduling_decision_leases(decision)],
            "admission": dict(S.admissions.get(str(tid), {})),
            "plan_generation": S.generations.get(str(tid), 0), "plan_expires_at": S.plan_expiry.get(str(tid)),
            "transfer_id": str(tid), "transfer_status": asdict(status),
            "planning": {"target_gpu": session.target_gpu, "profile_key": profile_key(session.target_gpu, relays),
                         "relay_eligibility": elig},
            "reservations": [asdict(r) for r in reservations],
            "lease_tokens": [asdict(S.leases[r.reservation_id]) for r in reservations if r.reservation_id in S.leases],
        }
        tk = S.transfer_tickets.get(str(tid))
        payload["ticket"] = None if tk is None else asdict(S.tickets[tk])
        return payload

    def _audit_transfer(self, event: str, tid: str, state, *, reason=None, failure_reason=None,
                        bytes_completed=None) -> None:
        S = self._st
        res = [S.reservations[r] for r, t in sorted(S.reservation_transfer.items()) if t == tid and r in S.reservations]
        if not res:
            build_audit_record(S, event_type=event, transfer_id=tid, state=state, reason=reason,
                               failure_reason=failure_reason, bytes_completed=bytes_completed)
        for r in res:
            build_audit_record(S, event_type=event, transfer_id=tid, reservation=r, lease=S.leases.get(r.reservation_id),
                               staging_record=S.staging.get(r.reservation_id), state=state, reason=reason,
                               failure_reason=failure_reason, bytes_completed=bytes_completed)

    # ---- queue records / runtime state -------------------------------------------------------------------
    def _record_planned(self, tid, status, intent_id, bids, total, chunk, ranges, direction, decision, now):
        S = self._st
        adm = S.admissions.get(tid, {})
        S.queue[tid] = None
        S.live[tid] = None
        S.queue_records[tid] = {
            "transfer_id": tid, "intent_id": None if intent_id is None else str(intent_id),
            "decision_id": decision.decision_id, "topology_snapshot_id": decision.topology_snapshot_id,
            "job_id": status.job_id, "session_id": status.session_id, "state": status.state.value,
            "direction": str(direction).lower(), "bytes_total": int(total),
            "bytes_completed": status.bytes_completed, "chunk_bytes": int(chunk),
            "ranges": tuple(dict(r) for r in ranges) if ranges is not None else (),
            "source_buffer_id": bids[0] if len(bids) >= 1 else None,
            "destination_buffer_id": bids[1] if len(bids) >= 2 else None, "buffer_ids": bids,
            # the plan request's kind and priority (an intent's own values replace them on refresh)
            "workload_kind": S.plan_requests.get(tid, {}).get("workload_kind"),
            "priority": int(S.plan_requests.get(tid, {}).get("priority", 0) or 0),
            "queued_at": float(now), "planned_at": decision.issued_at,
            "admission_state": adm.get("state", ADMITTED), "admission_reason": adm.get("reason"),
            "plan_generation": S.generations.get(tid, 0), "plan_expires_at": S.plan_expiry.get(tid),
            "started_at": None, "completed_at": None, "fallback_reason": decision.fallback_reason,
            "target_devices": plan_targets(decision.plan)}
        for g in S.queue_records[tid]["target_devices"]:
            S.target_seen[g] = float(now)
        self._refresh_record(tid, now)
        S.version += 1

    _SIG = ("state", "bytes_completed", "error", "intent_id", "source_buffer_id", "destination_buffer_id",
            "workload_kind", "priority", "admission_state", "plan_generation", "plan_expires_at",
            "started_at", "completed_at")

    def _store_ticket(self, tid: str, ticket: ExecutionTicket) -> None:
        S = self._st
        S.tickets[ticket.ticket_id] = ticket
        S.transfer_tickets[str(tid)] = ticket.ticket_id
        S.ticket_ids.setdefault(str(tid), []).append(ticket.ticket_id)

    def _trim_history(self) -> None:
        """Forget the oldest finished transfers beyond ``history_limit`` (a
        transfer whose leases are still held is kept until they are released)
        and the oldest audit / cleanup records beyond ``audit_limit``."""
        S = self._st
        held = None
        skipped = []
        while len(S.terminal_order) > self._history_limit:
            tid = S.terminal_order.popleft()
            if tid in S.live:
                continue
            if held is None:
                held = set(S.reservation_transfer.values())
            if tid in held:
                skipped.append(tid)
                if len(skipped) > 64:
                    break
                continue
            self._forget_transfer(tid)
        S.terminal_order.extendleft(reversed(skipped))
        for lst in (S.audit, S.cleanup_events, S.system_cleanup_events):
            if len(lst) > self._audit_limit + self._audit_limit // 8:
                del lst[:len(lst) - self._audit_limit]

    def _forget_transfer(self, tid: str) -> None:
        S = self._st
        req = S.plan_requests.get(tid) or {}
        iid = req.get("intent_id")
        if iid is not None and S.intent_transfer.get(str(iid)) == tid:
            S.intent_transfer.pop(str(iid), None)
            S.intents.pop(str(iid), None)
        for tk in S.ticket_ids.pop(tid, ()):
            S.tickets.pop(tk, None)
        for d in (S.queue, S.queue_records, S.statuses, S.plans, S.decisions, S.plan_requests, S.admissions,
                  S.generations, S.plan_expiry, S.completed_at, S.measured, S.transfer_tickets):
            d.pop(tid, None)

    def _refresh_record(self, tid: str, now: float | None = None) -> dict | None:
        S = self._st
        rec = S.queue_records.get(str(tid))
        st = S.statuses.get(str(tid))
        if rec is None or st is None:
            return rec
        before = tuple(rec.get(k) for k in self._SIG)
        rec["state"] = st.state.value
        rec["bytes_completed"] = st.bytes_completed
        adm = S.admissions.get(str(tid), {})
        if adm:
            rec["admission_state"] = adm.get("state", rec.get("admission_state"))
            rec["admission_reason"] = adm.get("reason")
            at0 = float(self._now() if now is None else now)
            if rec["admission_state"] == DELAYED and rec.get("delayed_at") is None:
                rec["delayed_at"] = at0
            elif rec["admission_state"] == ADMITTED and rec.get("delayed_at") is not None \
                    and rec.get("admitted_at") is None:
                rec["admitted_at"] = at0
        rec["plan_generation"] = S.generations.get(str(tid), rec.get("plan_generation", 0))
        rec["plan_expires_at"] = S.plan_expiry.get(str(tid), rec.get("plan_expires_at"))
        d = S.decisions.get(str(tid))
        if d is not None:
            rec["decision_id"] = d.decision_id
            rec["topology_snapshot_id"] = d.topology_snapshot_id
            rec["fallback_reason"] = d.fallback_reason
        if st.error is not None:
            rec["error"] = st.error
        at = float(self._now() if now is None else now)
        if st.state is TransferStatusState.RUNNING and rec.get("started_at") is None:
            rec["started_at"] = at
        if st.state in TERMINAL_STATES and rec.get("completed_at") is None:
            rec["completed_at"] = at
            for g in rec.get("target_devices", ()) or ():
                S.target_seen[int(g)] = max(at, S.target_seen.get(int(g), at))
        if st.state in TERMINAL_STATES and S.live.pop(str(tid), 0) is None:
            S.terminal_order.append(str(tid))
            self._trim_history()
        it = S.intents.get(str(rec.get("intent_id"))) if rec.get("intent_id") is not None else None
        if it is not None:
            rec.update(intent_id=it.intent_id, source_buffer_id=it.source_buffer_id,
                       destination_buffer_id=it.destination_buffer_id,
                       buffer_ids=(it.source_buffer_id, it.destination_buffer_id),
                       workload_kind=it.workload_kind.value, priority=it.priority)
        if tuple(rec.get(k) for k in self._SIG) != before:
            S.version += 1
        return rec

    def _runtime_state(self, now: float | None = None, active_only: bool = False) -> dict[str, Any]:
        """Resource state over the queued transfers.  ``active_only`` (what
        planning and admission need) covers only non-terminal transfers, so its
        cost does not grow with the daemon's history; ``describe`` reports the
        retained history as well."""
        S = self._st
        at = float(self._now() if now is None else now)
        for t in tuple(S.live):
            self._refresh_record(t, at)
        ids = S.live if active_only else S.queue
        recs = [dict(S.queue_records[t]) for t in ids if t in S.queue_records]
        sub, run = TransferStatusState.SUBMITTED.value, TransferStatusState.RUNNING.value
        queued = [r for r in recs if r.get("state") == sub]
        running = [r for r in recs if r.get("state") == run]
        active = [r for r in recs if r.get("state") in (sub, run)]
        by_dir: dict[str, dict[str, int]] = {}
        q_dir: dict[str, dict[str, int]] = {}
        for r in active:
            b = by_dir.setdefault(str(r.get("direction", "unknown")),
                                  {"transfer_count": 0, "bytes_total": 0, "bytes_remaining": 0})
            b["transfer_count"] += 1
            b["bytes_total"] += int(r.get("bytes_total", 0) or 0)
            b["bytes_remaining"] += max(0, int(r.get("bytes_total", 0) or 0) - int(r.get("bytes_completed", 0) or 0))
        for r in queued:
            b = q_dir.setdefault(str(r.get("direction", "unknown")), {"transfer_count": 0, "bytes_total": 0})
            b["transfer_count"] += 1
            b["bytes_total"] += int(r.get("bytes_total", 0) or 0)
        paths, path_sum = self._active_paths(active)
        reservations = []
        for rid, res in sorted(S.reservations.items()):
            rec = asdict(res)
            l = S.leases.get(rid)
            rec.update(transfer_id=S.reservation_transfer.get(rid), job_id=None if l is None else l.job_id,
                       buffer_ids=() if l is None else l.buffer_ids)
            reservations.append(rec)
        leases = [{"lease_id": l.lease_id, "session_id": l.session_id, "relay_gpu": l.relay_gpu,
                   "job_id": l.job_id, "buffer_ids": l.buffer_ids, "issued_at": l.issued_at,
                   "expires_at": l.expires_at, "transfer_id": S.reservation_transfer.get(lid)}
                  for lid, l in sorted(S.leases.items()) if lid in S.reservations]
        staging = [dict(v) for _, v in sorted(S.staging.items())]
        jobs = job_runtime_state({j: job.weight for j, job in S.jobs.items()}, recs)
        relay_sum = {"path_count": 0, "chunk_count": 0, "bytes_total": 0}
        for k, v in path_sum.items():
            if k.endswith(":relay"):
                for kk in relay_sum:
                    relay_sum[kk] += int(v.get(kk, 0) or 0)
        usage = {"h2d": dict(by_dir.get("h2d", {})), "d2h": dict(by_dir.get("d2h", {})), "p2p": dict(relay_sum),
                 "relay_staging": {"count": len(staging), "active_reservation_count": len(reservations),
                                   "active_lease_count": len(leases)}}
        terminal = {s.value for s in TERMINAL_STATES}
        recent = sorted(g for g, t in S.target_seen.items() if self._link_hold > 0 and at - t <= self._link_hold)
        return {
            "version": S.version, "captured_at": at, "transfer_order": tuple(S.queue), "transfers": recs,
            "recent_targets": recent, "link_hold_seconds": self._link_hold,
            "queued_transfers": queued, "running_transfers": running, "active_transfers": active,
            "active_paths": paths, "active_resource_usage": usage, "job_runtime_state": jobs,
            "active_reservations": reservations, "active_leases": leases, "relay_staging": staging,
            "summary": {
                "queued_transfer_count": len(queued), "running_transfer_count": len(running),
                "active_transfer_count": len(active),
                "terminal_transfer_count": sum(1 for r in recs if r.get("state") in terminal),
                "active_reservation_count": len(reservations), "active_lease_count": len(leases),
                "relay_staging_count": len(staging), "relay_path_count": relay_sum["path_count"],
                "relay_path_bytes_total": relay_sum["bytes_total"], "queued_bytes_by_direction": q_dir,
                "active_bytes_by_direction": by_dir, "active_paths": path_sum,
                "active_resource_usage": usage, "job_runtime_state": jobs}}

    def _active_paths(self, active) -> tuple[list[dict], dict[str, dict[str, int]]]:
        S = self._st
        recs: list[dict] = []
        summ: dict[str, dict[str, int]] = {}
        for tid in sorted({str(r["transfer_id"]) for r in active}):
            if S.admissions.get(tid, {}).get("state") != ADMITTED:
                continue
            d = S.decisions.get(tid)
            if d is None:
                continue
            for a in d.plan.get("assignments", ()) or ():
                if not isinstance(a, Mapping) or not isinstance(a.get("path"), Mapping):
                    continue
                p = a["path"]
                nchunks = assignment_chunk_count(a)
                nbytes = int(a.get("bytes", 0) or 0) or assignment_bytes(a)
                kind, dirn = str(p.get("kind", "unknown")), str(p.get("direction", "unknown"))
                b = summ.setdefault(f"{dirn}:{kind}", {"path_count": 0, "chunk_count": 0, "bytes_total": 0})
                b["path_count"] += 1
                b["chunk_count"] += nchunks
                b["bytes_total"] += nbytes
                recs.append({"transfer_id": tid, "kind": kind, "direction": dirn,
                             "target_device": p.get("target_device"), "relay_device": p.get("relay_device"),
                             "bytes_total": nbytes, "chunk_count": nchunks, "session_id": d.session_id})
        return recs, summ

    def _discovery(self, inv, target: int | None, cands: tuple[int, ...]) -> dict[str, Any]:
        if target is None:
            elig = {"requested_relays": list(cands), "eligible_relays": [], "filtered_relays": [],
                    "inventory_source": inv.source, "inventory_discovered_at": inv.discovered_at}
            by = {g: {"eligible": None, "reason": "target_gpu not provided"} for g in cands}
        else:
            elig = self._eligibility(target, cands, inv)
            by = {int(e["relay_gpu"]): {"eligible": True, "reason": str(e.get("reason", "eligible"))}
                  for e in elig["eligible_relays"]}
            by.update({int(e["relay_gpu"]): {"eligible": False, "reason": str(e.get("reason", "filtered"))}
                       for e in elig["filtered_relays"]})
        records = [self._relay_record(g, inv, target, by.get(g, {"eligible": False, "reason": "not requested"}))
                   for g in cands]
        return {
            "topology_snapshot_id": inv.topology_snapshot_id(), "topology_version": inv.version,
            "target_gpu": target, "requested_relays": list(cands), "inventory_source": inv.source,
            "inventory_discovered_at": inv.discovered_at, "relay_eligibility": elig, "relays": records,
            "summary": {
                "relay_count": len(records), "configured_relay_count": sum(1 for r in records if r["configured"]),
                "eligible_relay_count": sum(1 for r in records if r["eligibility"]["eligible"] is True),
                "active_session_count": sum(int(r["quota"]["active_sessions"]) for r in records if r["quota"]),
                "active_reservation_count": sum(len(r["reservations"]) for r in records),
                "active_lease_count": sum(len(r["leases"]) for r in records)}}

    def _relay_record(self, g: int, inv, target: int | None, elig: dict) -> dict[str, Any]:
        S = self._st
        q = self._quotas.get(g)
        links = [asdict(l) for l in inv.fabric_links
                 if (l.src_device_id == g or l.dst_device_id == g)
                 and (target is None or (l.src_device_id == g and l.dst_device_id == target)
                      or (l.bidirectional and l.src_device_id == target and l.dst_device_id == g))]
        sessions = []
        if q is not None:
            for sid in sorted(q.sessions):
                s = S.sessions.get(sid)
                if s is not None:
                    sessions.append({"session_id": s.session_id, "target_gpu": s.target_gpu, "active": s.active,
                                     "active_chunks": s.active_chunks, "max_inflight_chunks": s.max_inflight_chunks,
                                     "job_ids": sorted(j.job_id for j in S.jobs.values() if j.session_id == sid)})
        reservations = []
        for rid, res in sorted(S.reservations.items()):
            if res.relay_gpu == g:
                rec = asdict(res)
                l = S.leases.get(rid)
                rec.update(transfer_id=S.reservation_transfer.get(rid), job_id=None if l is None else l.job_id)
                reservations.append(rec)
        leases = [{"lease_id": l.lease_id, "session_id": l.session_id, "relay_gpu": l.relay_gpu,
                   "job_id": l.job_id, "buffer_ids": l.buffer_ids, "issued_at": l.issued_at,
                   "expires_at": l.expires_at, "transfer_id": S.reservation_transfer.get(lid)}
                  for lid, l in sorted(S.leases.items()) if l.relay_gpu == g and lid in S.reservations]
        return {
            "relay_gpu": g, "configured": q is not None,
            "eligibility": {"target_gpu": target, "eligible": elig["eligible"], "reason": elig["reason"]},
            "inventory": {"gpus": [asdict(x) for x in inv.gpus if x.device_id == g],
                          "pcie_paths": [asdict(p) for p in inv.pcie_paths if p.device_id == g],
                          "fabric_links": links,
                          "path_capabilities": path_capabilities(inv, g, target, links)},
            "quota": None if q is None else {
                "relay_gpu": q.relay_gpu, "max_sessions": q.max_sessions, "active_sessions": len(q.sessions),
                "available_sessions": max(0, q.max_sessions - len(q.sessions)),
                "max_inflight_chunks": q.max_inflight_chunks, "active_chunks": q.active_chunks,
                "available_chunks": max(0, q.max_inflight_chunks - q.active_chunks)},
            "sessions": sessions, "reservations": reservations, "leases": leases}


# ---- module helpers ------------------------------------------------------------------------------------

def norm_relays(relays: Iterable[int] | None) -> list[int]:
    return sorted({int(g) for g in (relays or ())})


def profile_key(target_gpu: int, relay_gpus: Iterable[int]) -> str:
    return f"target={int(target_gpu)};relays={','.join(str(g) for g in norm_relays(relay_gpus))}"


def normalize_profile(profile: dict, target: int) -> dict[str, Any]:
    if not isinstance(profile, dict):
        raise ValueError("profile must be a dict")
    h2d = float(profile.get("direct_h2d_bw_gbps", 0.0) or 0.0)
    if h2d <= 0.0:
        raise ValueError("profile direct_h2d_bw_gbps must be positive")
    relays = []
    for r in profile.get("relays", []) or []:
        if not isinstance(r, dict):
            raise ValueError("profile relays must be dicts")
        relays.append({"relay_device": int(r["relay_device"]),
                       "target_device": int(r.get("target_device", target)),
                       **{k: float(r.get(k, 0.0) or 0.0) for k in
                          ("h2d_bw_gbps", "d2h_bw_gbps", "p2p_bw_gbps", "effective_bw_gbps",
                           "effective_d2h_bw_gbps")},
                       "p2p_enabled": bool(r.get("p2p_enabled", False))})
    out = {"target_device": int(profile.get("target_device", target)), "direct_h2d_bw_gbps": h2d,
           "direct_d2h_bw_gbps": float(profile.get("direct_d2h_bw_gbps", 0.0) or 0.0), "relays": relays}
    for extra in ("concurrent", "uplink_groups", "lane_latency_s", "measured_by"):
        if extra in profile:
            out[extra] = profile[extra]
    return out


def norm_ranges(ranges) -> tuple[dict[str, int], ...] | None:
    if ranges is None:
        return None
    out = []
    for item in ranges:
        if not isinstance(item, dict):
            raise ValueError("transfer ranges must be objects")
        s, d, n = int(item["src_offset"]), int(item["dst_offset"]), int(item["bytes"])
        if s < 0 or d < 0:
            raise ValueError("range offsets must be non-negative")
        if n <= 0:
            raise ValueError("range bytes must be positive")
        out.append({"src_offset": s, "dst_offset": d, "bytes": n})
    return tuple(out)


def intent_chunk_bytes(intent: TransferIntent) -> int:
    """``chunk_bytes`` from policy hints or metadata; default: one chunk."""
    for src in (intent.policy_hints, intent.metadata):
        if isinstance(src, dict) and src.get("chunk_bytes") is not None:
            v = int(src["chunk_bytes"])
            if v <= 0:
                raise ValueError("chunk_bytes must be positive")
            return v
    return max(1, int(intent.total_bytes))


def _plan_chunks(plan, *, kind: str | None, relays: set[int] | None, direction: str):
    if not isinstance(plan, dict):
        raise ValueError("transfer plan is unavailable")
    for a in plan.get("assignments", ()) or ():
        if not isinstance(a, dict):
            raise ValueError("transfer plan assignment must be an object")
        p = a.get("path")
        if not isinstance(p, dict):
            raise ValueError("transfer plan assignment path must be an object")
        if kind is not None and str(p.get("kind", "")).lower() != kind:
            continue
        if str(p.get("direction", "")).lower() != direction:
            continue
        if relays is not None and int(p.get("relay_device", -1)) not in relays:
            continue
        yield a, p


def relay_ranges(plan, relay_gpu, direction: str) -> tuple[dict[str, int], ...]:
    relays = {int(relay_gpu)} if isinstance(relay_gpu, int) else {int(g) for g in relay_gpu}
    if not relays:
        raise ValueError("daemon plan has no authorized relay chunks")
    out = []
    for a, _p in _plan_chunks(plan, kind="relay", relays=relays, direction=str(direction).lower()):
        for s, d, n in assignment_spans(a):
            out.append({"src_offset": s, "dst_offset": d, "bytes": n})
    if not out:
        raise ValueError("daemon plan has no authorized relay chunks")
    return tuple(out)


def relay_devices(plan, direction: str) -> set[int]:
    return {int(p.get("relay_device", -1))
            for a, p in _plan_chunks(plan, kind="relay", relays=None, direction=str(direction).lower())
            if assignment_has_chunks(a)}


def transfer_timing(rec: Mapping[str, Any], completed_at: float | None) -> dict[str, Any]:
    """Daemon-side times of one transfer: when it was queued, started and
    finished, and the derived queueing, execution, lease-wait (time parked in
    delayed admission) and total milliseconds."""
    def ms(a, b):
        return None if a is None or b is None else round(max(0.0, (float(b) - float(a)) * 1e3), 3)

    q, s, d, adm = rec.get("queued_at"), rec.get("started_at"), rec.get("delayed_at"), rec.get("admitted_at")
    return {"queued_at": q, "started_at": s, "completed_at": completed_at, "queue_ms": ms(q, s),
            "execution_ms": ms(s, completed_at), "total_ms": ms(q, completed_at),
            "lease_wait_ms": ms(d, adm) if d is not None else 0.0}


def ticket_ranges(plan, direction: str) -> tuple[dict[str, int], ...]:
    chunks = []
    for a, _p in _plan_chunks(plan, kind=None, relays=None, direction=str(direction).lower()):
        chunks.extend({"src_offset": s, "dst_offset": d, "bytes": n} for s, d, n in assignment_spans(a))
    if not chunks:
        raise ValueError("daemon plan has no authorized chunks")
    return byte_ranges(chunks)


def decision_direction(decision: SchedulingDecision) -> str:
    for a in decision.plan.get("assignments", ()) or ():
        p = a.get("path") if isinstance(a, dict) else None
        if isinstance(p, dict) and str(p.get("direction", "")).lower() in ("h2d", "d2h"):
            return str(p["direction"]).lower()
    raise ValueError("scheduling decision plan has no direction")


def direct_only(decision: SchedulingDecision) -> bool:
    asg = decision.plan.get("assignments", ()) or ()
    return bool(asg) and all(isinstance(a, dict) and isinstance(a.get("path"), dict)
                             and str(a["path"].get("kind", "")).lower() == "direct" for a in asg)


def plan_targets(plan: Mapping[str, Any]) -> tuple[int, ...]:
    """Target devices named by a plan's paths."""
    out: set[int] = set()
    for a in plan.get("assignments", ()) or ():
        p = a.get("path") if isinstance(a, Mapping) else None
        if isinstance(p, Mapping) and p.get("target_device") is not None:
            out.add(int(p["target_device"]))
    return tuple(sorted(out))


def busy_relays(state: Mapping[str, Any], queue_behind: tuple | None = None) -> set[int]:
    """GPUs whose PCIe link is in use: relays of active relay paths and the
    targets of active direct paths.  (GPUs inside the link-hold window are
    only kept out of new plans; admission never waits on them.)
    ``queue_behind=(session_id, target, directions)`` leaves out the paths of
    that session's own transfers to that target in those directions."""
    out: set[int] = set()
    for p in state.get("active_paths", ()) or ():
        if not isinstance(p, Mapping):
            continue
        if queue_behind is not None and p.get("session_id") == queue_behind[0] \
                and p.get("target_device") is not None and int(p["target_device"]) == int(queue_behind[1]) \
                and str(p.get("direction", "")).lower() in queue_behind[2]:
            continue
        kind = str(p.get("kind", "")).lower()
        if kind == "relay" and p.get("relay_device") is not None:
            out.add(int(p["relay_device"]))
        elif kind == "direct" and p.get("target_device") is not None:
            out.add(int(p["target_device"]))
    return out


def job_runtime_state(weights: Mapping[str, float], records) -> dict[str, dict[str, Any]]:
    def blank(j, w):
        return {"job_id": j, "weight": float(w), "queued_transfer_count": 0, "running_transfer_count": 0,
                "active_transfer_count": 0, "active_bytes_total": 0, "active_bytes_remaining": 0}

    jobs = {j: blank(j, w) for j, w in weights.items()}
    sub, run = TransferStatusState.SUBMITTED.value, TransferStatusState.RUNNING.value
    for r in records:
        if not isinstance(r, Mapping) or r.get("job_id") is None:
            continue
        j = str(r["job_id"])
        rec = jobs.setdefault(j, blank(j, 1.0))
        state = str(r.get("state", ""))
        if state == sub:
            rec["queued_transfer_count"] += 1
        elif state == run:
            rec["running_transfer_count"] += 1
        if state in (sub, run):
            tot, done = int(r.get("bytes_total", 0) or 0), int(r.get("bytes_completed", 0) or 0)
            rec["active_transfer_count"] += 1
            rec["active_bytes_total"] += tot
            rec["active_bytes_remaining"] += max(0, tot - done)
    return dict(sorted(jobs.items()))


def state_without_transfer(state: dict[str, Any], tid: str) -> dict[str, Any]:
    out = dict(state)
    for k in ("transfers", "queued_transfers", "running_transfers", "active_transfers", "active_paths"):
        v = out.get(k)
        if isinstance(v, (list, tuple)):
            out[k] = [dict(i) for i in v if isinstance(i, Mapping) and str(i.get("transfer_id")) != tid]
    if isinstance(out.get("transfer_order"), (list, tuple)):
        out["transfer_order"] = tuple(str(i) for i in out["transfer_order"] if str(i) != tid)
    if isinstance(out.get("summary"), Mapping):
        s = dict(out["summary"])
        s["queued_transfer_count"] = len(out.get("queued_transfers", ()))
        s["running_transfer_count"] = len(out.get("running_transfers", ()))
        s["active_transfer_count"] = len(out.get("active_transfers", ()))
        out["summary"] = s
    jobs = out.get("job_runtime_state")
    if isinstance(jobs, Mapping):
        weights = {str(j): float(r.get("weight", 1.0) if isinstance(r, Mapping) else 1.0) for j, r in jobs.items()}
        out["job_runtime_state"] = job_runtime_state(weights, out.get("transfers", ()))
        if isinstance(out.get("summary"), Mapping):
            out["summary"] = {**out["summary"], "job_runtime_state": out["job_runtime_state"]}
    return out


def path_capabilities(inv, relay: int, target: int | None, links: list[dict]) -> dict[str, Any]:
    path = inv.pcie_path(relay)
    enabled = [l for l in links if bool(l.get("enabled", False))]
    return {
        "relay_gpu": int(relay), "target_gpu": target, "has_pcie_path": path is not None,
        "pcie_root_complex": None if path is None else path.root_complex,
        "pcie_numa_node": None if path is None else path.numa_node,
        "pcie_link_generation": None if path is None else path.link_generation,
        "pcie_link_width": None if path is None else path.link_width,
        "pcie_negotiated_speed_gtps": None if path is None else path.negotiated_speed_gtps,
        "pcie_bandwidth_gbps": 0.0 if path is None else path.bandwidth_gbps,
        "pcie_bandwidth_source": None if path is None else path.bandwidth_source,
        "pcie_switch_hierarchy": [] if path is None else list(path.switch_hierarchy),
        "fabric_link_count": len(links), "enabled_fabric_link_count": len(enabled),
        "fabric_kinds": sorted({str(l.get("fabric")) for l in enabled}),
        "fabric_capabilities": sorted({str(l.get("capability")) for l in enabled if l.get("capability") is not None}),
        "fabric_bandwidth_gbps": sum(float(l.get("bandwidth_gbps", 0.0) or 0.0) for l in enabled),
        "p2p_enabled": bool(enabled)}


def bind_job_to_peer(user_id, process_id, container_id, peer: PeerIdentity | None):
    """Authenticated peers own the jobs they register; stated ids must agree."""
    if peer is None or not peer.authenticated:
        return user_id, process_id, container_id
    if user_id is not None and str(user_id) != str(peer.user_id):
        raise ValueError("job user_id does not match authenticated peer")
    if process_id is not None and peer.process_id is not None and int(process_id) != int(peer.process_id):
        raise ValueError("job process_id does not match authenticated peer")
    if container_id is not None and peer.container_id is not None and str(container_id) != str(peer.container_id):
        raise ValueError("job container_id does not match authenticated peer")
    return (str(peer.user_id), peer.process_id if process_id is None else int(process_id),
            peer.container_id if container_id is None else str(container_id))


def same_owner(expected: PeerIdentity | None, actual: PeerIdentity | None, owner: str) -> None:
    if expected is None or actual is None or not expected.authenticated or not actual.authenticated:
        return
    if str(expected.user_id) != str(actual.user_id):
        raise ValueError(f"{owner} owner does not match authenticated peer")


def same_connection(expected: PeerIdentity | None, actual: PeerIdentity | None) -> bool:
    if expected is None or actual is None:
        return False
    if expected.authenticated and actual.authenticated:
        return (str(expected.user_id) == str(actual.user_id) and expected.process_id == actual.process_id
                and expected.group_id == actual.group_id)
    return (expected.authenticated == actual.authenticated and expected.source == actual.source
            and expected.unsupported_reason == actual.unsupported_reason)


def _as_int(v) -> int | None:
    try:
        return int(v)
    except (TypeError, ValueError):
        return None


def socket_path_for_user(base_dir: str = "/tmp") -> str:
    return f"{base_dir.rstrip('/')}/turbobusd.sock"


PoolDaemon = TurboBusDaemon

__all__ = ["PoolDaemon", "TurboBusDaemon", "profile_key", "reserve_socket", "socket_path_for_user"]
