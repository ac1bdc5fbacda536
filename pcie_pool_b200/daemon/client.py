"""Typed RPC stubs for the daemon (one method per request type).

Same method names and payloads as the reference client
(turbobus/daemon/client.py:17-397).  By default every call opens a fresh
connection; ``persistent=True`` keeps one connection open (lower latency,
and needed for connection-scoped sessions).
"""

from __future__ import annotations

from dataclasses import asdict

from ..schema import contract_asdict

from ..schema import (DaemonRequest, DaemonResponse, RequestType, TransferIntent,
                      WorkerTransferAuthorizationRequest)
from ..transfer import TransferRequest
from .wire import PersistentConnection, send_request


class TurboBusDaemonClient:
    def __init__(self, socket_path: str, *, persistent: bool = False, timeout: float | None = None) -> None:
        self.socket_path = str(socket_path)
        self._timeout = timeout
        self._conn = PersistentConnection(self.socket_path, timeout) if persistent else None

    def close(self) -> None:
        if self._conn is not None:
            self._conn.close()
            self._conn = None

    def send(self, request: DaemonRequest, fds=None) -> DaemonResponse:
        msg = asdict(request)
        msg["request_type"] = RequestType(request.request_type).value
        msg.pop("peer_identity", None)
        data = self._conn.request(msg, fds=fds) if self._conn is not None else send_request(
            self.socket_path, msg, self._timeout, fds=fds)
        return DaemonResponse(ok=bool(data["ok"]), payload=data.get("payload", {}) or {},
                              error=data.get("error"))

    def _call(self, rtype: RequestType, payload: dict | None = None,
              session_id: str | None = None, fds=None) -> DaemonResponse:
        req = DaemonRequest(request_type=rtype, session_id=session_id, payload=payload or {})
        return self.send(req, fds=fds) if fds else self.send(req)

    def register_session(self, target_gpu: int, relay_gpus: list[int], max_inflight_chunks: int = 8,
                         connection_scoped: bool = False) -> DaemonResponse:
        p = {"target_gpu": int(target_gpu), "relay_gpus": [int(g) for g in relay_gpus],
             "max_inflight_chunks": int(max_inflight_chunks)}
        if connection_scoped:
            p["connection_scoped"] = True
        return self._call(RequestType.REGISTER_SESSION, p)

    def close_session(self, session_id: str) -> DaemonResponse:
        return self._call(RequestType.CLOSE_SESSION, session_id=str(session_id))

    def register_job(self, job_id: str, user_id: str | None = None, session_id: str | None = None,
                     container_id: str | None = None, process_id: int | None = None,
                     weight: float = 1.0) -> DaemonResponse:
        p: dict[str, object] = {"job_id": str(job_id)}
        for k, v, f in (("user_id", user_id, str), ("session_id", session_id, str),
                        ("container_id", container_id, str), ("process_id", process_id, int)):
            if v is not None:
                p[k] = f(v)
        p["weight"] = float(weight)
        return self._call(RequestType.REGISTER_JOB, p)

    def register_buffer(self, buffer_id: str, job_id: str, kind: str, size_bytes: int,
                        device_index: int | None = None, address: int | None = None, pinned: bool = False,
                        handle_type: str = "registered_buffer", metadata: dict | None = None,
                        fds: list[int] | None = None) -> DaemonResponse:
        """``fds``: descriptors the buffer needs in the daemon (a CUDA VMM
        export), passed beside the request."""
        p: dict[str, object] = {"buffer_id": str(buffer_id), "job_id": str(job_id), "kind": str(kind),
                                "size_bytes": int(size_bytes), "pinned": bool(pinned),
                                "handle_type": str(handle_type)}
        if device_index is not None:
            p["device_index"] = int(device_index)
        if address is not None:
            p["address"] = int(address)
        if metadata is not None:
            p["metadata"] = dict(metadata)
        return self._call(RequestType.REGISTER_BUFFER, p, fds=fds)

    def reserve_transfer(self, session_id: str, relay_gpu: int, chunks: int, bytes_: int = 0,
                         direction: str = "unknown") -> DaemonResponse:
        return self._call(RequestType.RESERVE_TRANSFER, {"relay_gpu": int(relay_gpu), "chunks": int(chunks),
                                                          "bytes": int(bytes_), "direction": str(direction)},
                          session_id=str(session_id))

    def plan_transfer(self, session_id: str, total_bytes: int, chunk_bytes: int, mode: str = "pool",
                      direction: str = "h2d", job_id: str | None = None) -> DaemonResponse:
        req = TransferRequest(total_bytes=total_bytes, chunk_bytes=chunk_bytes, mode=mode,
                              direction=direction, job_id=job_id)
        return self.plan_transfer_request(session_id, req)

    def plan_transfer_request(self, session_id: str, request: TransferRequest,
                              mode: str | None = None) -> DaemonResponse:
        return self._call(RequestType.PLAN_TRANSFER, request.daemon_payload(mode=mode), session_id=str(session_id))

    def submit_transfer_intent(self, intent: TransferIntent) -> DaemonResponse:
        if not isinstance(intent, TransferIntent):
            raise TypeError("intent must be a TransferIntent")
        # shallow: an intent is immutable once built and may carry a large
        # landing spec (block ids), which a deep copy would walk element by element
        return self._call(RequestType.SUBMIT_TRANSFER_INTENT, {"intent": contract_asdict(intent)},
                          session_id=intent.session_id)

    def wait_transfer_receipt(self, intent_id: str, timeout_seconds: float | None = None) -> DaemonResponse:
        p: dict[str, object] = {"intent_id": str(intent_id)}
        if timeout_seconds is not None:
            p["timeout_seconds"] = float(timeout_seconds)
        return self._call(RequestType.WAIT_TRANSFER_RECEIPT, p)

    def reschedule_transfer(self, transfer_id: str, now: float | None = None) -> DaemonResponse:
        p: dict[str, object] = {"transfer_id": str(transfer_id)}
        if now is not None:
            p["now"] = float(now)
        return self._call(RequestType.RESCHEDULE_TRANSFER, p)

    def release_transfer(self, reservation_id: str) -> DaemonResponse:
        return self._call(RequestType.RELEASE_TRANSFER, {"reservation_id": str(reservation_id)})

    def cleanup(self, target_kind: str, target_id: str, reason: str = "manual",
                force: bool = False) -> DaemonResponse:
        return self._call(RequestType.CLEANUP, {"target_kind": str(target_kind), "target_id": str(target_id),
                                                "reason": str(reason), "force": bool(force)})

    def transfer_status(self, transfer_id: str, state: str | None = None, bytes_completed: int | None = None,
                        error: str | None = None) -> DaemonResponse:
        p: dict[str, object] = {"transfer_id": str(transfer_id)}
        if state is not None:
            p["state"] = str(state)
        if bytes_completed is not None:
            p["bytes_completed"] = int(bytes_completed)
        if error is not None:
            p["error"] = str(error)
        return self._call(RequestType.TRANSFER_STATUS, p)

    def validate_lease(self, lease_id: str, token: str, session_id: str | None = None,
                       relay_gpu: int | None = None, job_id: str | None = None,
                       buffer_ids: list[str] | None = None) -> DaemonResponse:
        p: dict[str, object] = {"lease_id": str(lease_id), "token": str(token)}
        if session_id is not None:
            p["session_id"] = str(session_id)
        if relay_gpu is not None:
            p["relay_gpu"] = int(relay_gpu)
        if job_id is not None:
            p["job_id"] = str(job_id)
        if buffer_ids is not None:
            p["buffer_ids"] = [str(b) for b in buffer_ids]
        return self._call(RequestType.VALIDATE_LEASE, p)

    def authorize_worker_transfer(self, request: WorkerTransferAuthorizationRequest) -> DaemonResponse:
        if not isinstance(request, WorkerTransferAuthorizationRequest):
            raise TypeError("request must be a WorkerTransferAuthorizationRequest")
        return self._call(RequestType.AUTHORIZE_WORKER_TRANSFER, asdict(request))

    def describe(self) -> DaemonResponse:
        return self._call(RequestType.PROFILE)

    def get_inventory(self) -> DaemonResponse:
        return self._call(RequestType.GET_INVENTORY)

    def invalidate_topology(self) -> DaemonResponse:
        return self._call(RequestType.INVALIDATE_TOPOLOGY)

    def discover_relays(self, target_gpu: int | None = None, relay_gpus: list[int] | None = None) -> DaemonResponse:
        p: dict[str, object] = {}
        if target_gpu is not None:
            p["target_gpu"] = int(target_gpu)
        if relay_gpus is not None:
            p["relay_gpus"] = [int(g) for g in relay_gpus]
        return self._call(RequestType.DISCOVER_RELAYS, p)

    def reap_expired_leases(self, now: float | None = None) -> DaemonResponse:
        return self._call(RequestType.REAP_EXPIRED_LEASES, {} if now is None else {"now": float(now)})

    def get_profile(self, target_gpu: int, relay_gpus: list[int]) -> DaemonResponse:
        return self._call(RequestType.GET_PROFILE, {"target_gpu": int(target_gpu),
                                                    "relay_gpus": [int(g) for g in relay_gpus]})

    def put_profile(self, target_gpu: int, relay_gpus: list[int], profile: dict, profile_bytes: int = 0,
                    updated_at: float | None = None) -> DaemonResponse:
        p: dict[str, object] = {"target_gpu": int(target_gpu), "relay_gpus": [int(g) for g in relay_gpus],
                                "profile": dict(profile), "profile_bytes": int(profile_bytes)}
        if updated_at is not None:
            p["updated_at"] = float(updated_at)
        return self._call(RequestType.PUT_PROFILE, p)

    def invalidate_profile(self, target_gpu: int, relay_gpus: list[int]) -> DaemonResponse:
        return self._call(RequestType.INVALIDATE_PROFILE, {"target_gpu": int(target_gpu),
                                                           "relay_gpus": [int(g) for g in relay_gpus]})


class InProcessDaemonClient(TurboBusDaemonClient):
    """Same stubs, but calls a daemon object in this process (no socket)."""

    def __init__(self, daemon) -> None:  # noqa: D107 - documented on the class
        self.socket_path = "<in-process>"
        self._daemon = daemon
        self._conn = None
        self._timeout = None

    def send(self, request: DaemonRequest, fds=None) -> DaemonResponse:
        # same process: the descriptors are valid here as they are
        return self._daemon.handle_request(request, fds=list(fds) if fds else None)


__all__ = ["InProcessDaemonClient", "TurboBusDaemonClient"]
