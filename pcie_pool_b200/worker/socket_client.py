"""Client of a worker helper socket (turbobus/worker/socket_client.py)."""

from __future__ import annotations

import socket
from dataclasses import dataclass

from .codec import decode_worker_response_envelope, encode_worker_request_envelope
from .helper import WorkerDataPlaneCompletionEnvelope, WorkerServiceRequestEnvelope, WorkerServiceResponseEnvelope
from .transport import read_worker_socket_message


@dataclass(frozen=True)
class WorkerServiceSocketClient:
    socket_path: str
    timeout_seconds: float | None = None

    def __post_init__(self) -> None:
        if not str(self.socket_path).strip():
            raise ValueError("socket_path must be non-empty")
        object.__setattr__(self, "socket_path", str(self.socket_path))

    def send_message(self, message: str | bytes) -> str:
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as c:
            if self.timeout_seconds is not None:
                c.settimeout(float(self.timeout_seconds))
            c.connect(self.socket_path)
            c.sendall((message.encode("utf-8") if isinstance(message, str) else message) + b"\n")
            return read_worker_socket_message(c).decode("utf-8")

    def submit(self, envelope: WorkerServiceRequestEnvelope) -> WorkerServiceResponseEnvelope:
        return decode_worker_response_envelope(self.send_message(encode_worker_request_envelope(envelope)))

    def submit_payload(self, payload: dict, cleanup_target_kind: str = "reservation") -> WorkerServiceResponseEnvelope:
        return self.submit(WorkerServiceRequestEnvelope(payload=payload, cleanup_target_kind=cleanup_target_kind))

    def submit_envelope(self, envelope: WorkerServiceRequestEnvelope) -> WorkerDataPlaneCompletionEnvelope:
        """Submit and return the completion envelope (turbobus/worker/socket_client.py:24-44):
        the worker's completion record with ``ok`` folded from the response and
        the record, or just ok / final state / error when the worker sent none."""
        if not isinstance(envelope, WorkerServiceRequestEnvelope):
            raise TypeError("envelope must be a WorkerServiceRequestEnvelope")
        resp = self.submit(envelope)
        if resp.completion is None:
            return WorkerDataPlaneCompletionEnvelope(ok=resp.ok, final_state=resp.final_state, error=resp.error)
        c = dict(resp.completion)
        c["ok"] = bool(resp.ok and c.get("ok", True))
        if c.get("final_state") is None and resp.final_state is not None:
            c["final_state"] = resp.final_state
        if c.get("error") is None and resp.error is not None:
            c["error"] = resp.error
        known = set(WorkerDataPlaneCompletionEnvelope.__dataclass_fields__)
        return WorkerDataPlaneCompletionEnvelope(**{k: v for k, v in c.items() if k in known})


__all__ = ["WorkerServiceSocketClient"]
