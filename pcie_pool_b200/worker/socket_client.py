"""Client of a worker helper socket (turbobus/worker/socket_client.py)."""

from __future__ import annotations

import socket
from dataclasses import dataclass

from .codec import decode_worker_response_envelope, encode_worker_request_envelope
from .helper import WorkerServiceRequestEnvelope, WorkerServiceResponseEnvelope
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


__all__ = ["WorkerServiceSocketClient"]
