"""AF_UNIX transport of the worker helper: one newline-terminated request
per connection, 100 ms accept poll, optional ``max_requests`` and stop event
(turbobus/worker/transport.py:28-66).  Connections are served on threads, so
a slow transfer does not hold the accept loop; the executor serialises work
per engine."""

from __future__ import annotations

import os
import socket
import threading
from dataclasses import dataclass, field
from threading import Event
from typing import Any

from .endpoint import WorkerServiceEndpoint

MAX_MESSAGE_BYTES = 64 << 20


def read_worker_socket_message(conn: Any) -> bytes:
    buf = bytearray()
    while b"\n" not in buf:
        part = conn.recv(1 << 16)
        if not part:
            break
        buf += part
        if len(buf) > MAX_MESSAGE_BYTES:
            raise ValueError("worker message too large")
    return bytes(buf).partition(b"\n")[0]


def _as_bytes(message: str | bytes) -> bytes:
    if isinstance(message, bytes):
        return message
    if isinstance(message, str):
        return message.encode("utf-8")
    raise TypeError("message must be str or bytes")


@dataclass
class WorkerServiceUnixSocketTransport:
    endpoint: WorkerServiceEndpoint
    socket_path: str
    threaded: bool = True
    _threads: list = field(default_factory=list, repr=False)

    def __post_init__(self) -> None:
        if not isinstance(self.endpoint, WorkerServiceEndpoint):
            raise TypeError("endpoint must be a WorkerServiceEndpoint")
        self.socket_path = str(self.socket_path)
        if not self.socket_path.strip():
            raise ValueError("socket_path must be non-empty")

    def handle_message(self, message: str | bytes) -> str:
        """Client side: send one message to the socket and return the reply."""
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as c:
            c.connect(self.socket_path)
            c.sendall(_as_bytes(message) + b"\n")
            return read_worker_socket_message(c).decode("utf-8")

    def _serve_one(self, conn) -> None:
        with conn:
            try:
                data = read_worker_socket_message(conn)
            except (OSError, ValueError):
                return
            if data:
                conn.sendall((self.endpoint.handle_message(data) + "\n").encode("utf-8"))

    def serve_forever(self, stop_event: Event | None = None, max_requests: int | None = None,
                      ready_event: Event | None = None) -> None:
        if max_requests is not None:
            max_requests = int(max_requests)
            if max_requests <= 0:
                raise ValueError("max_requests must be positive")
        if os.path.exists(self.socket_path):
            os.unlink(self.socket_path)
        srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        srv.bind(self.socket_path)
        srv.listen(64)
        srv.settimeout(0.1)
        if ready_event is not None:
            ready_event.set()
        served = 0
        try:
            while not (stop_event is not None and stop_event.is_set()):
                if max_requests is not None and served >= max_requests:
                    break
                try:
                    conn, _ = srv.accept()
                except socket.timeout:
                    continue
                served += 1
                if self.threaded:
                    t = threading.Thread(target=self._serve_one, args=(conn,), daemon=True)
                    t.start()
                    self._threads.append(t)
                else:
                    self._serve_one(conn)
            for t in self._threads:
                t.join()
        finally:
            srv.close()
            if os.path.exists(self.socket_path):
                os.unlink(self.socket_path)


__all__ = ["WorkerServiceUnixSocketTransport", "read_worker_socket_message"]
