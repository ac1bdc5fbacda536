"""AF_UNIX transport of the daemon: newline-delimited JSON requests
``{request_type, session_id, payload}`` answered by ``{ok, payload, error}``
(the reference's wire format, turbobus/daemon/client.py:21-42).

The server runs one thread per connection so a slow client (or a long
WAIT_TRANSFER_RECEIPT) never blocks the others; peer identity comes from
SO_PEERCRED; sessions registered as connection-scoped are closed when their
connection ends.

File descriptors (CUDA VMM buffer exports) travel beside a request as
``SCM_RIGHTS`` ancillary data; the request says how many with a top-level
``"attached_fds"`` count, and only the server -- never the JSON -- hands
descriptors to the daemon.
"""

from __future__ import annotations

import json
import os
import socket
import struct
import threading
import uuid
from dataclasses import asdict

from ..schema import PeerIdentity


def peer_identity_from_socket(conn: socket.socket) -> PeerIdentity:
    if hasattr(socket, "SO_PEERCRED"):
        try:
            raw = conn.getsockopt(socket.SOL_SOCKET, socket.SO_PEERCRED, struct.calcsize("3i"))
            pid, uid, gid = struct.unpack("3i", raw)
            return PeerIdentity(authenticated=True, source="unix_socket_peercred", user_id=str(uid),
                                process_id=pid, group_id=gid)
        except OSError as exc:
            return PeerIdentity(authenticated=False, source="unix_socket_peercred",
                                unsupported_reason=str(exc))
    return PeerIdentity(authenticated=False, source="unix_socket",
                        unsupported_reason="SO_PEERCRED is unavailable on this platform")


MAX_FDS_PER_MESSAGE = 8


def _attached_fd_count(line: bytes) -> int:
    if b'"attached_fds"' not in line:
        return 0
    try:
        n = json.loads(line).get("attached_fds", 0)
    except (ValueError, AttributeError):
        return 0
    return max(0, min(int(n), MAX_FDS_PER_MESSAGE)) if isinstance(n, int) else 0


def _serve_connection(daemon, conn: socket.socket) -> None:
    peer = peer_identity_from_socket(conn)
    conn_id = str(uuid.uuid4())
    buf = b""
    fds: list[int] = []  # received descriptors not yet claimed by a request
    try:
        with conn:
            while True:
                try:
                    data, got, _flags, _addr = socket.recv_fds(conn, 1 << 16, MAX_FDS_PER_MESSAGE)
                except OSError:
                    break
                fds.extend(got)
                if not data:
                    break
                buf += data
                while b"\n" in buf:
                    line, _, buf = buf.partition(b"\n")
                    if not line.strip():
                        continue
                    n = _attached_fd_count(line)
                    mine, fds = fds[:n], fds[n:]
                    try:
                        resp = daemon.handle_wire_message(line, peer_identity=peer, connection_id=conn_id,
                                                          fds=mine)
                    finally:
                        for fd in mine:  # the daemon keeps its own duplicates
                            os.close(fd)
                    try:
                        conn.sendall((json.dumps(asdict(resp), default=_json_default) + "\n").encode())
                    except OSError:
                        return
    finally:
        for fd in fds:
            os.close(fd)
        daemon.close_connection(peer, conn_id, reason="socket_disconnect")


def _json_default(o):
    if isinstance(o, (set, frozenset)):
        return sorted(o)
    if hasattr(o, "value"):
        return o.value
    raise TypeError(f"not JSON serialisable: {type(o).__name__}")


def reserve_socket(path: str, backlog: int = 128) -> socket.socket:
    """Bind and listen on the AF_UNIX socket ``path`` (turbobus/daemon/server.py:3680).

    A leftover socket file nobody listens on is removed first; a path that a
    live server still answers on is refused, so a second daemon cannot take
    over the first one's socket.
    """
    if os.path.exists(path):
        probe = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        probe.settimeout(0.5)
        try:
            probe.connect(path)
        except OSError:
            os.unlink(path)  # stale: no listener behind it
        else:
            raise RuntimeError(f"socket {path} is served by a running process")
        finally:
            probe.close()
    sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    try:
        sock.bind(path)
        sock.listen(int(backlog))
    except BaseException:
        sock.close()
        raise
    return sock


def serve_unix(daemon, socket_path: str, *, stop_event: threading.Event | None = None,
               ready_event: threading.Event | None = None, poll_seconds: float = 0.1,
               sock: socket.socket | None = None) -> None:
    """Accept connections until ``stop_event`` is set (forever if None).
    ``sock``: a socket already bound to ``socket_path`` by :func:`reserve_socket`."""
    server = sock if sock is not None else reserve_socket(socket_path)
    server.settimeout(poll_seconds)
    if ready_event is not None:
        ready_event.set()
    threads: list[threading.Thread] = []
    try:
        while stop_event is None or not stop_event.is_set():
            try:
                conn, _ = server.accept()
            except socket.timeout:
                continue
            except OSError:
                break
            conn.settimeout(None)
            t = threading.Thread(target=_serve_connection, args=(daemon, conn), daemon=True)
            t.start()
            threads.append(t)
            threads = [x for x in threads if x.is_alive()]
    finally:
        server.close()
        if os.path.exists(socket_path):
            os.unlink(socket_path)


def _send(sock: socket.socket, message: dict, fds=None) -> None:
    if fds:
        message = {**message, "attached_fds": len(fds)}
    data = (json.dumps(message, default=_json_default) + "\n").encode()
    if fds:
        sent = socket.send_fds(sock, [data], list(fds))
        if sent < len(data):
            sock.sendall(data[sent:])
    else:
        sock.sendall(data)


def send_request(socket_path: str, message: dict, timeout: float | None = None, fds=None) -> dict:
    """One request over a fresh connection; returns the decoded response.
    ``fds`` ride along as SCM_RIGHTS ancillary data."""
    c = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    if timeout is not None:
        c.settimeout(timeout)
    try:
        c.connect(socket_path)
        _send(c, message, fds)
        data = b""
        while b"\n" not in data:
            chunk = c.recv(1 << 16)
            if not chunk:
                break
            data += chunk
    finally:
        c.close()
    if not data:
        raise ConnectionError("daemon closed the connection without a response")
    return json.loads(data.split(b"\n", 1)[0].decode())


class PersistentConnection:
    """Reuses one socket for many requests (lower per-RPC latency); required
    for connection-scoped sessions, which live as long as the connection."""

    def __init__(self, socket_path: str, timeout: float | None = None) -> None:
        self._sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        if timeout is not None:
            self._sock.settimeout(timeout)
        self._sock.connect(socket_path)
        self._buf = b""
        self._lock = threading.Lock()

    def request(self, message: dict, fds=None) -> dict:
        with self._lock:
            _send(self._sock, message, fds)
            while b"\n" not in self._buf:
                chunk = self._sock.recv(1 << 16)
                if not chunk:
                    raise ConnectionError("daemon closed the connection")
                self._buf += chunk
            line, _, self._buf = self._buf.partition(b"\n")
            return json.loads(line.decode())

    def close(self) -> None:
        try:
            self._sock.close()
        except OSError:
            pass
