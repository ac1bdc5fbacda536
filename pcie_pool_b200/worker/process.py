"""Worker helper process: ``python -m pcie_pool_b200.worker
--daemon-socket-path D --socket-path W [--max-requests N]``
(turbobus/worker/process.py:41-67)."""

from __future__ import annotations

import argparse
import signal
import threading

from .endpoint import WorkerServiceEndpoint
from .helper import WorkerTransferClient, WorkerTransferService
from .transport import WorkerServiceUnixSocketTransport


def build_worker_helper_transport(daemon_socket_path: str, socket_path: str, *, daemon_client=None,
                                  executor=None, resource_binder=None,
                                  staging_pool=None) -> WorkerServiceUnixSocketTransport:
    if daemon_client is None:
        from ..daemon.client import TurboBusDaemonClient

        daemon_client = TurboBusDaemonClient(daemon_socket_path)
    kw = {}
    if executor is not None:
        kw["executor"] = executor
        kw["resource_binder"] = resource_binder
    if staging_pool is not None:
        kw["staging_pool"] = staging_pool
    service = WorkerTransferService(transfer_client=WorkerTransferClient(daemon_client, **kw))
    return WorkerServiceUnixSocketTransport(WorkerServiceEndpoint(service=service), socket_path)


def run_worker_helper_process(daemon_socket_path: str, socket_path: str, max_requests: int | None = None,
                              stop_event: threading.Event | None = None, **kw) -> None:
    build_worker_helper_transport(daemon_socket_path, socket_path, **kw).serve_forever(
        stop_event=stop_event, max_requests=max_requests)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m pcie_pool_b200.worker")
    ap.add_argument("--daemon-socket-path", required=True)
    ap.add_argument("--socket-path", required=True)
    ap.add_argument("--max-requests", type=int, default=None)
    a = ap.parse_args(argv)
    stop = threading.Event()
    for sig in (signal.SIGTERM, signal.SIGINT):
        signal.signal(sig, lambda *_: stop.set())
    run_worker_helper_process(a.daemon_socket_path, a.socket_path, max_requests=a.max_requests, stop_event=stop)
    return 0


__all__ = ["build_worker_helper_transport", "main", "run_worker_helper_process"]
