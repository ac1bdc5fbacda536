"""One worker-service request line in, one response line out.

The endpoint is the seam between a transport (the AF_UNIX socket server,
or a test harness) and ``WorkerTransferService``: it owns no state of its own
beyond the service, so transports stay thin.  Constructor keywords match
turbobus/worker/endpoint.py so callers of either project build it the same
way (``daemon_client=`` or ``service=``).
"""

from __future__ import annotations

from .codec import handle_worker_service_message
from .helper import WorkerTransferService


def _service_for(daemon_client, service) -> WorkerTransferService:
    # accept the service in the first position too (older call sites)
    if service is None and isinstance(daemon_client, WorkerTransferService):
        return daemon_client
    if service is not None:
        if not isinstance(service, WorkerTransferService):
            raise TypeError(f"service must be a WorkerTransferService, not {type(service).__name__}")
        return service
    if daemon_client is None:
        raise ValueError("a worker endpoint needs a WorkerTransferService or a daemon client to build one")
    return WorkerTransferService(daemon_client)


class WorkerServiceEndpoint:
    def __init__(self, daemon_client=None, service: WorkerTransferService | None = None) -> None:
        self.service = _service_for(daemon_client, service)

    def handle_message(self, message: str | bytes) -> str:
        """Decode a request envelope, run it on the service, encode the reply."""
        return handle_worker_service_message(self.service, message)


__all__ = ["WorkerServiceEndpoint"]
