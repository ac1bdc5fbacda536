"""Message-level endpoint: decodes a request line, runs the service, encodes
the response (turbobus/worker/endpoint.py)."""

from __future__ import annotations

from dataclasses import dataclass

from .codec import handle_worker_service_message
from .helper import WorkerTransferService


@dataclass
class WorkerServiceEndpoint:
    service: WorkerTransferService

    def __post_init__(self) -> None:
        if not isinstance(self.service, WorkerTransferService):
            raise TypeError("service must be a WorkerTransferService")

    def handle_message(self, message: str | bytes) -> str:
        return handle_worker_service_message(self.service, message)


__all__ = ["WorkerServiceEndpoint"]
