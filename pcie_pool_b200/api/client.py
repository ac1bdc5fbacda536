"""Public daemon-first transfer client: submit a ``TransferIntent``, wait for
its ``TransferReceipt`` (turbobus/api/client.py:23-67)."""

from __future__ import annotations

from dataclasses import fields
from typing import Protocol, runtime_checkable

from ..schema import DaemonResponse, TransferIntent, TransferReceipt


@runtime_checkable
class DaemonIntentClient(Protocol):
    def submit_transfer_intent(self, intent: TransferIntent) -> DaemonResponse:
        ...

    def wait_transfer_receipt(self, intent_id: str, timeout_seconds: float | None = None) -> DaemonResponse:
        ...


class TurboBusClient:
    """``TurboBusClient(daemon=...)`` with any object speaking the two calls
    above (a socket client, an in-process daemon client or a fake), or
    ``TurboBusClient(socket_path=...)``."""

    def __init__(self, daemon: DaemonIntentClient | None = None, *, socket_path: str | None = None) -> None:
        if daemon is None and socket_path is None:
            raise ValueError("daemon or socket_path is required")
        if daemon is not None and socket_path is not None:
            raise ValueError("provide daemon or socket_path, not both")
        if daemon is None:
            from ..daemon.client import TurboBusDaemonClient

            daemon = TurboBusDaemonClient(socket_path)
        self._daemon = daemon

    @property
    def daemon(self) -> DaemonIntentClient:
        return self._daemon

    def submit(self, intent: TransferIntent) -> TransferReceipt:
        return self.submit_transfer_intent(intent)

    def submit_transfer(self, intent: TransferIntent) -> TransferReceipt:
        return self.submit_transfer_intent(intent)

    def submit_transfer_intent(self, intent: TransferIntent) -> TransferReceipt:
        if not isinstance(intent, TransferIntent):
            raise TypeError("intent must be a TransferIntent")
        return receipt_from_response(self._daemon.submit_transfer_intent(intent), intent.intent_id)

    def wait(self, intent: TransferIntent | str, timeout_seconds: float | None = None) -> TransferReceipt:
        iid = intent.intent_id if isinstance(intent, TransferIntent) else str(intent)
        return receipt_from_response(self._daemon.wait_transfer_receipt(iid, timeout_seconds=timeout_seconds), iid)

    def wait_transfer_receipt(self, intent_id: str, timeout_seconds: float | None = None) -> TransferReceipt:
        return self.wait(intent_id, timeout_seconds=timeout_seconds)

    def transfer(self, intent: TransferIntent, timeout_seconds: float = 600.0) -> TransferReceipt:
        """Submit and wait for a terminal receipt in one call."""
        self.submit_transfer_intent(intent)
        return self.wait(intent.intent_id, timeout_seconds=timeout_seconds)


def receipt_from_response(response: DaemonResponse, expected_intent_id: str) -> TransferReceipt:
    if not isinstance(response, DaemonResponse):
        raise TypeError("daemon response must be a DaemonResponse")
    if not response.ok:
        raise RuntimeError(response.error or "daemon request failed")
    payload = response.payload.get("receipt")
    if not isinstance(payload, dict):
        raise ValueError("daemon response missing receipt")
    names = {f.name for f in fields(TransferReceipt)}
    unknown = sorted(k for k in payload if k not in names)
    if unknown:
        raise ValueError("daemon receipt contains unknown fields: " + ", ".join(unknown))
    receipt = TransferReceipt(**payload)
    if receipt.intent_id != str(expected_intent_id):
        raise ValueError("daemon receipt intent_id does not match request")
    return receipt


__all__ = ["DaemonIntentClient", "TurboBusClient", "receipt_from_response"]
