"""Public client API."""

from .client import DaemonIntentClient, TurboBusClient

__all__ = ["DaemonIntentClient", "TurboBusClient"]
