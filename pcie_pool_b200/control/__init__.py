"""Control-plane entry points (daemon and its client)."""

from ..daemon.client import TurboBusDaemonClient
from ..daemon.server import TurboBusDaemon

__all__ = ["TurboBusDaemon", "TurboBusDaemonClient"]
