"""Node daemon: control plane, wire protocol and intent execution."""

from .client import InProcessDaemonClient, TurboBusDaemonClient
from .executor import EngineDataPlane, ExecutionResult, IntentExecutor
from .server import PoolDaemon, TurboBusDaemon
from .startup import DaemonStartupConfig, DaemonStartupError, create_production_daemon

__all__ = ["DaemonStartupConfig", "DaemonStartupError", "EngineDataPlane", "ExecutionResult",
           "InProcessDaemonClient", "IntentExecutor", "PoolDaemon", "TurboBusDaemon", "TurboBusDaemonClient",
           "create_production_daemon"]
