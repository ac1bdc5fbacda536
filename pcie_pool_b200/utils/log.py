"""Structured logging: ``logger("daemon").info("transfer_complete",
transfer_id=..., gb_per_s=...)`` emits one ``event key=value ...`` record
through the standard ``logging`` module under ``pcie_pool_b200.<name>``, so
deployments route, filter and level it like any other library log."""

from __future__ import annotations

import logging
import os

ROOT = "pcie_pool_b200"


def _fmt(v) -> str:
    s = f"{v:.3f}" if isinstance(v, float) else str(v)
    return s.replace(" ", "_") if s else '""'


class StructuredLogger:
    def __init__(self, name: str) -> None:
        self._log = logging.getLogger(f"{ROOT}.{name}")

    def _emit(self, level: int, event: str, fields: dict) -> None:
        if self._log.isEnabledFor(level):
            self._log.log(level, " ".join([event] + [f"{k}={_fmt(v)}" for k, v in fields.items()]))

    def debug(self, event: str, **fields) -> None:
        self._emit(logging.DEBUG, event, fields)

    def info(self, event: str, **fields) -> None:
        self._emit(logging.INFO, event, fields)

    def warning(self, event: str, **fields) -> None:
        self._emit(logging.WARNING, event, fields)

    def error(self, event: str, **fields) -> None:
        self._emit(logging.ERROR, event, fields)


def logger(name: str) -> StructuredLogger:
    return StructuredLogger(name)


def configure_from_env() -> None:
    """``PCIE_POOL_LOG=debug|info|warning`` attaches a stderr handler."""
    level = os.environ.get("PCIE_POOL_LOG", "").upper()
    if not level:
        return
    root = logging.getLogger(ROOT)
    if not root.handlers:
        h = logging.StreamHandler()
        h.setFormatter(logging.Formatter("%(asctime)s %(name)s %(levelname)s %(message)s"))
        root.addHandler(h)
    root.setLevel(getattr(logging, level, logging.INFO))


__all__ = ["StructuredLogger", "configure_from_env", "logger"]
