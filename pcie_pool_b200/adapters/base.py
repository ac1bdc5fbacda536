"""Marker protocol for framework-facing adapters."""

from typing import Protocol


class FrameworkAdapter(Protocol):
    """Anything that moves a framework's tensors through the pool."""


__all__ = ["FrameworkAdapter"]
