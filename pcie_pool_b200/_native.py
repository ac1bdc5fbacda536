"""Loader for the native core ``pcie_pool_b200._C``.

On a machine with a visible GPU a missing or broken extension is an error
(raised on first use), never a silent fallback to a slower path.
"""

from __future__ import annotations

import importlib
import os
from types import ModuleType

_MOD: ModuleType | None = None
_ERR: BaseException | None = None


def _gpu_visible() -> bool:
    if os.environ.get("CUDA_VISIBLE_DEVICES", None) == "":
        return False
    return any(os.path.exists(p) for p in ("/dev/nvidia0", "/dev/nvidiactl"))


def native(build_if_missing: bool = True) -> ModuleType:
    """Return the loaded extension module, building it in-tree if needed."""
    global _MOD, _ERR
    if _MOD is not None:
        return _MOD
    try:
        _MOD = importlib.import_module("pcie_pool_b200._C")
        return _MOD
    except ImportError as exc:  # pragma: no cover - depends on build state
        _ERR = exc
    if build_if_missing and os.environ.get("PCIE_POOL_NO_BUILD") != "1":
        from . import _build

        _build.build()
        _MOD = importlib.import_module("pcie_pool_b200._C")
        return _MOD
    raise RuntimeError(
        "pcie_pool_b200 native extension is not built; run "
        "`python -m pcie_pool_b200._build`"
        + (" (a GPU is visible, so no fallback is used)" if _gpu_visible() else "")
    ) from _ERR


def available() -> bool:
    try:
        native(build_if_missing=False)
        return True
    except Exception:
        return False
