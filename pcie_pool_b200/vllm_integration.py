"""Top-level alias of ``pcie_pool_b200.adapters.vllm_integration`` (the reference exposes
the same module both at package level and under adapters)."""

import sys as _sys

from .adapters import vllm_integration as _impl

_sys.modules[__name__] = _impl
