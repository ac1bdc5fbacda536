"""CUDA backend: the native core (``pcie_pool_b200._C``) plus ``PoolRuntime``.

Same facade as the reference's ``CudaNativeBackend``
(turbobus/backends/cuda.py:9-172) so the worker and client layers stay
backend-agnostic; a runtime here is a persistent ``PoolRuntime``.
"""

from __future__ import annotations

from typing import Any, Iterable

from ..schema import TransferMode

IPC_HANDLE_BYTES = 64


class CudaNativeBackend:
    """``runtime_engine_module``: a module whose ``_turbobus`` attribute is the
    native core to use (the reference's constructor argument,
    turbobus/backends/cuda.py:12); ``native_loader``: a callable returning it.
    Neither: the in-tree ``pcie_pool_b200._C``."""

    def __init__(self, runtime_engine_module=None, native_loader=None) -> None:
        self._loader = native_loader
        native_core = getattr(runtime_engine_module, "_turbobus", None)
        if native_core is not None:
            self._loader = lambda: native_core

    def _native(self):
        if self._loader is not None:
            return self._loader()
        from .._native import native

        return native()

    def bind_runtime(self, native_module: Any, torch_module: Any = None) -> None:
        """Use ``native_module`` as the native core (tests inject a stand-in;
        turbobus/backends/cuda.py:15-17).  ``torch_module`` is accepted for the
        same signature; this backend imports torch itself where it needs it."""
        self._loader = (lambda: native_module) if native_module is not None else None

    def _call(self, name: str, what: str):
        fn = getattr(self._native(), name, None)
        if not callable(fn):
            raise RuntimeError(f"native runtime does not support {what}")
        return fn

    def require_available(self) -> None:
        self._native()

    def require_torch(self) -> None:
        import torch  # noqa: F401

    def set_device(self, device_index: int) -> None:
        d = int(device_index)
        if d < 0:
            raise ValueError("device_index must be non-negative")
        self._call("set_device", "device selection")(d)

    def transfer_mode_value(self, mode: TransferMode | str) -> TransferMode:
        return TransferMode(mode)

    def create_runtime(self, options: Any) -> Any:
        from ..runtime_engine import PoolRuntime

        self.require_available()
        return PoolRuntime(options)

    def initialize_runtime(self, runtime: Any, target_device: int, relay_gpus: Iterable[int]) -> None:
        init = getattr(runtime, "init", None)
        if not callable(init):
            raise RuntimeError("runtime does not support initialization")
        init(int(target_device), [int(g) for g in relay_gpus])

    def make_ranges(self, ranges: Iterable, source_bytes: int, destination_bytes: int) -> list:
        from ..runtime_engine import validate_ranges

        return validate_ranges(ranges, source_bytes, destination_bytes)

    def make_transfer_plan(self, plan: Any) -> Any:
        from ..plan_trace import transfer_plan_to_dict, validate_plan_dict

        d = transfer_plan_to_dict(plan)
        validate_plan_dict(d)
        return d

    def register_host_memory(self, host_ptr: int, bytes_: int) -> None:
        if int(host_ptr) <= 0:
            raise ValueError("host_ptr must be positive")
        if int(bytes_) <= 0:
            raise ValueError("bytes must be positive")
        self._call("host_register", "host memory registration")(int(host_ptr), int(bytes_))

    def unregister_host_memory(self, host_ptr: int) -> None:
        if int(host_ptr) <= 0:
            raise ValueError("host_ptr must be positive")
        self._call("host_unregister", "host memory registration")(int(host_ptr))

    def export_device_ipc_handle(self, device_ptr: int) -> bytes:
        if int(device_ptr) <= 0:
            raise ValueError("device_ptr must be positive")
        return ipc_handle_bytes(bytes(self._call("export_ipc_handle", "CUDA IPC export")(int(device_ptr))))

    def device_allocation_offset(self, device_ptr: int) -> int:
        """Offset of ``device_ptr`` inside its CUDA allocation (an IPC handle
        names the allocation; the receiver adds this offset to the mapping)."""
        if int(device_ptr) <= 0:
            raise ValueError("device_ptr must be positive")
        return int(device_ptr) - int(self._call("allocation_base", "allocation lookup")(int(device_ptr)))

    def open_device_ipc_handle(self, cuda_ipc_handle: bytes | bytearray | str, device_index: int = 0) -> int:
        handle = coerce_ipc_handle(cuda_ipc_handle)  # malformed handles fail before the native call
        ptr = int(self._call("open_ipc_handle", "CUDA IPC open")(handle, int(device_index)))
        if ptr <= 0:
            raise RuntimeError("native runtime returned an invalid CUDA IPC pointer")
        return ptr

    def close_device_ipc_handle(self, device_ptr: int) -> None:
        if int(device_ptr) <= 0:
            raise ValueError("device_ptr must be positive")
        self._call("close_ipc_handle", "CUDA IPC close")(int(device_ptr))

    def fetch_plan_to_gpu(self, runtime, host_ptr, host_bytes, target_ptr, target_bytes, plan):
        fn = getattr(runtime, "fetch_plan_to_gpu", None)
        if not callable(fn):
            raise RuntimeError("runtime does not support exact transfer plans")
        return fn(host_ptr, host_bytes, target_ptr, target_bytes, plan)

    def offload_plan_to_cpu(self, runtime, target_ptr, target_bytes, host_ptr, host_bytes, plan):
        fn = getattr(runtime, "offload_plan_to_cpu", None)
        if not callable(fn):
            raise RuntimeError("runtime does not support exact transfer plans")
        return fn(target_ptr, target_bytes, host_ptr, host_bytes, plan)

    def wait(self, runtime, handle) -> None:
        fn = getattr(runtime, "wait", None)
        if not callable(fn):
            raise RuntimeError("runtime does not support transfer waiting")
        fn(handle)

    def stats(self, runtime, handle):
        fn = getattr(runtime, "stats", None)
        if not callable(fn):
            raise RuntimeError("runtime does not support transfer stats")
        return fn(handle)


def coerce_ipc_handle(handle: bytes | bytearray | str) -> bytes:
    if isinstance(handle, str):
        try:
            return ipc_handle_bytes(bytes.fromhex(handle))
        except ValueError as exc:
            if "64 bytes" in str(exc):
                raise
            raise ValueError("cuda_ipc_handle string must be hex encoded") from exc
    return ipc_handle_bytes(bytes(handle))


def ipc_handle_bytes(handle: bytes) -> bytes:
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("cuda_ipc_handle must be 64 bytes")
    return handle


default_cuda_backend = CudaNativeBackend()

__all__ = ["CudaNativeBackend", "coerce_ipc_handle", "default_cuda_backend"]
