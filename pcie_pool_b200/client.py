"""Cross-process buffers.

``SharedPinnedCpuBuffer``: POSIX shared memory that the owner and the data
plane both map and page-lock (``cudaHostRegister``, portable + mapped), so the
daemon's executor can DMA from the application's host memory without a copy.
``CudaIpcDeviceBuffer``: a device allocation exported with a legacy CUDA IPC
handle (64 bytes, hex on the wire).  Same API as the reference
(turbobus/client.py:57-352).
"""

from __future__ import annotations

import ctypes
import os
import threading
import uuid
from dataclasses import dataclass, field
from multiprocessing import resource_tracker, shared_memory
from typing import Any

from .schema import BufferRegistration, DaemonResponse

_OWNED_NAMES: set[str] = set()
_ATTACH_LOCK = threading.Lock()


def _shm_name(prefix: str) -> str:
    clean = "".join(c if c.isalnum() or c in "_-" else "_" for c in str(prefix)).strip("_") or "pcie_pool"
    return f"{clean}_{uuid.uuid4().hex}"


def _tracker_name(shm: shared_memory.SharedMemory) -> str:
    name = getattr(shm, "_name", None) or str(shm.name)
    return name if (os.name != "posix" or name.startswith("/")) else f"/{name}"


def _open_borrowed(name: str) -> shared_memory.SharedMemory:
    """Map someone else's segment without making this process its owner."""
    try:
        return shared_memory.SharedMemory(name=name, create=False, track=False)
    except TypeError:  # Python < 3.13 has no ``track``
        # Attaching would register the name with the resource tracker, which
        # processes started by ``multiprocessing`` share with their parent; a
        # register + unregister pair here would drop the owner's registration.
        # Skip the registration for the duration of the attach instead.
        with _ATTACH_LOCK:
            saved = resource_tracker.register
            resource_tracker.register = lambda *_a, **_k: None
            try:
                return shared_memory.SharedMemory(name=name, create=False)
            finally:
                resource_tracker.register = saved


def default_backend():
    from .backends.cuda import default_cuda_backend

    return default_cuda_backend


@dataclass
class SharedPinnedCpuBuffer:
    buffer_id: str
    job_id: str
    size_bytes: int
    shared_memory_name: str
    shared_memory_size_bytes: int
    _shared_memory: shared_memory.SharedMemory = field(repr=False, compare=False)
    offset_bytes: int = 0
    owner: bool = False
    _cuda_registered: bool = field(default=False, init=False, repr=False)
    _cuda_backend: Any | None = field(default=None, init=False, repr=False)
    _cuda_registered_address: int | None = field(default=None, init=False, repr=False)
    _closed: bool = field(default=False, init=False, repr=False)
    _unlinked: bool = field(default=False, init=False, repr=False)

    @classmethod
    def allocate(cls, buffer_id: str, job_id: str, size_bytes: int, *,
                 name_prefix: str = "pcie_pool") -> "SharedPinnedCpuBuffer":
        size_bytes = int(size_bytes)
        if size_bytes <= 0:
            raise ValueError("size_bytes must be positive")
        shm = shared_memory.SharedMemory(name=_shm_name(name_prefix), create=True, size=size_bytes)
        _OWNED_NAMES.add(_tracker_name(shm))
        return cls(buffer_id=str(buffer_id), job_id=str(job_id), size_bytes=size_bytes,
                   shared_memory_name=shm.name, shared_memory_size_bytes=size_bytes, owner=True,
                   _shared_memory=shm)

    @classmethod
    def open_from_registration(cls, registration: BufferRegistration) -> "SharedPinnedCpuBuffer":
        if not isinstance(registration, BufferRegistration):
            raise TypeError("registration must be a BufferRegistration")
        if registration.handle_type != "shared_pinned_cpu":
            raise ValueError("registration must be a shared_pinned_cpu buffer")
        md = registration.metadata
        if "shared_memory_size_bytes" not in md:
            raise ValueError("shared_pinned_cpu metadata requires shared_memory_size_bytes")
        name, off, declared = str(md["shared_memory_name"]), int(md["offset_bytes"]), int(md["shared_memory_size_bytes"])
        shm = _open_borrowed(name)
        try:
            check_backing(off, registration.size_bytes, declared, len(shm.buf))
        except Exception:
            shm.close()
            raise
        return cls(buffer_id=registration.buffer_id, job_id=registration.job_id,
                   size_bytes=registration.size_bytes, shared_memory_name=name,
                   shared_memory_size_bytes=declared, offset_bytes=off, owner=False, _shared_memory=shm)

    @property
    def metadata(self) -> dict[str, object]:
        return {"shared_memory_name": self.shared_memory_name, "offset_bytes": self.offset_bytes,
                "shared_memory_size_bytes": self.shared_memory_size_bytes}

    @property
    def view(self) -> memoryview:
        if self._closed:
            raise RuntimeError("shared CPU buffer is closed")
        return self._shared_memory.buf[self.offset_bytes:self.offset_bytes + self.size_bytes]

    @property
    def address(self) -> int:
        v = self.view
        c = ctypes.c_char.from_buffer(v)
        try:
            return ctypes.addressof(c)
        finally:
            del c
            v.release()

    @property
    def closed(self) -> bool:
        return self._closed

    @property
    def cuda_registered(self) -> bool:
        return self._cuda_registered

    def numpy(self):
        import numpy as np

        return np.frombuffer(self._shared_memory.buf, dtype=np.uint8, count=self.size_bytes,
                             offset=self.offset_bytes)

    def write(self, data, offset: int = 0) -> None:
        payload = bytes(data)
        offset = int(offset)
        if offset < 0:
            raise ValueError("offset must be non-negative")
        if offset + len(payload) > self.size_bytes:
            raise ValueError("write exceeds shared CPU buffer")
        v = self.view
        try:
            v[offset:offset + len(payload)] = payload
        finally:
            v.release()

    def read(self, size: int | None = None, offset: int = 0) -> bytes:
        offset = int(offset)
        if offset < 0:
            raise ValueError("offset must be non-negative")
        n = self.size_bytes - offset if size is None else int(size)
        if n < 0:
            raise ValueError("size must be non-negative")
        if offset + n > self.size_bytes:
            raise ValueError("read exceeds shared CPU buffer")
        v = self.view
        try:
            return bytes(v[offset:offset + n])
        finally:
            v.release()

    def buffer_registration(self) -> BufferRegistration:
        return BufferRegistration(buffer_id=self.buffer_id, job_id=self.job_id, kind="cpu_pinned",
                                  size_bytes=self.size_bytes, pinned=True, handle_type="shared_pinned_cpu",
                                  metadata=self.metadata)

    def register_with_daemon(self, daemon_client) -> DaemonResponse:
        return daemon_client.register_buffer(buffer_id=self.buffer_id, job_id=self.job_id, kind="cpu_pinned",
                                             size_bytes=self.size_bytes, pinned=True,
                                             handle_type="shared_pinned_cpu", metadata=self.metadata)

    def register_for_cuda(self, backend=None) -> None:
        if self._cuda_registered:
            return
        backend = backend or default_backend()
        addr = self.address
        backend.register_host_memory(addr, self.size_bytes)
        self._cuda_backend, self._cuda_registered_address, self._cuda_registered = backend, addr, True

    def unregister_from_cuda(self) -> None:
        if not self._cuda_registered:
            return
        (self._cuda_backend or default_backend()).unregister_host_memory(self._cuda_registered_address)
        self._cuda_backend, self._cuda_registered_address, self._cuda_registered = None, None, False

    def close(self) -> None:
        if self._closed:
            return
        self.unregister_from_cuda()
        self._shared_memory.close()
        self._closed = True

    def unlink(self) -> None:
        if self._unlinked:
            return
        self._shared_memory.unlink()
        _OWNED_NAMES.discard(_tracker_name(self._shared_memory))
        self._unlinked = True

    def release(self) -> None:
        try:
            self.close()
        finally:
            if self.owner:
                self.unlink()

    def __enter__(self) -> "SharedPinnedCpuBuffer":
        return self

    def __exit__(self, *exc) -> None:
        self.release()


class SharedPinnedCpuBufferAllocator:
    def __init__(self, name_prefix: str = "pcie_pool") -> None:
        self.name_prefix = str(name_prefix)

    def allocate(self, buffer_id: str, job_id: str, size_bytes: int) -> SharedPinnedCpuBuffer:
        return SharedPinnedCpuBuffer.allocate(buffer_id, job_id, size_bytes, name_prefix=self.name_prefix)


@dataclass(frozen=True)
class CudaIpcDeviceBuffer:
    buffer_id: str
    job_id: str
    device_index: int
    size_bytes: int
    cuda_ipc_handle: bytes
    device_ptr: int | None = None
    ipc_offset: int = 0  # device_ptr - base of its allocation (the handle maps the base)

    @classmethod
    def from_device_pointer(cls, buffer_id: str, job_id: str, device_index: int, size_bytes: int,
                            device_ptr: int, *, backend=None) -> "CudaIpcDeviceBuffer":
        if int(size_bytes) <= 0:
            raise ValueError("size_bytes must be positive")
        if int(device_ptr) <= 0:
            raise ValueError("device_ptr must be positive")
        backend = backend or default_backend()
        setter = getattr(backend, "set_device", None)
        if callable(setter):
            setter(int(device_index))
        off = getattr(backend, "device_allocation_offset", None)
        return cls(buffer_id=str(buffer_id), job_id=str(job_id), device_index=int(device_index),
                   size_bytes=int(size_bytes), cuda_ipc_handle=backend.export_device_ipc_handle(int(device_ptr)),
                   device_ptr=int(device_ptr), ipc_offset=int(off(int(device_ptr))) if callable(off) else 0)

    @classmethod
    def from_tensor(cls, buffer_id: str, job_id: str, tensor, *, backend=None) -> "CudaIpcDeviceBuffer":
        return cls.from_device_pointer(buffer_id, job_id, tensor.device.index, tensor.numel() * tensor.element_size(),
                                       tensor.data_ptr(), backend=backend)

    @property
    def metadata(self) -> dict[str, object]:
        md: dict[str, object] = {"cuda_ipc_handle": self.cuda_ipc_handle.hex()}
        if self.ipc_offset:
            md["cuda_ipc_offset"] = int(self.ipc_offset)
        return md

    def buffer_registration(self) -> BufferRegistration:
        return BufferRegistration(buffer_id=self.buffer_id, job_id=self.job_id, kind="gpu",
                                  size_bytes=self.size_bytes, device_index=self.device_index,
                                  address=self.device_ptr, handle_type="cuda_ipc_device", metadata=self.metadata)

    def register_with_daemon(self, daemon_client) -> DaemonResponse:
        return daemon_client.register_buffer(buffer_id=self.buffer_id, job_id=self.job_id, kind="gpu",
                                             size_bytes=self.size_bytes, device_index=self.device_index,
                                             address=self.device_ptr, handle_type="cuda_ipc_device",
                                             metadata=self.metadata)


def check_backing(offset: int, size: int, declared: int, actual: int) -> None:
    span = int(offset) + int(size)
    if span > int(declared):
        raise ValueError("shared_pinned_cpu shared_memory_size_bytes is smaller than buffer span")
    if span > int(actual):
        raise ValueError("shared_pinned_cpu backing is smaller than authorized buffer span")
    if int(declared) > int(actual):
        raise ValueError("shared_pinned_cpu backing is smaller than declared shared memory size")


__all__ = ["CudaIpcDeviceBuffer", "SharedPinnedCpuBuffer", "SharedPinnedCpuBufferAllocator"]
