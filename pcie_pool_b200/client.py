"""Buffers an application shares with the node's data plane.

``SharedPinnedCpuBuffer`` is a window into a POSIX shared-memory segment.
The application creates (owns) the segment; the daemon's executor or a
worker maps the same segment by name and page-locks its own mapping, so the
copy engines move the application's bytes with no intermediate copy.
``CudaIpcDeviceBuffer`` describes a device allocation exported through a
legacy CUDA IPC handle (64 bytes, hex on the wire) plus the buffer's offset
inside that allocation.

Public names, constructors and registration metadata keys match the
reference's client module (turbobus/client.py:57-352) so applications and
daemons of either project interoperate; the implementation is this
project's own: one ``_Segment`` per mapping owns the shared memory and its
base address, a buffer is a bounds-checked window onto it, and CUDA
page-locking is a separate, reversible record.
"""

from __future__ import annotations

import os
import threading
import uuid
from dataclasses import dataclass
from multiprocessing import resource_tracker, shared_memory
from typing import Any

from .schema import BufferRegistration, DaemonResponse

SHARED_HANDLE = "shared_pinned_cpu"
IPC_HANDLE = "cuda_ipc_device"
VMM_HANDLE = "cuda_vmm_fd"


def default_backend():
    from .backends.cuda import default_cuda_backend

    return default_cuda_backend


# ---- shared-memory segments -------------------------------------------------------------

class _Segment:
    """One mapping of a shared-memory segment and its base address.

    The creator owns the name (it unlinks it); a process that attaches to a
    segment it did not create maps it without registering the name with the
    ``multiprocessing`` resource tracker, which a spawned daemon shares with
    its parent and which would otherwise unlink the owner's segment."""

    _attach_lock = threading.Lock()

    def __init__(self, shm: shared_memory.SharedMemory, owner: bool) -> None:
        import numpy as np

        self.shm = shm
        self.owner = owner
        self.size = len(shm.buf)
        self.base = int(np.frombuffer(shm.buf, dtype=np.uint8).ctypes.data) if self.size else 0
        self.mapped = True
        self.unlinked = False

    @classmethod
    def create(cls, prefix: str, size: int) -> "_Segment":
        stem = "".join(c if c.isalnum() or c in "_-" else "_" for c in str(prefix)).strip("_") or "pcie_pool"
        return cls(shared_memory.SharedMemory(name=f"{stem}_{uuid.uuid4().hex}", create=True, size=size), True)

    @classmethod
    def attach(cls, name: str) -> "_Segment":
        try:
            return cls(shared_memory.SharedMemory(name=name, create=False, track=False), False)
        except TypeError:  # Python < 3.13: no ``track``; suppress the registration while attaching
            with cls._attach_lock:
                keep = resource_tracker.register
                resource_tracker.register = lambda *_a, **_k: None
                try:
                    return cls(shared_memory.SharedMemory(name=name, create=False), False)
                finally:
                    resource_tracker.register = keep

    @property
    def name(self) -> str:
        return str(self.shm.name)

    def unmap(self) -> None:
        if self.mapped:
            self.shm.close()
            self.mapped = False

    def unlink(self) -> None:
        if not self.unlinked:
            self.shm.unlink()
            self.unlinked = True


def validate_backing(offset: int, size: int, declared: int, mapped: int) -> None:
    """A registration may only name bytes that exist: its window must fit the
    size the owner declared, and the declared size must fit what was mapped."""
    end = int(offset) + int(size)
    if end > int(declared):
        raise ValueError(f"shared_pinned_cpu window ends at byte {end}, past the declared "
                         f"segment size {int(declared)}")
    if int(declared) > int(mapped) or end > int(mapped):
        raise ValueError(f"shared_pinned_cpu backing maps {int(mapped)} bytes, fewer than the "
                         f"{max(end, int(declared))} the registration needs")


check_backing = validate_backing


@dataclass
class _Pinning:
    backend: Any
    address: int


# ---- shared pinned host buffer ---------------------------------------------------------------

class SharedPinnedCpuBuffer:
    """``size_bytes`` bytes at ``offset_bytes`` of a shared-memory segment."""

    def __init__(self, buffer_id: str, job_id: str, segment: _Segment, offset_bytes: int, size_bytes: int,
                 declared_bytes: int | None = None) -> None:
        self.buffer_id = str(buffer_id)
        self.job_id = str(job_id)
        self._seg = segment
        self.offset_bytes = int(offset_bytes)
        self.size_bytes = int(size_bytes)
        self.shared_memory_size_bytes = int(segment.size if declared_bytes is None else declared_bytes)
        self._pin: _Pinning | None = None

    # -- construction --------------------------------------------------------------------
    @classmethod
    def allocate(cls, buffer_id: str, job_id: str, size_bytes: int, *,
                 name_prefix: str = "pcie_pool") -> "SharedPinnedCpuBuffer":
        """Create a new segment of ``size_bytes`` owned by this process."""
        n = int(size_bytes)
        if n <= 0:
            raise ValueError(f"a shared buffer needs a positive size, got {n}")
        return cls(buffer_id, job_id, _Segment.create(name_prefix, n), 0, n)

    @classmethod
    def open_from_registration(cls, registration: BufferRegistration) -> "SharedPinnedCpuBuffer":
        """Map the segment a registration names (this process does not own it)."""
        if not isinstance(registration, BufferRegistration):
            raise TypeError("registration must be a BufferRegistration")
        if registration.handle_type != SHARED_HANDLE:
            raise ValueError(f"registration {registration.buffer_id} is a {registration.handle_type} buffer, "
                             f"not {SHARED_HANDLE}")
        md = registration.metadata
        for key in ("shared_memory_name", "offset_bytes", "shared_memory_size_bytes"):
            if key not in md:
                raise ValueError(f"{SHARED_HANDLE} registration lacks metadata {key!r}")
        seg = _Segment.attach(str(md["shared_memory_name"]))
        try:
            validate_backing(int(md["offset_bytes"]), registration.size_bytes, int(md["shared_memory_size_bytes"]),
                             seg.size)
        except ValueError:
            seg.unmap()
            raise
        return cls(registration.buffer_id, registration.job_id, seg, int(md["offset_bytes"]),
                   registration.size_bytes, int(md["shared_memory_size_bytes"]))

    # -- identity ----------------------------------------------------------------------------
    @property
    def shared_memory_name(self) -> str:
        return self._seg.name

    @property
    def owner(self) -> bool:
        return self._seg.owner

    @property
    def closed(self) -> bool:
        return not self._seg.mapped

    @property
    def metadata(self) -> dict[str, object]:
        return {"shared_memory_name": self.shared_memory_name, "offset_bytes": self.offset_bytes,
                "shared_memory_size_bytes": self.shared_memory_size_bytes}

    def buffer_registration(self) -> BufferRegistration:
        return BufferRegistration(buffer_id=self.buffer_id, job_id=self.job_id, kind="cpu_pinned",
                                  size_bytes=self.size_bytes, pinned=True, handle_type=SHARED_HANDLE,
                                  metadata=self.metadata)

    def register_with_daemon(self, daemon_client) -> DaemonResponse:
        r = self.buffer_registration()
        return daemon_client.register_buffer(buffer_id=r.buffer_id, job_id=r.job_id, kind=r.kind,
                                             size_bytes=r.size_bytes, pinned=True, handle_type=r.handle_type,
                                             metadata=dict(r.metadata))

    # -- data ----------------------------------------------------------------------------------
    def _live(self) -> _Segment:
        if not self._seg.mapped:
            raise RuntimeError(f"shared buffer {self.buffer_id} is closed")
        return self._seg

    @property
    def address(self) -> int:
        """Address of the window's first byte in this process."""
        return self._live().base + self.offset_bytes

    @property
    def view(self) -> memoryview:
        return self._live().shm.buf[self.offset_bytes:self.offset_bytes + self.size_bytes]

    def numpy(self):
        """The window as a writable uint8 array (no copy)."""
        import numpy as np

        return np.frombuffer(self._live().shm.buf, dtype=np.uint8, count=self.size_bytes, offset=self.offset_bytes)

    def _span(self, offset: int, n: int) -> slice:
        o, n = int(offset), int(n)
        if o < 0 or n < 0 or o + n > self.size_bytes:
            raise ValueError(f"bytes [{o}, {o + n}) fall outside shared buffer {self.buffer_id} "
                             f"of {self.size_bytes} bytes")
        return slice(o, o + n)

    def write(self, data, offset: int = 0) -> None:
        import numpy as np

        src = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
        self.numpy()[self._span(offset, src.size)] = src

    def read(self, size: int | None = None, offset: int = 0) -> bytes:
        n = self.size_bytes - int(offset) if size is None else int(size)
        return self.numpy()[self._span(offset, n)].tobytes()

    # -- page-locking for CUDA ----------------------------------------------------------------
    @property
    def cuda_registered(self) -> bool:
        return self._pin is not None

    def register_for_cuda(self, backend=None) -> None:
        if self._pin is None:
            b = backend or default_backend()
            addr = self.address
            b.register_host_memory(addr, self.size_bytes)
            self._pin = _Pinning(b, addr)

    def unregister_from_cuda(self) -> None:
        pin, self._pin = self._pin, None
        if pin is not None:
            pin.backend.unregister_host_memory(pin.address)

    # -- lifetime ---------------------------------------------------------------------------------
    def close(self) -> None:
        """Drop this process's mapping (CUDA page-locking first)."""
        if self._seg.mapped:
            self.unregister_from_cuda()
            self._seg.unmap()

    def unlink(self) -> None:
        """Remove the segment's name (the memory lives until every mapping closes)."""
        self._seg.unlink()

    def release(self) -> None:
        """Close; the owner also unlinks."""
        try:
            self.close()
        finally:
            if self.owner:
                self.unlink()

    def __enter__(self) -> "SharedPinnedCpuBuffer":
        return self

    def __exit__(self, *exc) -> None:
        self.release()

    def __repr__(self) -> str:
        return (f"SharedPinnedCpuBuffer({self.buffer_id!r}, job={self.job_id!r}, segment={self.shared_memory_name!r}, "
                f"offset={self.offset_bytes}, size={self.size_bytes}, owner={self.owner})")


class SharedPinnedCpuBufferAllocator:
    """Allocates owned shared buffers whose segment names share a prefix."""

    def __init__(self, name_prefix: str = "pcie_pool") -> None:
        self.name_prefix = str(name_prefix)

    def allocate(self, buffer_id: str, job_id: str, size_bytes: int) -> SharedPinnedCpuBuffer:
        return SharedPinnedCpuBuffer.allocate(buffer_id, job_id, size_bytes, name_prefix=self.name_prefix)


# ---- CUDA IPC device buffer -------------------------------------------------------------------

@dataclass(frozen=True)
class CudaIpcDeviceBuffer:
    """A device buffer another process opens through its allocation's IPC
    handle; ``ipc_offset`` is the buffer's distance from the allocation base
    (the handle always maps the base)."""

    buffer_id: str
    job_id: str
    device_index: int
    size_bytes: int
    cuda_ipc_handle: bytes
    device_ptr: int | None = None
    ipc_offset: int = 0

    @classmethod
    def from_device_pointer(cls, buffer_id: str, job_id: str, device_index: int, size_bytes: int,
                            device_ptr: int, *, backend=None) -> "CudaIpcDeviceBuffer":
        if int(size_bytes) <= 0 or int(device_ptr) <= 0:
            raise ValueError("an IPC buffer needs a positive size and a device pointer")
        b = backend or default_backend()
        if callable(getattr(b, "set_device", None)):
            b.set_device(int(device_index))
        base_offset = getattr(b, "device_allocation_offset", None)
        return cls(str(buffer_id), str(job_id), int(device_index), int(size_bytes),
                   b.export_device_ipc_handle(int(device_ptr)), int(device_ptr),
                   int(base_offset(int(device_ptr))) if callable(base_offset) else 0)

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
                                  address=self.device_ptr, handle_type=IPC_HANDLE, metadata=self.metadata)

    def register_with_daemon(self, daemon_client) -> DaemonResponse:
        r = self.buffer_registration()
        return daemon_client.register_buffer(buffer_id=r.buffer_id, job_id=r.job_id, kind=r.kind,
                                             size_bytes=r.size_bytes, device_index=r.device_index, address=r.address,
                                             handle_type=r.handle_type, metadata=dict(r.metadata))


# ---- CUDA VMM device buffer (POSIX file descriptor) ----------------------------------------------

class CudaVmmDeviceBuffer:
    """A device buffer made with CUDA virtual memory management and exported
    as a POSIX file descriptor.  The descriptor is passed to the daemon with
    the registration (``SCM_RIGHTS`` on its socket; the number itself for an
    in-process daemon), which imports and maps the allocation.  Unlike a
    legacy IPC handle the export is an ordinary descriptor: it can be
    duplicated, passed on and closed, and the memory lives until every
    mapping and descriptor is gone.  Legacy IPC (``CudaIpcDeviceBuffer``)
    stays available as the other import path."""

    def __init__(self, buffer_id: str, job_id: str, device_index: int, size_bytes: int, device_ptr: int,
                 mapped_bytes: int, fd: int, owner: bool) -> None:
        self.buffer_id, self.job_id = str(buffer_id), str(job_id)
        self.device_index, self.size_bytes = int(device_index), int(size_bytes)
        self.device_ptr, self.mapped_bytes, self.fd, self.owner = int(device_ptr), int(mapped_bytes), int(fd), owner

    @classmethod
    def allocate(cls, buffer_id: str, job_id: str, device_index: int, size_bytes: int) -> "CudaVmmDeviceBuffer":
        from ._native import native

        if int(size_bytes) <= 0:
            raise ValueError("a VMM buffer needs a positive size")
        ptr, mapped, fd = native().vmm_alloc(int(device_index), int(size_bytes))
        return cls(buffer_id, job_id, device_index, size_bytes, ptr, mapped, fd, True)

    @classmethod
    def import_fd(cls, buffer_id: str, job_id: str, device_index: int, size_bytes: int, fd: int,
                  mapped_bytes: int) -> "CudaVmmDeviceBuffer":
        """Map a descriptor received from the exporting process."""
        from ._native import native

        ptr = native().vmm_import(int(fd), int(device_index), int(mapped_bytes))
        return cls(buffer_id, job_id, device_index, size_bytes, ptr, mapped_bytes, fd, False)

    @property
    def metadata(self) -> dict[str, object]:
        return {"vmm_mapped_bytes": self.mapped_bytes}

    def buffer_registration(self, *, with_fd: bool = False) -> BufferRegistration:
        md = dict(self.metadata)
        if with_fd:
            md["vmm_fd"] = self.fd
        return BufferRegistration(buffer_id=self.buffer_id, job_id=self.job_id, kind="gpu",
                                  size_bytes=self.size_bytes, device_index=self.device_index,
                                  address=self.device_ptr, handle_type=VMM_HANDLE, metadata=md)

    def register_with_daemon(self, daemon_client) -> DaemonResponse:
        r = self.buffer_registration()
        return daemon_client.register_buffer(buffer_id=r.buffer_id, job_id=r.job_id, kind=r.kind,
                                             size_bytes=r.size_bytes, device_index=r.device_index,
                                             address=r.address, handle_type=r.handle_type,
                                             metadata=dict(r.metadata), fds=[self.fd])

    def release(self) -> None:
        from ._native import native

        if self.device_ptr:
            native().vmm_release(self.device_ptr)
            self.device_ptr = 0
        if self.owner and self.fd >= 0:
            os.close(self.fd)
            self.fd = -1


__all__ = ["CudaIpcDeviceBuffer", "CudaVmmDeviceBuffer", "SharedPinnedCpuBuffer", "SharedPinnedCpuBufferAllocator",
           "validate_backing"]
