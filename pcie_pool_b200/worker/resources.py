"""Bind a worker request's client buffers into this process.

The host side is the client's POSIX shared-memory segment (opened, then
page-locked with ``cudaHostRegister(Portable|Mapped)``); the device side is
the client's CUDA IPC handle (opened with lazy peer access).  Both are closed
when the binding exits.  Behaviour as turbobus/worker/resources.py:14-168;
the CUDA calls go through a backend object so tests can bind fake handles.
"""

from __future__ import annotations

from dataclasses import dataclass

from ..client import SharedPinnedCpuBuffer
from ..schema import BufferRegistration, WorkerBufferHandle, WorkerDataPlaneRequest


class WorkerDataPlaneResourceError(RuntimeError):
    pass


@dataclass(frozen=True)
class WorkerDataPlaneResources:
    request: WorkerDataPlaneRequest
    cpu_buffer: SharedPinnedCpuBuffer
    device_ptr: int
    device_bytes: int
    device_index: int
    cuda_host_registered: bool = False

    @property
    def host_ptr(self) -> int:
        return self.cpu_buffer.address

    @property
    def host_bytes(self) -> int:
        return self.cpu_buffer.size_bytes

    source_cpu_buffer = property(lambda self: self.cpu_buffer)
    source_host_ptr = property(lambda self: self.host_ptr)
    source_bytes = property(lambda self: self.host_bytes)
    target_device_ptr = property(lambda self: self.device_ptr)
    target_device_bytes = property(lambda self: self.device_bytes)

    def close(self) -> None:
        """Close this process's mapping of the shared CPU buffer."""
        self.cpu_buffer.close()

    def as_dict(self) -> dict[str, object]:
        return {"transfer_id": self.request.transfer_id, "direction": self.request.direction,
                "cpu_buffer_id": self.cpu_buffer.buffer_id, "host_bytes": self.host_bytes,
                "shared_memory_name": self.cpu_buffer.shared_memory_name,
                "device_index": self.device_index, "device_bytes": self.device_bytes,
                "cuda_host_registered": self.cuda_host_registered}


class WorkerDataPlaneResourceBinding:
    """Context manager: ``with binder.bind(request) as resources: ...``."""

    def __init__(self, request: WorkerDataPlaneRequest, backend=None, register_cuda_host: bool = True) -> None:
        if not isinstance(request, WorkerDataPlaneRequest):
            raise TypeError("request must be a WorkerDataPlaneRequest")
        self.request = request
        self.backend = backend
        self.register_cuda_host = bool(register_cuda_host)
        self._resources: WorkerDataPlaneResources | None = None
        self._cpu: SharedPinnedCpuBuffer | None = None
        self._dev_ptr: int | None = None

    def _be(self):
        if self.backend is None:
            from ..backends.cuda import default_cuda_backend

            self.backend = default_cuda_backend
        return self.backend

    def __enter__(self) -> WorkerDataPlaneResources:
        req = self.request
        cpu_h, dev_h = (req.src_handle, req.dst_handle) if req.direction == "h2d" else (req.dst_handle,
                                                                                         req.src_handle)
        try:
            self._cpu = SharedPinnedCpuBuffer.open_from_registration(_registration(cpu_h))
            if self.register_cuda_host:
                self._cpu.register_for_cuda(self._be())
            if dev_h.handle_type != "cuda_ipc_device" or "cuda_ipc_handle" not in dev_h.metadata:
                raise WorkerDataPlaneResourceError("worker device handle must carry a CUDA IPC handle")
            be = self._be()
            if dev_h.device_index is not None:
                be.set_device(int(dev_h.device_index))
            self._dev_ptr = int(be.open_device_ipc_handle(str(dev_h.metadata["cuda_ipc_handle"]),
                                                          int(dev_h.device_index or 0)))
            # the handle maps its allocation's base; the buffer may start inside it
            dev_ptr = self._dev_ptr + int(dev_h.metadata.get("cuda_ipc_offset", 0) or 0)
            self._resources = WorkerDataPlaneResources(req, self._cpu, dev_ptr, dev_h.size_bytes,
                                                       int(dev_h.device_index or 0), self.register_cuda_host)
            return self._resources
        except WorkerDataPlaneResourceError:
            self._close()
            raise
        except Exception as exc:  # noqa: BLE001 - surfaced as a resource error
            self._close()
            raise WorkerDataPlaneResourceError(f"failed to bind worker data-plane resources: {exc}") from exc

    def __exit__(self, exc_type, exc, tb) -> None:
        self._close()

    def _close(self) -> None:
        if self._dev_ptr is not None:
            try:
                self._be().close_device_ipc_handle(self._dev_ptr)
            finally:
                self._dev_ptr = None
        if self._cpu is not None:
            try:
                if self._cpu.cuda_registered:
                    self._cpu.unregister_from_cuda()
            finally:
                self._cpu.close()
                self._cpu = None
        self._resources = None


class WorkerDataPlaneResourceBinder:
    def __init__(self, backend=None, register_cuda_host: bool = True) -> None:
        self.backend = backend
        self.register_cuda_host = bool(register_cuda_host)

    def bind(self, request: WorkerDataPlaneRequest) -> WorkerDataPlaneResourceBinding:
        return WorkerDataPlaneResourceBinding(request, backend=self.backend,
                                              register_cuda_host=self.register_cuda_host)


def _registration(handle: WorkerBufferHandle) -> BufferRegistration:
    if not isinstance(handle, WorkerBufferHandle):
        raise TypeError("handle must be a WorkerBufferHandle")
    if handle.handle_type != "shared_pinned_cpu":
        raise WorkerDataPlaneResourceError("worker CPU handle must be a shared_pinned_cpu buffer")
    return BufferRegistration(buffer_id=handle.buffer_id, job_id=handle.job_id, kind=handle.kind,
                              size_bytes=handle.size_bytes, device_index=handle.device_index,
                              address=handle.address, pinned=handle.pinned, handle_type=handle.handle_type,
                              metadata=dict(handle.metadata))


__all__ = ["WorkerDataPlaneResourceBinder", "WorkerDataPlaneResourceBinding", "WorkerDataPlaneResourceError",
           "WorkerDataPlaneResources"]
