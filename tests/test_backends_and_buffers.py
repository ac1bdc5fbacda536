"""Shared pinned CPU buffers, CUDA IPC buffer descriptors, the CUDA backend
facade over a stand-in native module, and the CUDA worker executor over a
stand-in engine: argument checks, attach/close/unlink, registration
metadata, plan scoping and result mapping.  Behaviours follow
unit/test_client_shared_buffer.py, unit/test_backend_cuda.py and
unit/test_worker_cuda_executor.py of the reference with independent fakes."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from pcie_pool_b200.backends.cuda import CudaNativeBackend, coerce_ipc_handle
from pcie_pool_b200.client import CudaIpcDeviceBuffer, SharedPinnedCpuBuffer
from pcie_pool_b200.schema import BufferRegistration

MiB = 1 << 20


class FakeNative:
    def __init__(self):
        self.registered, self.opened, self.devices = {}, [], []

    def host_register(self, ptr, n):
        self.registered[ptr] = n

    def host_unregister(self, ptr):
        self.registered.pop(ptr)

    def export_ipc_handle(self, ptr):
        return bytes([ptr % 251]) * 64

    def allocation_base(self, ptr):
        return ptr - ptr % 4096

    def open_ipc_handle(self, handle, device):
        self.opened.append((handle, device))
        return 0 if handle[0] == 0 else 1 << 30

    def close_ipc_handle(self, ptr):
        self.opened.append(("close", ptr))

    def set_device(self, d):
        self.devices.append(d)


@pytest.fixture
def be():
    fake = FakeNative()
    b = CudaNativeBackend(native_loader=lambda: fake)
    b.fake = fake
    return b


# ---- shared pinned CPU buffers ---------------------------------------------------------------------

def test_shared_buffer_write_read_and_bounds():
    with SharedPinnedCpuBuffer.allocate("b", "j", 4096, name_prefix="ppbtest") as buf:
        buf.write(b"abc", offset=10)
        assert buf.read(3, offset=10) == b"abc" and bytes(buf.numpy()[10:13]) == b"abc"
        for bad in (lambda: buf.write(b"x", offset=-1), lambda: buf.write(b"x" * 10, offset=4090),
                    lambda: buf.read(10, offset=4090), lambda: buf.read(-1)):
            with pytest.raises(ValueError):
                bad()
        assert buf.owner and buf.address > 0
    with pytest.raises(ValueError, match="positive"):
        SharedPinnedCpuBuffer.allocate("b", "j", 0)


def test_attach_from_registration_shares_bytes_and_checks_backing():
    owner = SharedPinnedCpuBuffer.allocate("b", "j", 8192, name_prefix="ppbtest")
    try:
        owner.write(b"\x07" * 16, offset=100)
        reg = owner.buffer_registration()
        assert reg.handle_type == "shared_pinned_cpu" and reg.metadata["shared_memory_size_bytes"] == 8192
        peer = SharedPinnedCpuBuffer.open_from_registration(reg)
        try:
            assert not peer.owner and peer.read(16, offset=100) == b"\x07" * 16
            peer.write(b"\x09", offset=0)
            assert owner.read(1) == b"\x09"
        finally:
            peer.close()
        assert peer.closed and owner.read(1) == b"\x09", "closing a borrower leaves the owner usable"
        big = BufferRegistration("b", "j", "cpu_pinned", 8192, pinned=True, handle_type="shared_pinned_cpu",
                                 metadata={**reg.metadata, "offset_bytes": 4096, "shared_memory_size_bytes": 16384})
        with pytest.raises(ValueError, match="backing"):
            SharedPinnedCpuBuffer.open_from_registration(big)
        with pytest.raises(ValueError, match="shared_pinned_cpu"):
            SharedPinnedCpuBuffer.open_from_registration(
                BufferRegistration("g", "j", "gpu", 10, device_index=0))
    finally:
        owner.release()


def test_cuda_registration_is_idempotent_and_undone_on_close(be):
    buf = SharedPinnedCpuBuffer.allocate("b", "j", 4096, name_prefix="ppbtest")
    buf.register_for_cuda(be)
    buf.register_for_cuda(be)
    assert be.fake.registered == {buf.address: 4096} and buf.cuda_registered
    buf.release()
    assert be.fake.registered == {} and buf.closed
    with pytest.raises(RuntimeError, match="closed"):
        buf.view


# ---- CUDA IPC descriptors ----------------------------------------------------------------------------

def test_ipc_buffer_descriptor(be):
    d = CudaIpcDeviceBuffer.from_device_pointer("g", "j", 2, MiB, 0x10000 + 256, backend=be)
    assert be.fake.devices == [2] and d.ipc_offset == 256 and len(d.cuda_ipc_handle) == 64
    reg = d.buffer_registration()
    assert reg.handle_type == "cuda_ipc_device" and reg.metadata["cuda_ipc_offset"] == 256
    assert reg.device_index == 2 and reg.address == 0x10000 + 256
    base = CudaIpcDeviceBuffer.from_device_pointer("g", "j", 0, MiB, 0x20000, backend=be)
    assert "cuda_ipc_offset" not in base.metadata, "a buffer at its allocation base carries no offset"
    for kw in ({"size_bytes": 0, "device_ptr": 1}, {"size_bytes": 1, "device_ptr": 0}):
        with pytest.raises(ValueError):
            CudaIpcDeviceBuffer.from_device_pointer("g", "j", 0, backend=be, **kw)


# ---- backend facade ------------------------------------------------------------------------------------

def test_backend_argument_checks_and_ipc(be):
    with pytest.raises(ValueError):
        be.register_host_memory(0, 10)
    with pytest.raises(ValueError):
        be.register_host_memory(4096, 0)
    with pytest.raises(ValueError):
        be.unregister_host_memory(0)
    h = be.export_device_ipc_handle(4097)
    assert len(h) == 64
    assert be.open_device_ipc_handle(h.hex(), 1) == 1 << 30
    with pytest.raises(RuntimeError, match="invalid CUDA IPC pointer"):
        be.open_device_ipc_handle(bytes(64))
    be.close_device_ipc_handle(1 << 30)
    assert be.fake.opened[-1] == ("close", 1 << 30)
    with pytest.raises(ValueError):
        be.close_device_ipc_handle(0)
    assert be.device_allocation_offset(4096 * 3 + 17) == 17
    with pytest.raises(ValueError, match="hex"):
        coerce_ipc_handle("not hex")
    with pytest.raises(ValueError, match="64 bytes"):
        coerce_ipc_handle("ab" * 10)


def test_backend_runtime_delegation(be):
    bare = SimpleNamespace()
    for call in (lambda: be.initialize_runtime(bare, 0, [1]), lambda: be.fetch_plan_to_gpu(bare, 1, 1, 1, 1, {}),
                 lambda: be.offload_plan_to_cpu(bare, 1, 1, 1, 1, {}), lambda: be.wait(bare, 0),
                 lambda: be.stats(bare, 0)):
        with pytest.raises(RuntimeError, match="runtime does not support"):
            call()
    calls = []
    rt = SimpleNamespace(init=lambda t, r: calls.append(("init", t, r)),
                         fetch_plan_to_gpu=lambda *a: calls.append(("fetch",) + a) or 7,
                         wait=lambda h: calls.append(("wait", h)), stats=lambda h: {"bytes": 3})
    be.initialize_runtime(rt, 0, (1, 2))
    assert be.fetch_plan_to_gpu(rt, 1, 2, 3, 4, "p") == 7
    be.wait(rt, 7)
    assert be.stats(rt, 7) == {"bytes": 3}
    assert calls[0] == ("init", 0, [1, 2]) and calls[-1] == ("wait", 7)
    assert be.make_ranges([{"src_offset": 0, "dst_offset": 0, "bytes": 8}], 8, 8)
    with pytest.raises(ValueError):
        be.make_ranges([{"src_offset": 4, "dst_offset": 0, "bytes": 8}], 8, 8)
    assert be.transfer_mode_value("pool").value == "pool"


# ---- CUDA worker executor over a stand-in engine --------------------------------------------------------

class FakeEngine:
    def __init__(self, devices, fail=None, raise_=None):
        self.devices, self.fail, self.raise_, self.runs = devices, fail, raise_, []

    def run(self, direction, target, host_ptr, host_bytes, dev_ptr, dev_bytes, lanes, checksum=False):
        if self.raise_:
            raise RuntimeError(self.raise_)
        self.runs.append((direction, target, [(l.device, list(l.bytes)) for l in lanes], checksum))
        lane_stats = [SimpleNamespace(device=l.device, direct=l.device == target, bytes=int(sum(l.bytes)),
                                      chunks=len(l.bytes), cuda_ms=1.0) for l in lanes]
        return SimpleNamespace(ok=self.fail is None, error=self.fail, bytes=sum(s.bytes for s in lane_stats),
                               lanes=lane_stats, cuda_ms=1.0, gb_per_s=1.0)


def _worker_request(mode="pool"):
    from test_worker_lifecycle import Rig

    rig = Rig()
    req, _p = rig.authorization(mode=mode)
    return rig, rig.client.authorize(req)


def test_scoped_plan_keeps_only_authorized_relays():
    from pcie_pool_b200.worker.cuda_executor import scoped_plan

    rig, wr = _worker_request()
    try:
        plan = scoped_plan(wr, 0)
        kinds = sorted({a["path"]["kind"] for a in plan["assignments"]})
        assert "relay" in kinds
        relays = {a["path"]["relay_device"] for a in plan["assignments"] if a["path"]["kind"] == "relay"}
        assert relays <= set(wr.relay_gpus)
        with pytest.raises(ValueError, match="target"):
            scoped_plan(wr, 3)
    finally:
        rig.close()


def test_cuda_executor_maps_engine_results():
    from pcie_pool_b200.worker.cuda_executor import CudaWorkerExecutor
    from pcie_pool_b200.worker.helper import WorkerTransferState

    rig, wr = _worker_request()
    engines = []

    def factory(devs):
        e = FakeEngine(devs)
        engines.append(e)
        return e

    try:
        ex = CudaWorkerExecutor(engine_factory=factory)
        slot = rig.pool.allocate(wr.data_plane)
        with rig.client.resource_binder.bind(wr.data_plane) as res:
            r = ex.execute_bound(wr, slot, res)
            r2 = ex.execute_bound(wr, slot, res)
        assert len(engines) == 1, "one engine per device set, reused"
        assert r.state is WorkerTransferState.COMPLETE and r.bytes_completed == r2.bytes_completed
        md = r.metadata
        assert md["executor"] == "cuda_worker" and md["relay_bytes"] > 0
        assert md["direct_bytes"] + md["relay_bytes"] == r.bytes_completed
        direction, target, lanes, checksum = engines[0].runs[0]
        assert target == 0 and checksum and {d for d, _ in lanes} - {0} <= set(wr.relay_gpus)
        bad = CudaWorkerExecutor(engine_factory=lambda d: FakeEngine(d, fail="lane kernel error"))
        with rig.client.resource_binder.bind(wr.data_plane) as res:
            f = bad.execute_bound(wr, slot, res)
        assert f.state is WorkerTransferState.FAILED and "lane kernel error" in f.error
        boom = CudaWorkerExecutor(engine_factory=lambda d: FakeEngine(d, raise_="no device"))
        with rig.client.resource_binder.bind(wr.data_plane) as res:
            f = boom.execute_bound(wr, slot, res)
        assert f.state is WorkerTransferState.FAILED and "no device" in f.error
        f = ex.execute(wr, slot)
        assert f.state is WorkerTransferState.FAILED and "bound data-plane resources" in f.error
    finally:
        rig.close()


def test_backend_names_missing_native_support_and_checks_handles_before_native_calls():
    opened = []
    partial = SimpleNamespace(export_ipc_handle=lambda p: b"\x01" * 10,
                              open_ipc_handle=lambda h, d: opened.append(h) or 4096)
    be = CudaNativeBackend(native_loader=lambda: partial)
    for call, what in ((lambda: be.register_host_memory(4096, 8), "host memory registration"),
                       (lambda: be.unregister_host_memory(4096), "host memory registration"),
                       (lambda: be.close_device_ipc_handle(4096), "CUDA IPC close"),
                       (lambda: be.device_allocation_offset(4096), "allocation lookup"),
                       (lambda: be.set_device(0), "device selection")):
        with pytest.raises(RuntimeError, match=f"does not support {what}"):
            call()
    with pytest.raises(ValueError, match="64 bytes"):
        be.export_device_ipc_handle(4096)  # the native side returned a malformed handle
    with pytest.raises(ValueError):
        be.open_device_ipc_handle("zz" * 64)
    assert opened == [], "a malformed handle never reaches the native open"
    assert be.open_device_ipc_handle(b"\x02" * 64) == 4096 and len(opened) == 1
    with pytest.raises(ValueError):
        be.set_device(-1)
