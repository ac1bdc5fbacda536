"""CUDA VMM shareable handles on a GPU: a buffer allocated with cuMemCreate
and exported as a POSIX descriptor is imported by a second process (the
descriptor passed over a socket with SCM_RIGHTS), which lands bytes into it
through the engine's landing kernel; the exporting process reads exactly
those bytes back.  The legacy IPC path is covered by tests/test_worker.py."""

import multiprocessing as mp
from multiprocessing import reduction

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N = (8 << 20) + 4096


def _child(conn, size, mapped):
    import numpy as np

    from pcie_pool_b200.client import CudaVmmDeviceBuffer
    from pcie_pool_b200.parallel.engine import H2D, PoolEngine, split_even
    from pcie_pool_b200.utils.host_memory import PinnedHostBuffer

    fd = reduction.recv_handle(conn)
    buf = CudaVmmDeviceBuffer.import_fd("v", "j", 0, size, fd, mapped)
    host = PinnedHostBuffer(size, fill=None)
    host.numpy()[:] = np.random.default_rng(7).integers(0, 256, size, dtype=np.uint8)
    eng = PoolEngine([0], slot_bytes=2 << 20, slots=3, timeout_s=10.0)
    r = eng.run(H2D, 0, host.ptr, size, buf.device_ptr, size, split_even(size, 2 << 20, [0]), checksum=True,
                stage_direct=True)
    conn.send((bool(r.ok), r.error))
    conn.recv()  # parent has read the bytes
    buf.release()
    host.release()


def test_vmm_buffer_imported_in_a_second_process_receives_landed_bytes(need_gpu):
    from pcie_pool_b200._native import native
    from pcie_pool_b200.client import CudaVmmDeviceBuffer

    buf = CudaVmmDeviceBuffer.allocate("v", "j", 0, N)
    try:
        assert buf.mapped_bytes >= N and buf.mapped_bytes % native().vmm_granularity(0) == 0
        ctx = mp.get_context("spawn")
        parent, child = ctx.Pipe()
        p = ctx.Process(target=_child, args=(child, N, buf.mapped_bytes))
        p.start()
        reduction.send_handle(parent, buf.fd, p.pid)
        ok, err = parent.recv()
        assert ok, err
        got = np.empty(N, dtype=np.uint8)
        native().memcpy(got.ctypes.data, buf.device_ptr, N)
        want = np.random.default_rng(7).integers(0, 256, N, dtype=np.uint8)
        assert np.array_equal(got, want)
        parent.send("done")
        p.join(60)
        assert p.exitcode == 0
    finally:
        buf.release()


def test_vmm_buffer_through_the_daemon_executor(need_gpu):
    """An in-process daemon executes an intent into a VMM buffer it knows
    only by its exported descriptor."""
    import torch

    from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
    from pcie_pool_b200._native import native
    from pcie_pool_b200.client import CudaVmmDeviceBuffer
    from pcie_pool_b200.e2e import build_inprocess_node
    from pcie_pool_b200.parallel.engine import PoolEngine

    eng = PoolEngine([0], slot_bytes=2 << 20, slots=3, timeout_s=10.0)
    _daemon, dc = build_inprocess_node(eng, [0], 0, None)
    sid = dc.register_session(0, [], max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job("j", session_id=sid).ok
    buf = CudaVmmDeviceBuffer.allocate("v", "j", 0, N)
    host = torch.randint(0, 256, (N,), dtype=torch.uint8).pin_memory()
    try:
        assert dc.register_buffer("h", "j", "cpu_pinned", N, address=host.data_ptr(), pinned=True).ok
        assert buf.register_with_daemon(dc).ok
        it = TransferIntent("vmm-1", "j", sid, "h", "v", "h2d", N, ({"src_offset": 0, "dst_offset": 0, "bytes": N},),
                            metadata={"chunk_bytes": 2 << 20})
        r = TurboBusClient(daemon=dc).transfer(it, timeout_seconds=60)
        assert r.state is TransferStatusState.COMPLETE, r.error
        got = np.empty(N, dtype=np.uint8)
        native().memcpy(got.ctypes.data, buf.device_ptr, N)
        assert np.array_equal(got, host.numpy())
    finally:
        buf.release()
