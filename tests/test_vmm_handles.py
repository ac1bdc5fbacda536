"""CUDA VMM shareable handles: the descriptor plumbing on the CPU.

A ``cuda_vmm_fd`` buffer registration carries its exported POSIX
descriptor beside the request (SCM_RIGHTS over the daemon socket, the
number itself for an in-process daemon); the daemon keeps a duplicate for as
long as the buffer is registered and closes it on cleanup.  An ordinary file
descriptor stands in for the CUDA export here -- the daemon never looks
inside it until an executor imports it (tests/test_gpu_vmm.py does that on a
GPU)."""

from __future__ import annotations

import os
import tempfile
import threading
import time

import pytest

from pcie_pool_b200.daemon import InProcessDaemonClient, TurboBusDaemon
from pcie_pool_b200.daemon.client import TurboBusDaemonClient
from pcie_pool_b200.daemon.wire import serve_unix
from pcie_pool_b200.schema import BufferRegistration
from pcie_pool_b200.topology import StaticTopologyProvider


@pytest.fixture
def served(tmp_path):
    d = TurboBusDaemon(relay_gpus=[1], topology_provider=StaticTopologyProvider(gpu_count=2))
    path = str(tmp_path / "d.sock")
    stop, ready = threading.Event(), threading.Event()
    t = threading.Thread(target=serve_unix, args=(d, path), kwargs={"stop_event": stop, "ready_event": ready},
                         daemon=True)
    t.start()
    assert ready.wait(5)
    yield d, path
    stop.set()
    t.join(5)


def _file():
    fh = tempfile.TemporaryFile()
    fh.write(b"stand-in for a CUDA VMM export")
    fh.flush()
    return fh


def _job(dc):
    sid = dc.register_session(0, [1]).payload["session"]["session_id"]
    assert dc.register_job("j", session_id=sid).ok


def test_descriptor_travels_with_the_registration_over_the_socket(served):
    d, path = served
    dc = TurboBusDaemonClient(path, persistent=True)
    _job(dc)
    fh = _file()
    r = dc.register_buffer("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 1 << 21}, fds=[fh.fileno()])
    assert r.ok, r.error
    mine = d._st.buffer_fds["v"]
    assert mine != fh.fileno(), "the daemon holds its own duplicate"
    assert os.fstat(mine).st_ino == os.fstat(fh.fileno()).st_ino
    assert d._st.buffers["v"].metadata["vmm_fd"] == mine
    # the client may close its copy; the daemon's stays valid until cleanup
    fh.close()
    assert os.fstat(mine).st_size > 0
    assert dc.cleanup("buffer", "v", "done").ok
    assert "v" not in d._st.buffer_fds
    with pytest.raises(OSError):
        os.fstat(mine)
    dc.close()


def test_descriptor_numbers_in_json_are_refused_over_the_socket(served):
    _d, path = served
    dc = TurboBusDaemonClient(path)
    _job(dc)
    r = dc.register_buffer("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 1 << 21, "vmm_fd": 0})
    assert not r.ok and "attach the descriptor" in r.error
    r = dc.register_buffer("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 1 << 21})
    assert not r.ok and "descriptor attached" in r.error


def test_in_process_registration_duplicates_the_callers_descriptor():
    d = TurboBusDaemon(relay_gpus=[1], topology_provider=StaticTopologyProvider(gpu_count=2))
    dc = InProcessDaemonClient(d)
    _job(dc)
    fh = _file()
    r = dc.register_buffer("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 1 << 21}, fds=[fh.fileno()])
    assert r.ok, r.error
    mine = d._st.buffer_fds["v"]
    assert mine != fh.fileno() and os.fstat(mine).st_ino == os.fstat(fh.fileno()).st_ino
    # re-registering replaces (and closes) the old duplicate
    r = dc.register_buffer("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 1 << 21}, fds=[fh.fileno()])
    assert r.ok, r.error
    new = d._st.buffer_fds["v"]
    assert new != mine and os.fstat(new).st_ino == os.fstat(fh.fileno()).st_ino
    with pytest.raises(OSError):
        os.fstat(mine)
    fh.close()


def test_schema_rules_for_vmm_registrations():
    with pytest.raises(ValueError, match="vmm_mapped_bytes"):
        BufferRegistration("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 1024})
    with pytest.raises(ValueError, match="device_index"):
        BufferRegistration("v", "j", "gpu", 4096, handle_type="cuda_vmm_fd", metadata={"vmm_mapped_bytes": 4096})
    with pytest.raises(ValueError, match="descriptor"):
        BufferRegistration("v", "j", "gpu", 4096, device_index=0, handle_type="cuda_vmm_fd",
                           metadata={"vmm_mapped_bytes": 4096, "vmm_fd": -3})
