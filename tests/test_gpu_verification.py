"""Live worker-managed verification on GPUs: daemon and worker helper run as
separate processes, bytes cross a real CUDA IPC mapping."""

import pytest

from pcie_pool_b200.verification import verify


@pytest.mark.gpu
def test_verify_direct_h2d_and_d2h(need_gpu):
    r = verify("h2d", mode="direct", bytes_to_copy=3 << 20, chunk_bytes=1 << 20, src_offset=4096,
               dst_offset=512, source_buffer_bytes=4 << 20, destination_buffer_bytes=4 << 20)
    assert r.state == "complete" and r.worker_path == "direct_h2d" and r.worker_relay_bytes == 0
    assert r.daemon_reservations_released
    r = verify("d2h", mode="direct", bytes_to_copy=3 << 20, chunk_bytes=1 << 20)
    assert r.state == "complete" and r.bytes_completed == 3 << 20


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("direction,mode", [("h2d", "relay"), ("d2h", "relay"), ("h2d", "pool")])
def test_verify_worker_relay(need_two_gpus, direction, mode):
    r = verify(direction, mode=mode, bytes_to_copy=24 << 20, chunk_bytes=2 << 20, max_inflight_chunks=64)
    assert r.state == "complete" and r.worker_final_state == "complete"
    assert r.worker_relay_bytes > 0 and r.worker_relay_bytes + r.worker_direct_bytes == 24 << 20
    assert r.daemon_reservations_released and r.daemon_relay_active_chunks == 0
