"""Fused landing ops driven through the daemon (CPU, mock data plane).

A paged-KV prefix is saved with the fused gather and restored into a
permuted block table with the fused scatter, each as ONE intent under the
daemon's plan and relay leases; an fp8 landing intent quantises bf16
matrices to e4m3 + per-128x128 scales.  The mock data plane applies the same
addressing rules as the GPU kernels, so these tests pin the control path:
spec validation, ownership and bounds checks, chunk-to-unit / chunk-to-row
mapping, lease release.  The same intents run on the GPU in
tests/test_gpu_daemon_landing.py."""

import numpy as np
import pytest
import torch

from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
from pcie_pool_b200.adapters.kv_offload import DaemonKVOffloader
from pcie_pool_b200.daemon import InProcessDaemonClient, IntentExecutor, TurboBusDaemon
from pcie_pool_b200.daemon.landing import LandingSpec, kv_spec
from pcie_pool_b200.mock import MockDataPlane, MockWorld
from pcie_pool_b200.topology import StaticTopologyProvider
from pcie_pool_b200.utils.fp8 import block_quant

LAYERS, BLOCKS, BS, HEADS, DIM = 4, 64, 16, 2, 16  # unit = 16*2*16*2 = 1 KiB


def node(gpus=4):
    world = MockWorld(gpu_count=gpus)
    plane = MockDataPlane(world, checksum=False)
    daemon = TurboBusDaemon(relay_gpus=range(1, gpus), max_inflight_chunks_per_relay=4096,
                            topology_provider=StaticTopologyProvider(gpu_count=gpus), executor=IntentExecutor(plane))
    daemon.put_profile(0, list(range(1, gpus)), world.profile(0))
    dc = InProcessDaemonClient(daemon)
    sid = dc.register_session(0, list(range(1, gpus)), max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job("job", session_id=sid).ok
    return daemon, dc, sid, plane


def kv_caches(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(2, BLOCKS, BS, HEADS, DIM, generator=g).to(torch.bfloat16) for _ in range(LAYERS)]


def test_kv_save_then_restore_into_permuted_blocks_through_the_daemon():
    daemon, dc, sid, plane = node()
    kvs = kv_caches(1)
    off = DaemonKVOffloader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="job", kv_caches=kvs,
                            units_per_chunk=4, sync_stream=False)
    src_ids = [int(x) for x in torch.randperm(BLOCKS, generator=torch.Generator().manual_seed(2))[:24]]
    host = torch.zeros(off.prefix_bytes(len(src_ids)), dtype=torch.uint8)
    st = off.save(src_ids, host)
    assert st.bytes == host.numel() and st.units == LAYERS * 2 * len(src_ids)
    # host layout: [layer][lane][index]
    want = torch.cat([kv[lane, src_ids].reshape(-1).view(torch.uint8) for kv in kvs for lane in range(2)])
    assert torch.equal(host, want)
    # restore into a different (permuted) block table of fresh caches
    dst_ids = [int(x) for x in torch.randperm(BLOCKS, generator=torch.Generator().manual_seed(3))[:24]]
    for kv in kvs:
        kv.zero_()
    off.restore(dst_ids, host)
    for kv, kv0 in zip(kvs, kv_caches(1)):
        assert torch.equal(kv[:, dst_ids], kv0[:, src_ids])
        untouched = sorted(set(range(BLOCKS)) - set(dst_ids))
        assert int(kv[:, untouched].view(torch.int16).abs().sum()) == 0
    # every intent used the relay lanes, and released every lease
    lanes = {t["lane"] for t in plane.trace}
    assert lanes >= {0, 1, 2, 3}
    d = dc.describe().payload
    assert not d.get("reservations")
    assert all(int(q.get("active_chunks", 0)) == 0 for q in (d.get("relay_quotas") or {}).values())
    assert not (d.get("runtime_resource_state") or {}).get("active_paths")


def test_restore_of_a_shorter_request_from_a_longer_saved_span():
    daemon, dc, sid, _ = node()
    kvs = kv_caches(4)
    off = DaemonKVOffloader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="job", kv_caches=kvs,
                            units_per_chunk=8, sync_stream=False)
    ids = list(range(10, 30))
    host = torch.zeros(off.prefix_bytes(len(ids)), dtype=torch.uint8)
    off.save(ids, host)
    ref = [kv.clone() for kv in kvs]
    for kv in kvs:
        kv.zero_()
    off.restore(ids[:7], host, span_blocks=len(ids))
    for kv, r in zip(kvs, ref):
        assert torch.equal(kv[:, ids[:7]], r[:, ids[:7]])


def _fp8_job(dc, sid, mats, pad=0):
    """Host image of bf16 matrices + one device buffer for codes and scales."""
    host_parts, table, q_off, s_total = [], [], 0, 0
    h = 0
    for m in mats:
        host_parts.append(m.contiguous().view(torch.uint8).reshape(-1))
        table.append((h, m.shape[0], m.shape[1]))
        h += m.numel() * 2
    host = torch.cat(host_parts)
    tensors, q_off = [], 0
    for hoff, r, c in table:
        tensors.append({"host_offset": hoff, "rows": r, "cols": c, "q_offset": q_off, "scales_offset": 0})
        q_off += r * c
    s_off = -(-q_off // 16) * 16
    for t in tensors:
        t["scales_offset"] = s_off
        s_off += -(-t["rows"] // 128) * (t["cols"] // 128) * 4
    dev = torch.zeros(s_off + pad, dtype=torch.uint8)
    assert dc.register_buffer("w-host", "job", "cpu_pinned", host.numel(), address=host.data_ptr(), pinned=True).ok
    assert dc.register_buffer("w-dev", "job", "gpu", dev.numel(), device_index=0, address=dev.data_ptr()).ok
    return host, dev, tensors


def _fp8_ranges(tensors, chunk):
    out = []
    for t in tensors:
        rb, rows = 2 * t["cols"], t["rows"]
        step = max(1, chunk // (128 * rb)) * 128
        for r in range(0, rows, step):
            n = min(step, rows - r) * rb
            out.append({"src_offset": t["host_offset"] + r * rb, "dst_offset": t["host_offset"] + r * rb, "bytes": n})
    return tuple(out)


def test_fp8_landing_intent_matches_the_ocp_oracle():
    daemon, dc, sid, _ = node()
    g = torch.Generator().manual_seed(7)
    mats = [(torch.randn(384, 256, generator=g) * 0.02).to(torch.bfloat16),
            (torch.randn(200, 128, generator=g) * 3).to(torch.bfloat16)]
    host, dev, tensors = _fp8_job(dc, sid, mats)
    chunk = 128 * 512
    ranges = _fp8_ranges(tensors, chunk)
    spec = {"op": "fp8_quant", "tensors": tensors}
    it = TransferIntent("fp8-1", "job", sid, "w-host", "w-dev", "h2d", sum(r["bytes"] for r in ranges), ranges,
                        workload_kind="model_weights", metadata={"chunk_bytes": chunk, "landing": spec})
    r = TurboBusClient(daemon=dc).transfer(it, timeout_seconds=60)
    assert r.state is TransferStatusState.COMPLETE, r.error
    for m, t in zip(mats, tensors):
        q, sc = block_quant(m.float().numpy())
        got_q = dev[t["q_offset"]:t["q_offset"] + m.numel()].numpy().reshape(m.shape)
        ns = sc.size * 4
        got_s = dev[t["scales_offset"]:t["scales_offset"] + ns].numpy().view(np.float32).reshape(sc.shape)
        assert np.array_equal(got_q, q)
        assert np.array_equal(got_s, sc)


@pytest.mark.parametrize("mutate,msg", [
    (lambda s: s["kv"].update(block_ids=[0, BLOCKS]), "block id outside"),
    (lambda s: s.update(op="gather_units"), "d2h only"),
    (lambda s: s.update(unit_bytes=8), "multiple of 16"),
    (lambda s: s["kv"].update(buffers=["kv-layer0", "nope"]), "not registered"),
    (lambda s: s["kv"].update(block_stride=BS * HEADS * DIM * 2 * 4), "exceeds buffer"),
    (lambda s: s.update(op="transpose"), "landing op must be one of"),
], ids=["block-range", "direction", "unit-align", "unregistered", "extent", "unknown-op"])
def test_unsafe_landing_specs_are_rejected_at_submit(mutate, msg):
    daemon, dc, sid, plane = node()
    kvs = kv_caches(9)
    for i, kv in enumerate(kvs):
        assert dc.register_buffer(f"kv-layer{i}", "job", "gpu", kv.numel() * 2, device_index=0,
                                  address=kv.data_ptr()).ok
    host = torch.zeros(LAYERS * 2 * 4 * 1024, dtype=torch.uint8)
    assert dc.register_buffer("h", "job", "cpu_pinned", host.numel(), address=host.data_ptr(), pinned=True).ok
    spec = kv_spec(kvs, [1, 2, 3, 4], [f"kv-layer{i}" for i in range(LAYERS)], op="scatter_units").to_metadata()
    mutate(spec)
    n = host.numel()
    it = TransferIntent("bad-1", "job", sid, "h", "kv-layer0", "h2d", n, ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                        metadata={"chunk_bytes": 4096, "landing": spec})
    resp = dc.submit_transfer_intent(it)
    assert not resp.ok and msg in (resp.error or "")
    assert not plane.trace


def test_kv_buffer_of_another_job_is_rejected():
    daemon, dc, sid, _ = node()
    assert dc.register_job("other", session_id=sid).ok
    kvs = kv_caches(11)
    assert dc.register_buffer("kv-layer0", "job", "gpu", kvs[0].numel() * 2, device_index=0,
                              address=kvs[0].data_ptr()).ok
    assert dc.register_buffer("kv-layer1", "other", "gpu", kvs[1].numel() * 2, device_index=0,
                              address=kvs[1].data_ptr()).ok
    host = torch.zeros(2 * 2 * 2 * 1024, dtype=torch.uint8)
    assert dc.register_buffer("h", "job", "cpu_pinned", host.numel(), address=host.data_ptr(), pinned=True).ok
    spec = kv_spec(kvs[:2], [1, 2], ["kv-layer0", "kv-layer1"], op="scatter_units").to_metadata()
    n = host.numel()
    it = TransferIntent("x-1", "job", sid, "h", "kv-layer0", "h2d", n, ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                        metadata={"chunk_bytes": 4096, "landing": spec})
    resp = dc.submit_transfer_intent(it)
    assert not resp.ok and "another job" in resp.error


def test_landing_spec_round_trips_through_its_wire_form():
    kvs = kv_caches(12)
    spec = kv_spec(kvs, [5, 3, 9], ["a", "b", "c", "d"], op="gather_units", ctas_per_lane=6)
    back = LandingSpec.from_metadata({"landing": spec.to_metadata()})
    assert back == spec and back.kv.units == 4 * 2 * 3
