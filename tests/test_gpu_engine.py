"""GPU tests of the native data plane (PoolEngine + lane kernels).

Every device result is compared with a host oracle: byte equality for copies,
scatters and gathers; the numpy checksum for per-chunk checksums; the OCP-spec
e4m3 oracle (bit-exact) for fp8 landing.  Single-GPU tests route the direct
lane through the landing ring (``stage_direct``) so the staged kernel path is
exercised without a peer; relay tests need two GPUs.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _engine(devices, **kw):
    from pcie_pool_b200.parallel.engine import PoolEngine

    kw.setdefault("slot_bytes", 1 << 20)
    kw.setdefault("slots", 3)
    kw.setdefault("timeout_s", 5.0)
    return PoolEngine(devices, **kw)


def _host(nbytes, seed=0):
    from pcie_pool_b200.utils.host_memory import PinnedHostBuffer

    buf = PinnedHostBuffer(nbytes)
    rng = np.random.default_rng(seed)
    buf.numpy()[:] = rng.integers(0, 256, size=nbytes, dtype=np.uint8)
    return buf


def _chunk_sums(data: np.ndarray, lanes):
    from pcie_pool_b200.utils.checksum import checksum_bytes

    out = []
    for lane in lanes:
        for s, b in zip(lane.src_off, lane.bytes):
            out.append(checksum_bytes(data[int(s):int(s) + int(b)]))
    return np.array(out, dtype=np.uint64)


@pytest.mark.parametrize("checksum", [False, True])
def test_direct_h2d_copy_exact(need_gpu, checksum):
    from pcie_pool_b200.parallel.engine import H2D, split_even

    n = (5 << 20) + 4096 + 12
    host = _host(n)
    dev = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    eng = _engine([0])
    lanes = split_even(n, 1 << 20, [0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, n, dev.data_ptr(), n, lanes, checksum=checksum)
    assert r.ok, r.error
    assert torch.equal(dev.cpu(), torch.from_numpy(host.numpy().copy()))
    if checksum:
        assert np.array_equal(r.checksums, _chunk_sums(host.numpy(), lanes))
    assert r.cuda_ms > 0


@pytest.mark.parametrize("total", [(3 << 20) + 9, 1 << 20, 7777])
def test_staged_h2d_ragged_exact(need_gpu, total):
    from pcie_pool_b200.parallel.engine import H2D, split_even

    host = _host(total, seed=1)
    dev = torch.zeros(total, dtype=torch.uint8, device="cuda:0")
    eng = _engine([0])
    lanes = split_even(total, 1 << 20, [0])
    for _ in range(3):  # ring reuse across transfers
        dev.zero_()
        torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
        r = eng.run(H2D, 0, host.ptr, total, dev.data_ptr(), total, lanes, checksum=True,
                    stage_direct=True)
        assert r.ok, r.error
        assert torch.equal(dev.cpu(), torch.from_numpy(host.numpy().copy()))
        assert np.array_equal(r.checksums, _chunk_sums(host.numpy(), lanes))


def test_misaligned_destination(need_gpu):
    from pcie_pool_b200.parallel.engine import H2D, make_lane

    total = 200000
    host = _host(total, seed=2)
    dev = torch.zeros(total + 64, dtype=torch.uint8, device="cuda:0")
    eng = _engine([0])
    lane = make_lane(0, [(0, 3, 100000), (100000, 100003, 100000)])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, total, dev.data_ptr(), total + 64, [lane], checksum=True,
                stage_direct=True)
    assert r.ok, r.error
    got = dev.cpu().numpy()
    assert np.array_equal(got[3:3 + total], host.numpy())
    assert np.array_equal(r.checksums, _chunk_sums(host.numpy(), [lane]))


@pytest.mark.parametrize("stage", [False, True])
def test_d2h_copy_exact(need_gpu, stage):
    from pcie_pool_b200.parallel.engine import D2H, split_even

    n = (4 << 20) + 48
    host = _host(n, seed=3)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda:0")
    eng = _engine([0])
    lanes = split_even(n, 1 << 20, [0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(D2H, 0, host.ptr, n, src.data_ptr(), n, lanes, checksum=True, stage_direct=stage)
    assert r.ok, r.error
    ref = src.cpu().numpy()
    assert np.array_equal(host.numpy(), ref)
    assert np.array_equal(r.checksums, _chunk_sums(ref, lanes))


def _kv_setup(num_blocks=48, unit=32768, seed=4):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).numpy()
    kv = torch.zeros(num_blocks, unit, dtype=torch.uint8, device="cuda:0")
    addrs = (kv.data_ptr() + perm.astype(np.uint64) * np.uint64(unit)).astype(np.uint64)
    return kv, perm, addrs


def test_scatter_units_paged_kv(need_gpu):
    from pcie_pool_b200.parallel.engine import H2D, Lane

    C = pytest.importorskip("pcie_pool_b200._C")
    unit = 32768
    kv, perm, addrs = _kv_setup(unit=unit)
    n = kv.numel()
    host = _host(n, seed=5)
    per_chunk = 8  # units per chunk (256 KiB)
    starts = np.arange(0, perm.size, per_chunk)
    lane = Lane(0, (starts * unit).astype(np.uint64), np.zeros(starts.size, np.uint64),
                np.full(starts.size, per_chunk * unit, np.uint64), unit0=starts.astype(np.uint32))
    eng = _engine([0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, n, kv.data_ptr(), n, [lane], op=C.OP_SCATTER_UNITS,
                checksum=True, unit_bytes=unit, unit_addrs=addrs)
    assert r.ok, r.error
    got = kv.cpu().numpy()
    src = host.numpy().reshape(perm.size, unit)
    for i, b in enumerate(perm):
        assert np.array_equal(got[b], src[i])
    assert np.array_equal(r.checksums, _chunk_sums(host.numpy(), [lane]))


def test_gather_units_paged_kv(need_gpu):
    from pcie_pool_b200.parallel.engine import D2H, Lane

    C = pytest.importorskip("pcie_pool_b200._C")
    unit = 32768
    kv, perm, addrs = _kv_setup(unit=unit, seed=6)
    kv.copy_(torch.randint(0, 256, kv.shape, dtype=torch.uint8, device="cuda:0"))
    n = kv.numel()
    host = _host(n, seed=7)
    per_chunk = 4
    starts = np.arange(0, perm.size, per_chunk)
    lane = Lane(0, np.zeros(starts.size, np.uint64), (starts * unit).astype(np.uint64),
                np.full(starts.size, per_chunk * unit, np.uint64), unit0=starts.astype(np.uint32))
    eng = _engine([0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(D2H, 0, host.ptr, n, kv.data_ptr(), n, [lane], op=C.OP_GATHER_UNITS,
                checksum=True, unit_bytes=unit, unit_addrs=addrs)
    assert r.ok, r.error
    kvh = kv.cpu().numpy()
    expect = np.concatenate([kvh[b] for b in perm])
    assert np.array_equal(host.numpy(), expect)


def test_fp8_landing_bit_exact(need_gpu):
    from pcie_pool_b200.parallel.engine import H2D, Lane
    from pcie_pool_b200.utils.fp8 import block_quant

    C = pytest.importorskip("pcie_pool_b200._C")
    rows, cols = 300, 384
    w = (torch.randn(rows, cols, generator=torch.Generator().manual_seed(8)) * 0.02).to(torch.bfloat16)
    raw = w.view(torch.uint8).numpy().reshape(-1)
    host = _host(raw.size)
    host.numpy()[:] = raw
    q = torch.zeros(rows, cols, dtype=torch.uint8, device="cuda:0")
    scales = torch.zeros((rows + 127) // 128, cols // 128, dtype=torch.float32, device="cuda:0")
    row_bytes = cols * 2
    r0 = np.array([0, 128, 256], dtype=np.uint32)
    nrows = np.minimum(128, rows - r0)
    lane = Lane(0, (r0.astype(np.uint64) * row_bytes), np.zeros(3, np.uint64),
                (nrows * row_bytes).astype(np.uint64), unit0=r0, tensor=np.zeros(3, np.uint32))
    eng = _engine([0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, raw.size, q.data_ptr(), q.numel(), [lane], op=C.OP_FP8_QUANT,
                checksum=True, tensors=[(q.data_ptr(), scales.data_ptr(), rows, cols)])
    assert r.ok, r.error
    q_ref, s_ref = block_quant(w.float().numpy())
    assert np.array_equal(scales.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


def test_ranges_unpack_and_pack(need_gpu):
    from pcie_pool_b200.parallel.engine import D2H, H2D, Lane

    C = pytest.importorskip("pcie_pool_b200._C")
    rng = np.random.default_rng(9)
    sizes = (rng.integers(1, 2048, size=40) * 16).astype(np.uint32)  # <= 32 KiB each
    total = int(sizes.sum())
    # each range lands in its own shuffled 32 KiB slot (16-aligned start)
    dst = torch.zeros(40 * 32768, dtype=torch.uint8, device="cuda:0")
    slots = rng.permutation(40)
    offs = np.arange(40, dtype=np.int64) * 32768
    addrs = (dst.data_ptr() + offs[slots]).astype(np.uint64)
    # two chunks: first 25 ranges, then 15
    pos = np.zeros(40, np.uint64)
    bounds = [(0, 25), (25, 40)]
    src_off, cbytes = [], []
    running = 0
    for a, b in bounds:
        p = 0
        for i in range(a, b):
            pos[i] = p
            p += int(sizes[i])
        src_off.append(running)
        cbytes.append(p)
        running += p
    host = _host(total, seed=10)
    lane = Lane(0, np.array(src_off, np.uint64), np.zeros(2, np.uint64), np.array(cbytes, np.uint64),
                unit0=np.array([0, 25], np.uint32), count=np.array([25, 15], np.uint32))
    eng = _engine([0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, total, dst.data_ptr(), dst.numel(), [lane], op=C.OP_SCATTER_RANGES,
                checksum=True, ranges=(addrs, sizes, pos))
    assert r.ok, r.error
    got = dst.cpu().numpy()
    h = host.numpy()
    stream = 0
    for i in range(40):
        o = int(offs[slots[i]])
        assert np.array_equal(got[o:o + sizes[i]], h[stream:stream + sizes[i]])
        stream += int(sizes[i])
    # pack it back
    back = _host(total, seed=11)
    lane2 = Lane(0, np.zeros(2, np.uint64), np.array(src_off, np.uint64), np.array(cbytes, np.uint64),
                 unit0=np.array([0, 25], np.uint32), count=np.array([25, 15], np.uint32))
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r2 = eng.run(D2H, 0, back.ptr, total, dst.data_ptr(), dst.numel(), [lane2], op=C.OP_GATHER_RANGES,
                 checksum=True, ranges=(addrs, sizes, pos))
    assert r2.ok, r2.error
    assert np.array_equal(back.numpy(), h)


def test_lane_timeout_reports_status_and_recovers(need_gpu):
    """A lane whose producer never publishes: the landing kernel gives up after
    its bounded wait, reports the status, and the engine stays usable."""
    from pcie_pool_b200.parallel.engine import H2D, split_even

    n = 2 << 20
    host = _host(n, seed=12)
    dev = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    eng = _engine([0], timeout_s=0.5)
    lanes = split_even(n, 1 << 20, [0])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, n, dev.data_ptr(), n, lanes, stage_direct=True,
                debug_drop_publish=0)
    assert not r.ok
    assert r.status_code == 1
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r2 = eng.run(H2D, 0, host.ptr, n, dev.data_ptr(), n, lanes, stage_direct=True, checksum=True)
    assert r2.ok, r2.error
    assert torch.equal(dev.cpu(), torch.from_numpy(host.numpy().copy()))


# ---- multi-GPU: relay lanes over NVLink ---------------------------------------------

@pytest.mark.multigpu
def test_relay_h2d_and_d2h_exact(need_two_gpus):
    from pcie_pool_b200.parallel.engine import D2H, H2D, split_even

    ndev = min(torch.cuda.device_count(), 8)
    devs = list(range(ndev))
    n = (16 << 20) + 4096 + 4
    host = _host(n, seed=13)
    dev = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    eng = _engine(devs)
    lanes = split_even(n, 1 << 20, devs)
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, n, dev.data_ptr(), n, lanes, checksum=True)
    assert r.ok, r.error
    assert torch.equal(dev.cpu(), torch.from_numpy(host.numpy().copy()))
    assert np.array_equal(r.checksums, _chunk_sums(host.numpy(), lanes))
    back = _host(n, seed=14)
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r2 = eng.run(D2H, 0, back.ptr, n, dev.data_ptr(), n, lanes, checksum=True)
    assert r2.ok, r2.error
    assert np.array_equal(back.numpy(), host.numpy())


@pytest.mark.multigpu
def test_relay_scatter_units(need_two_gpus):
    from pcie_pool_b200.parallel.engine import H2D, Lane

    C = pytest.importorskip("pcie_pool_b200._C")
    unit = 32768
    kv, perm, addrs = _kv_setup(num_blocks=64, unit=unit, seed=15)
    n = kv.numel()
    host = _host(n, seed=16)
    starts = np.arange(0, 64, 8)
    lanes = []
    for li, dev in enumerate([0, 1]):
        sel = starts[li::2]
        lanes.append(Lane(dev, (sel * unit).astype(np.uint64), np.zeros(sel.size, np.uint64),
                          np.full(sel.size, 8 * unit, np.uint64), unit0=sel.astype(np.uint32)))
    eng = _engine([0, 1])
    torch.cuda.synchronize()  # torch's stream and the engine's streams are not ordered
    r = eng.run(H2D, 0, host.ptr, n, kv.data_ptr(), n, lanes, op=C.OP_SCATTER_UNITS,
                checksum=True, unit_bytes=unit, unit_addrs=addrs)
    assert r.ok, r.error
    got = kv.cpu().numpy()
    src = host.numpy().reshape(64, unit)
    for i, b in enumerate(perm):
        assert np.array_equal(got[b], src[i])


@pytest.mark.multigpu
def test_daemon_lane_failover_reruns_failed_relay(need_two_gpus):
    """A relay lane whose chunks are never published (the landing wait runs
    out after 1 s) is re-run over the direct lane; the intent completes and
    the bytes are exact."""
    from pcie_pool_b200 import TransferIntent, TransferStatusState, TurboBusClient
    from pcie_pool_b200.daemon import EngineDataPlane, InProcessDaemonClient, IntentExecutor, TurboBusDaemon
    from pcie_pool_b200.topology import StaticTopologyProvider, synthetic_inventory

    n = 64 << 20
    host = _host(n, seed=21)
    dev = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    plane = EngineDataPlane(engine=_engine([0, 1], slot_bytes=4 << 20), checksum=True)
    d = TurboBusDaemon([1], max_inflight_chunks_per_relay=4096,
                       topology_provider=StaticTopologyProvider(synthetic_inventory(2, source="declared")),
                       executor=IntentExecutor(plane))
    link = {"h2d_bw_gbps": 50.0, "d2h_bw_gbps": 50.0, "p2p_bw_gbps": 700.0, "effective_bw_gbps": 50.0,
            "effective_d2h_bw_gbps": 50.0, "p2p_enabled": True}
    d.put_profile(0, [1], {"target_device": 0, "direct_h2d_bw_gbps": 50.0, "direct_d2h_bw_gbps": 50.0,
                           "relays": [{"relay_device": 1, "target_device": 0, **link}]})
    dc = InProcessDaemonClient(d)
    sid = dc.register_session(0, [1], max_inflight_chunks=4096).payload["session"]["session_id"]
    dc.register_job("fo", session_id=sid)
    dc.register_buffer("h", "fo", "cpu_pinned", n, address=host.ptr, pinned=True)
    dc.register_buffer("g", "fo", "gpu", n, device_index=0, address=dev.data_ptr())
    plane.debug_drop_publish = 1  # the relay lane (spec lane 1) never publishes
    plane.failover_timeout_s = 1.0
    it = TransferIntent("fo-0", "fo", sid, "h", "g", "h2d", n, ({"src_offset": 0, "dst_offset": 0, "bytes": n},),
                        metadata={"chunk_bytes": 4 << 20})
    r = TurboBusClient(daemon=dc).transfer(it, timeout_seconds=120)
    assert r.state is TransferStatusState.COMPLETE, r.error
    assert torch.equal(dev.cpu(), torch.from_numpy(host.numpy()))
    meas = r.metadata.get("measured", {})
    assert meas.get("failover", {}).get("failed_lane_device") == 1
    host.release()


def test_device_trace_stamps_are_ordered(need_gpu):
    """trace=True records per-chunk %globaltimer stamps: wait begin <= ready
    <= done for every staged chunk, exported as Chrome-trace spans."""
    from pcie_pool_b200.parallel.engine import H2D, split_even
    from pcie_pool_b200.plan_trace import device_trace_events

    n = 24 << 20
    host = _host(n, seed=31)
    dev = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    lanes = split_even(n, 4 << 20, [0])
    r = _engine([0], slot_bytes=4 << 20).run(H2D, 0, host.ptr, n, dev.data_ptr(), n, lanes, checksum=True,
                                             stage_direct=True, trace=True)
    assert r.ok, r.error
    assert r.trace is not None and r.trace.shape == (6, 4)
    for a, b, c, ctas in r.trace.astype(np.int64):
        assert 0 < a <= b <= c and ctas >= 1
    ev = device_trace_events(r, lanes)
    assert len(ev) == 12 and {e["name"] for e in ev} == {"transfer:wait", "transfer:move"}
    host.release()


def test_h2d_and_d2h_on_one_target_run_concurrently(need_gpu):
    """A GPU's H2D and D2H transfers overlap on the full-duplex link: both in
    flight together take clearly less than one after the other."""
    import time

    from pcie_pool_b200.parallel.engine import D2H, H2D, split_even

    n = 1 << 30
    up = _host(n, seed=11)
    down = _host(n, seed=12)
    dst = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda:0")
    torch.cuda.synchronize()
    eng = _engine([0], slot_bytes=16 << 20)
    lanes = split_even(n, 16 << 20, [0])

    def both(serial: bool) -> float:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        a = eng.submit(H2D, 0, up.ptr, n, dst.data_ptr(), n, lanes)
        if serial:
            assert eng.wait(a).ok
        b = eng.submit(D2H, 0, down.ptr, n, src.data_ptr(), n, lanes)
        rb = eng.wait(b)
        if not serial:
            assert eng.wait(a).ok
        assert rb.ok, rb.error
        return time.perf_counter() - t0

    both(True)
    serial = min(both(True) for _ in range(2))
    duplex = min(both(False) for _ in range(2))
    assert torch.equal(dst[:1 << 20].cpu(), torch.from_numpy(up.numpy()[:1 << 20].copy()))
    assert np.array_equal(down.numpy()[-(1 << 20):], src[-(1 << 20):].cpu().numpy())
    assert duplex < 0.9 * serial, (duplex, serial)  # serial would be ~1.0; duplex measured well below


def test_overlapping_opposite_transfers_stay_ordered(need_gpu):
    """D2H of a device region into host memory followed at once by H2D of that
    host memory into another region: the H2D sees the D2H's bytes."""
    from pcie_pool_b200.parallel.engine import D2H, H2D, split_even

    n = 64 << 20
    host = _host(n, seed=13)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda:0")
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    eng = _engine([0], slot_bytes=4 << 20)
    lanes = split_even(n, 4 << 20, [0])
    for _ in range(3):
        src.random_(0, 256)
        torch.cuda.synchronize()  # the engine's streams do not wait for torch's stream
        a = eng.submit(D2H, 0, host.ptr, n, src.data_ptr(), n, lanes)
        b = eng.submit(H2D, 0, host.ptr, n, dst.data_ptr(), n, lanes, checksum=True)
        assert eng.wait(b).ok and eng.wait(a).ok
        assert torch.equal(dst, src)
