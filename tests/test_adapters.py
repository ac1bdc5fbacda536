"""Adapters on the CPU mock world: the real daemon, planner and executor move
bytes through simulated lanes (threads + memmove), so every adapter call
below is checked byte for byte, not just for the intents it emits.

Mirrors the reference's adapter suites (test_inference_adapters,
test_model_loading, test_training_offload, test_vllm_integration,
test_vllm_kv_connector) with different fixtures."""

import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from pcie_pool_b200 import TransferStatusState, TurboBusClient
from pcie_pool_b200.adapters import (AdapterTransferContext, InferenceKVSlot, InferenceKVSlotAdapter,
                                     ModelWeightLoader, TrainingOffloadManager, TurboBusConnector,
                                     TurboBusConnectorConfig, TurboBusConnectorMetadata, TurboBusSavedPrefix,
                                     VllmTurboBusIntegration, block_table_units, clear_connector_events,
                                     clear_saved_prefixes, extract_vllm_block_ids, get_connector_events,
                                     get_saved_prefix, make_contiguous_kv_slots,
                                     make_vllm_layer_range_refs_from_ids)
from pcie_pool_b200.adapters.vllm_kv_connector import TurboBusCPUBackingPool, TurboBusPrefixStore
from pcie_pool_b200.daemon import InProcessDaemonClient, IntentExecutor, TurboBusDaemon
from pcie_pool_b200.mock import MockDataPlane, MockWorld
from pcie_pool_b200.offload_store import BlockState, summarize_transfer_handles
from pcie_pool_b200.schema import WorkloadKind
from pcie_pool_b200.topology import StaticTopologyProvider

KiB = 1 << 10
MiB = 1 << 20


class Node:
    def __init__(self, gpus=4):
        self.world = MockWorld(gpu_count=gpus)
        self.plane = MockDataPlane(self.world)
        self.daemon = TurboBusDaemon(relay_gpus=range(1, gpus), max_inflight_chunks_per_relay=4096,
                                     topology_provider=StaticTopologyProvider(gpu_count=gpus),
                                     executor=IntentExecutor(self.plane))
        self.daemon.put_profile(0, list(range(1, gpus)), self.world.profile(0))
        self.dc = InProcessDaemonClient(self.daemon)
        r = self.dc.register_session(0, list(range(1, gpus)), max_inflight_chunks=4096)
        assert r.ok, r.error
        self.sid = r.payload["session"]["session_id"]
        assert self.dc.register_job("job", session_id=self.sid).ok
        self.client = TurboBusClient(daemon=self.dc)

    def register(self, name, tensor, kind, device=None):
        nbytes = tensor.numel() * tensor.element_size()
        r = self.dc.register_buffer(name, "job", kind, nbytes, device_index=device, address=tensor.data_ptr(),
                                    pinned=kind == "cpu_pinned")
        assert r.ok, r.error

    def ctx(self, kind=WorkloadKind.GENERIC, chunk=256 * KiB, **kw):
        return AdapterTransferContext("job", self.sid, "cpu", "gpu", workload_kind=kind,
                                      metadata={"chunk_bytes": chunk}, wait_timeout_seconds=60, **kw)


@pytest.fixture
def node():
    return Node()


def _rand(nbytes, seed):
    return torch.from_numpy(np.random.default_rng(seed).integers(0, 256, nbytes, dtype=np.uint8))


def test_training_offload_roundtrip(node):
    cpu, gpu = _rand(4 * MiB, 1), torch.zeros(4 * MiB, dtype=torch.uint8)
    node.register("cpu", cpu, "cpu_pinned")
    node.register("gpu", gpu, "gpu", device=0)
    m = TrainingOffloadManager(node.client, node.ctx(WorkloadKind.TRAINING_STATE))
    m.add_packed_buckets("p", cpu, gpu, bucket_bytes=1 * MiB, bucket_count=4)
    hs = m.prefetch_all()  # asynchronous: handles come back before the bytes land
    m.wait_all()
    assert torch.equal(gpu, cpu)
    assert all(m.block(n).state is BlockState.GPU for n in m.names())
    st = summarize_transfer_handles(hs)
    assert st.bytes == 4 * MiB and st.direct_chunks + st.relay_chunks == 16
    gpu.add_(1)
    m.offload_buckets(["p1", "p3"])
    m.wait_many(["p1", "p3"])
    want = _rand(4 * MiB, 1)
    want[1 * MiB:2 * MiB] += 1
    want[3 * MiB:] += 1
    assert torch.equal(cpu, want)
    assert m.block("p0").state is BlockState.GPU and m.block("p1").state is BlockState.CPU


def test_model_weight_loader_batch(node):
    cpu, gpu = _rand(3 * MiB, 2), torch.zeros(3 * MiB, dtype=torch.uint8)
    node.register("cpu", cpu, "cpu_pinned")
    node.register("gpu", gpu, "gpu", device=0)
    loader = ModelWeightLoader(node.client, node.ctx(WorkloadKind.MODEL_WEIGHTS))
    loader.add_packed_buckets("w", cpu, gpu, bucket_bytes=MiB, bucket_count=3)
    batch = loader.load_batch(loader.names())
    batch.wait()
    assert torch.equal(gpu, cpu)
    assert batch.transfer_stats().bytes == 3 * MiB
    assert [i.state for i in batch.block_infos()] == [BlockState.GPU] * 3
    loader.mark_unloaded()
    assert all(loader.block(n).state is BlockState.CPU for n in loader.names())


def test_inference_kv_slots_save_restore(node):
    block = 64 * KiB
    cpu, gpu = torch.zeros(16 * block, dtype=torch.uint8), _rand(16 * block, 3)
    node.register("cpu", cpu, "cpu_pinned")
    node.register("gpu", gpu, "gpu", device=0)
    ad = InferenceKVSlotAdapter(node.client, node.ctx(WorkloadKind.KV_CACHE), cpu, gpu)
    # gpu blocks 5..9 -> cpu slots 0..4, then back into gpu blocks 10..14
    slots = [InferenceKVSlot(f"b{i}", i, cpu_offset=i * block, gpu_offset=(5 + i) * block, byte_count=block)
             for i in range(5)]
    ad.register_slots(slots)
    ad.save_prefix([s.name for s in slots])
    assert torch.equal(cpu[:5 * block], gpu[5 * block:10 * block])
    back = [InferenceKVSlot(f"r{i}", i, cpu_offset=i * block, gpu_offset=(10 + i) * block, byte_count=block)
            for i in range(5)]
    ad.register_slots(back)
    ad.restore_prefix([s.name for s in back])
    assert torch.equal(gpu[10 * block:15 * block], gpu[5 * block:10 * block])
    assert len(make_contiguous_kv_slots("c", 4, block)) == 4


def test_vllm_range_refs_follow_cpu_slot_layout():
    kv = torch.zeros(2, 8, 16, 4, dtype=torch.bfloat16)  # [K/V, blocks, tokens, dim]
    bb = 16 * 4 * 2
    refs = make_vllm_layer_range_refs_from_ids("r", [3, 4, 7], [kv])
    # K lane: run [3,4] and [7]; V lane likewise; CPU slot = lane*n + index
    got = [(r.lane_id, r.cpu_slot, r.gpu_offset, r.byte_count) for r in refs]
    assert got == [(0, 0, 3 * bb, 2 * bb), (0, 2, 7 * bb, bb),
                   (1, 3, 8 * bb + 3 * bb, 2 * bb), (1, 5, 8 * bb + 7 * bb, bb)]
    addrs, unit = block_table_units([kv, kv], [3, 4, 7])
    base = kv.data_ptr()
    assert unit == bb and addrs.size == 12
    assert list(addrs[:6] - base) == [3 * bb, 4 * bb, 7 * bb, 11 * bb, 12 * bb, 15 * bb]


def test_vllm_integration_hooks_record_allocations(node):
    class Runner:
        def __init__(self):
            self.kv_caches = []

        def initialize_kv_cache(self, cfg):
            self.kv_caches = [torch.zeros(2, 8, 4, dtype=torch.uint8)]
            return "init"

    class Manager:
        def allocate_slots(self, request, n):
            return SimpleNamespace(get_block_ids=lambda allow_none=False: ([1, 2, 2 + n],))

    integ = VllmTurboBusIntegration(node.client, node.ctx(WorkloadKind.KV_CACHE))
    integ.install_on_classes(Runner, Manager)
    integ.install_on_classes(Runner, Manager)  # idempotent
    runner, mgr = Runner(), Manager()
    assert runner.initialize_kv_cache("cfg") == "init"
    assert len(integ.state.kv_caches) == 1
    seen = []
    integ.set_allocation_callback(lambda i, req, blocks, ev: seen.append(ev.block_ids))
    req = SimpleNamespace(request_id="q")
    mgr.allocate_slots(req, 1)
    mgr.allocate_slots(req, 2)
    assert integ.block_ids_for_request("q") == (1, 2, 3, 4)
    assert seen == [(1, 2, 3), (1, 2, 3, 4)]
    assert integ.state.allocations["q"].event_count == 2
    assert extract_vllm_block_ids([[5, None, 6]]) == ((5, 6),)
    with pytest.raises(RuntimeError):
        integ.require_adapter()


# ---- vLLM V1 connector --------------------------------------------------------------------------


class Cfg:
    def __init__(self, extra=None):
        self.cache_config = SimpleNamespace(block_size=16)
        self.kv_transfer_config = SimpleNamespace(engine_id=None, kv_connector_extra_config=dict(extra or {}))


class Req:
    def __init__(self, rid="r0", params=None, num_tokens=128):
        self.request_id, self.kv_transfer_params, self.num_tokens = rid, dict(params or {}), num_tokens


def blocks(ids):
    return SimpleNamespace(get_block_ids=lambda allow_none=False: (list(ids),))


@pytest.fixture(autouse=True)
def _quiet(monkeypatch):
    monkeypatch.setenv("TURBOBUS_CONNECTOR_EVENTS", "0")
    clear_saved_prefixes()
    clear_connector_events()
    yield
    clear_saved_prefixes()


def test_prefix_store_replace_isolate_evict():
    st = TurboBusPrefixStore(max_prefixes=2)
    a = TurboBusSavedPrefix("k", [], 1, 16)
    b = TurboBusSavedPrefix("k", [], 2, 32)
    assert st.put(a) == [] and st.put(b) == [a]
    assert st.get("k").block_count == 2
    st.put(TurboBusSavedPrefix("k", [], 3, 48, session_id="s2"))
    assert st.get("k", "s2").block_count == 3 and len(st) == 2
    ev = st.put(TurboBusSavedPrefix("z", [], 1, 16))
    assert [e.block_count for e in ev] == [2]  # oldest went first
    st.clear("s2")
    assert st.get("k", "s2") is None and len(st) == 1


def test_cpu_backing_pool_reuses_by_signature():
    kv = torch.zeros(2, 8, 4, dtype=torch.uint8)
    pool = TurboBusCPUBackingPool()
    b1, reused = pool.acquire(3, [kv, kv])
    assert not reused and b1["tensor"].numel() == 2 * 2 * 3 * 4
    pool.release(3, [kv, kv], b1)
    b2, reused = pool.acquire(3, [kv, kv])
    assert reused and b2 is b1
    assert not pool.acquire(4, [kv, kv])[1]


def test_connector_config_extra_and_env(monkeypatch):
    monkeypatch.setenv("TURBOBUS_CHUNK_BYTES", str(MiB))
    monkeypatch.setenv("TURBOBUS_RELAY_GPUS", "1,2")
    c = TurboBusConnectorConfig.from_vllm_config(Cfg({"turbobus.session_id": "s", "turbobus.restore_enabled": "true",
                                                      "turbobus.max_saved_prefixes": 4}))
    assert (c.session_id, c.job_id, c.chunk_bytes, c.restore_enabled, c.max_saved_prefixes, c.relay_gpus) == \
        ("s", "s", MiB, True, 4, (1, 2))
    assert c.wait_timeout_seconds == 600.0 and c.data_path == "engine"
    assert TurboBusConnector.requires_piecewise_for_cudagraph({})


def test_connector_match_needs_restore_enabled_and_saved_prefix():
    off = TurboBusConnector(Cfg(), "scheduler")
    r = Req(params={"turbobus.do_restore": True, "turbobus.prefix_key": "p", "turbobus.matched_tokens": 64})
    assert off.get_num_new_matched_tokens(r, 0) == (0, False)
    on = TurboBusConnector(Cfg({"turbobus.restore_enabled": True}), "scheduler")
    assert on.get_num_new_matched_tokens(r, 0) == (0, False)  # nothing saved yet
    from pcie_pool_b200.adapters import vllm_kv_connector as K

    K._PREFIX_STORE.put(TurboBusSavedPrefix("p", [], 4, 64))
    assert on.get_num_new_matched_tokens(r, 0) == (64, False)  # loaded synchronously in start_load_kv
    assert on.get_num_new_matched_tokens(r, 32) == (32, False)
    full = Req(params=dict(r.kv_transfer_params), num_tokens=64)
    assert on.get_num_new_matched_tokens(full, 0) == (63, False)  # last token is always computed
    asy = TurboBusConnector(Cfg({"turbobus.restore_enabled": True, "turbobus.load_async": True}), "scheduler")
    assert asy.get_num_new_matched_tokens(r, 0) == (64, True)
    assert [e["event"] for e in get_connector_events()].count("match") == 4


def test_connector_save_waits_then_collects_from_scheduler_output():
    c = TurboBusConnector(Cfg(), "scheduler")
    r = Req("s1", {"turbobus.do_save": True, "turbobus.prefix_key": "p", "turbobus.save_blocks": 4})
    c.update_state_after_alloc(r, blocks([7, 8]), 0)
    assert len(c.build_connector_meta(None)) == 0
    out = SimpleNamespace(scheduled_new_reqs=[], scheduled_cached_reqs=SimpleNamespace(
        req_ids=["s1"], new_block_ids=[([7, 8, 9, 10],)]))
    md = c.build_connector_meta(out)
    assert [(m.request_id, m.block_ids, m.matched_tokens) for m in md.save_requests] == [("s1", (7, 8, 9, 10), 64)]
    assert c.request_finished(r, [7, 8, 9, 10]) == (False, {"turbobus.prefix_key": "p",
                                                           "turbobus.matched_tokens": 64})
    assert c.request_finished(Req("x"), []) == (False, None)


def test_connector_wait_for_save_rejects_missing_layer():
    c = TurboBusConnector(Cfg(), "worker")
    c.register_kv_caches({"l0": torch.zeros(2, 8, 4), "l1": torch.zeros(2, 8, 4)})
    md = TurboBusConnectorMetadata()
    from pcie_pool_b200.adapters.vllm_kv_connector import TurboBusRequestMetadata

    md.add_save_request(TurboBusRequestMetadata("r", "p", (1, 2), 32, 2))
    c.bind_connector_metadata(md)
    with pytest.raises(RuntimeError, match="save_kv_layer"):
        c.wait_for_save()
    c.save_kv_layer("l0", None, None)
    with pytest.raises(RuntimeError, match="1 of 2"):
        c.wait_for_save()


def test_connector_intent_path_save_then_restore_permuted(node):
    """Full lifecycle on the intent path: save blocks [9, 2, 5] of one layer,
    restore into [0, 11, 4] -- the data must land through the mock lanes."""
    nblk, bb = 16, 4 * KiB
    kv = _rand(2 * nblk * bb, 7).view(2, nblk, bb)
    node.register("gpu", kv, "gpu", device=0)
    cfg = Cfg({"turbobus.session_id": node.sid, "turbobus.job_id": "job", "turbobus.cpu_buffer_id": "cpu",
               "turbobus.gpu_buffer_id": "gpu", "turbobus.chunk_bytes": 4 * KiB, "turbobus.data_path": "intent",
               "turbobus.restore_enabled": True})
    sched, work = TurboBusConnector(cfg, "scheduler"), TurboBusConnector(cfg, "worker")
    work.client = node.client
    work.register_kv_caches({"l0": kv})
    # the backing the pool will hand out is registered as the daemon's "cpu" buffer
    backing, _ = work._backing_pool.acquire(3, [kv])
    node.register("cpu", backing["tensor"], "cpu_pinned")
    work._backing_pool.release(3, [kv], backing)

    save = Req("s", {"turbobus.do_save": True, "turbobus.prefix_key": "pfx", "turbobus.save_blocks": 3})
    sched.update_state_after_alloc(save, blocks([9, 2, 5]), 0)
    work.bind_connector_metadata(sched.build_connector_meta(None))
    work.save_kv_layer("l0", kv, None)
    work.wait_for_save()
    saved = get_saved_prefix("pfx", node.sid)
    assert saved is not None and saved.block_count == 3 and saved.bytes == 2 * 3 * bb
    host = backing["tensor"].view(2, 3, bb)
    for lane in range(2):
        for i, b in enumerate([9, 2, 5]):
            assert torch.equal(host[lane, i], kv[lane, b])
    work.clear_connector_metadata()
    expect = kv[:, [9, 2, 5]].clone()

    load = Req("l", {"turbobus.do_restore": True, "turbobus.prefix_key": "pfx"}, num_tokens=100)
    n, async_ = sched.get_num_new_matched_tokens(load, 0)
    assert (n, async_) == (48, False)
    sched.update_state_after_alloc(load, blocks([0, 11, 4, 13]), n)
    work.bind_connector_metadata(sched.build_connector_meta(None))
    work.start_load_kv(None)
    assert torch.equal(kv[:, [0, 11, 4]], expect)
    assert work.get_finished(set()) == (None, None)  # synchronous load: nothing pending
    evs = [e["event"] for e in get_connector_events()]
    assert "save" in evs and "restore" in evs


@pytest.mark.gpu
def test_connector_engine_path_gpu(need_gpu):
    """Engine data path on a real GPU: the whole prefix (2 layers x K/V) is
    one gather on save and one scatter on restore, including a partial
    restore of the first blocks."""
    nblk, tok, dim = 64, 16, 128
    kvs = {f"l{i}": torch.randn(2, nblk, tok, dim, device="cuda").to(torch.bfloat16) for i in range(2)}
    cfg = Cfg({"turbobus.restore_enabled": True, "turbobus.chunk_bytes": 64 * KiB})
    sched, work = TurboBusConnector(cfg, "scheduler"), TurboBusConnector(cfg, "worker")
    work.register_kv_caches(kvs)
    src = [40, 3, 17, 9, 63, 0]
    sched.update_state_after_alloc(Req("s", {"turbobus.do_save": True, "turbobus.prefix_key": "g",
                                             "turbobus.save_blocks": len(src)}), blocks(src), 0)
    work.bind_connector_metadata(sched.build_connector_meta(None))
    for name, kv in kvs.items():
        work.save_kv_layer(name, kv, None)
    work.wait_for_save()
    torch.cuda.synchronize()
    expect = {n: kv[:, src].clone() for n, kv in kvs.items()}
    work.clear_connector_metadata()
    dst = [5, 6, 60, 1, 2, 30]
    ld = Req("l", {"turbobus.do_restore": True, "turbobus.prefix_key": "g"}, num_tokens=1000)
    n, _ = sched.get_num_new_matched_tokens(ld, 0)
    sched.update_state_after_alloc(ld, blocks(dst), n)
    work.bind_connector_metadata(sched.build_connector_meta(None))
    work.start_load_kv(None)
    torch.cuda.synchronize()
    for name, kv in kvs.items():
        assert torch.equal(kv[:, dst], expect[name])
    # partial restore: the first 2 blocks only, into fresh ids
    work.clear_connector_metadata()
    sched.restore_block_limit = 2
    ld2 = Req("l2", {"turbobus.do_restore": True, "turbobus.prefix_key": "g"}, num_tokens=1000)
    n, _ = sched.get_num_new_matched_tokens(ld2, 0)
    sched.update_state_after_alloc(ld2, blocks([20, 21]), n)
    work.bind_connector_metadata(sched.build_connector_meta(None))
    work.start_load_kv(None)
    torch.cuda.synchronize()
    for name, kv in kvs.items():
        assert torch.equal(kv[:, [20, 21]], expect[name][:, :2])
