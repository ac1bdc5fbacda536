"""Framework adapters over a recording intent client: KV slots (save =
D2H evict, restore = H2D prefetch, batches, stats, contiguous slot layout),
the model-weight loader and the training offload manager (bucket packing,
load / prefetch / offload batches, state marks), and their intent shapes.
Behaviours follow e2e/test_inference_adapters.py, test_model_loading.py and
test_training_offload.py of the reference with independent fakes."""

from __future__ import annotations

import pytest

from pcie_pool_b200.adapters import (FrameworkKVSlotAdapter, InferenceKVSlot, InferenceKVSlotAdapter,
                                     ModelWeightLoader, TrainingOffloadManager, make_contiguous_kv_slots)
from pcie_pool_b200.offload_store import AdapterTransferContext, BlockState, TransferStats
from pcie_pool_b200.schema import TransferReceipt, TransferStatusState, WorkloadKind


class Tensor:
    def __init__(self, n):
        self.n = n

    def numel(self):
        return self.n

    def element_size(self):
        return 1


class Client:
    def __init__(self):
        self.intents = []

    def submit_transfer_intent(self, it):
        self.intents.append(it)
        return self._receipt(it, TransferStatusState.RUNNING)

    def wait_transfer_receipt(self, intent_id, timeout_seconds=None):
        return self._receipt(next(i for i in self.intents if i.intent_id == intent_id), TransferStatusState.COMPLETE)

    @staticmethod
    def _receipt(it, state):
        done = it.total_bytes if state is TransferStatusState.COMPLETE else 0
        return TransferReceipt(receipt_id="r" + it.intent_id, ticket_id="t", intent_id=it.intent_id, decision_id="d",
                               topology_snapshot_id="s", job_id=it.job_id, session_id=it.session_id, state=state,
                               bytes_total=it.total_bytes, bytes_completed=done,
                               path_stats=({"kind": "relay", "bytes": it.total_bytes, "chunk_count": 2},))


def ctx(kind=WorkloadKind.GENERIC, **kw):
    return AdapterTransferContext("job", "sess", "cpu", "gpu", workload_kind=kind, intent_prefix="a", **kw)


# ---- KV slots --------------------------------------------------------------------------------------------

def kv_adapter(client=None):
    c = client or Client()
    ad = InferenceKVSlotAdapter(c, ctx(WorkloadKind.KV_CACHE), Tensor(1 << 20), Tensor(1 << 20))
    return c, ad


def test_contiguous_slot_layout():
    slots = make_contiguous_kv_slots("L0.", 3, 4096)
    assert [(s.name, s.block_id, s.cpu_offset, s.gpu_offset, s.byte_count) for s in slots] == [
        ("L0.0", 0, 0, 0, 4096), ("L0.1", 1, 4096, 4096, 4096), ("L0.2", 2, 8192, 8192, 4096)]
    assert FrameworkKVSlotAdapter is InferenceKVSlotAdapter


def test_save_is_one_d2h_intent_from_gpu_slots_to_cpu_slots():
    c, ad = kv_adapter()
    ad.register_slots([InferenceKVSlot(f"b{i}", 10 + i, cpu_offset=i * 4096, gpu_offset=(7 - i) * 4096,
                                       byte_count=4096) for i in range(3)])
    ad.save_prefix(["b0", "b1", "b2"])
    (it,) = c.intents
    assert it.direction == "d2h" and it.workload_kind is WorkloadKind.KV_CACHE
    assert (it.source_buffer_id, it.destination_buffer_id) == ("gpu", "cpu")
    assert [r["src_offset"] for r in it.ranges] == [7 * 4096, 6 * 4096, 5 * 4096]
    assert [r["dst_offset"] for r in it.ranges] == [0, 4096, 8192]
    assert all(ad.block(n).state is BlockState.CPU for n in ("b0", "b1", "b2"))
    assert ad.block("b1").block_id == 11


def test_restore_prefix_and_batches():
    c, ad = kv_adapter()
    ad.register_slots(make_contiguous_kv_slots("s", 4, 1024))
    names, handles = ad.submit_restore_prefix(["s0", "s1"])
    assert names == ["s0", "s1"] and handles[0] is handles[1]
    assert ad.block("s0").state is BlockState.PREFETCHING
    ad.wait_prefix(names)
    assert ad.block("s0").state is BlockState.GPU
    batch = ad.save_batch(["s2", "s3"])
    assert batch.operation == "save" and batch.names == ("s2", "s3")
    batch.wait()
    assert ad.transfer_stats(["s2", "s3"]) == TransferStats(bytes=2048, direct_chunks=0, relay_chunks=2)
    rb = ad.restore_batch(["s3"])
    assert rb.as_dict()["operation"] == "restore" and c.intents[-1].direction == "h2d"


def test_duplicate_slot_names_are_refused():
    _c, ad = kv_adapter()
    ad.register_slots(make_contiguous_kv_slots("s", 1, 1024))
    with pytest.raises(ValueError, match="already exists"):
        ad.register_slots(make_contiguous_kv_slots("s", 1, 1024))


# ---- model weights -------------------------------------------------------------------------------------

def test_model_loader_packs_buckets_and_loads_them_as_one_intent():
    c = Client()
    ml = ModelWeightLoader(c, ctx(WorkloadKind.MODEL_WEIGHTS, priority=3))
    ml.add_packed_buckets("w", Tensor(8192), Tensor(8192), bucket_bytes=2048, bucket_count=4)
    assert ml.names() == ["w0", "w1", "w2", "w3"]
    ml.load_all()
    (it,) = c.intents
    assert it.direction == "h2d" and it.total_bytes == 8192 and it.priority == 3
    assert it.workload_kind is WorkloadKind.MODEL_WEIGHTS and len(it.ranges) == 4
    ml.wait_all()
    assert all(ml.bucket(n).state is BlockState.GPU for n in ml.names())
    ml.mark_unloaded(["w1"])
    assert ml.bucket("w1").state is BlockState.CPU and ml.bucket("w1").last_handle is None
    b = ml.load_batch(["w1", "w2"])
    assert b.names == ("w1", "w2") and len(c.intents) == 2


# ---- training offload -------------------------------------------------------------------------------------

def test_training_manager_prefetch_offload_cycle():
    c = Client()
    tm = TrainingOffloadManager(c, ctx(WorkloadKind.TRAINING_STATE))
    tm.add_packed_buckets("p", Tensor(4096), Tensor(4096), bucket_bytes=1024, bucket_count=4)
    tm.prefetch_buckets(["p0", "p1"])
    tm.wait_all()
    assert [tm.bucket(n).state for n in ("p0", "p1", "p2")] == [BlockState.GPU, BlockState.GPU, BlockState.CPU]
    tm.offload_buckets(["p0", "p1"])
    tm.wait_all()
    assert [i.direction for i in c.intents] == ["h2d", "d2h"]
    assert tm.bucket("p0").state is BlockState.CPU
    tm.mark_on_gpu()
    assert all(tm.bucket(n).state is BlockState.GPU for n in tm.names())
    tm.mark_on_cpu(["p3"])
    assert tm.bucket("p3").state is BlockState.CPU
    assert [b.info().as_dict()["bytes"] for b in tm.blocks()] == [1024] * 4


# ---- model loading and training offload, rule by rule ---------------------------------------------------

def test_buckets_carry_their_metadata_and_load_as_model_weight_intents():
    c = Client()
    ml = ModelWeightLoader(c, ctx(WorkloadKind.MODEL_WEIGHTS))
    cpu, gpu = Tensor(4 << 20), Tensor(4 << 20)
    b = ml.add_bucket("embed", cpu, gpu, bucket_id=7, cpu_offset=0, gpu_offset=1 << 20, byte_count=1 << 20)
    assert (b.block_id, b.cpu_slot, b.gpu_slot, b.bytes) == (7, 7, 7, 1 << 20)
    info = ml.bucket_info("embed")
    assert info.state is not BlockState.GPU
    ml.load_bucket("embed")
    (it,) = c.intents
    assert (it.direction, it.workload_kind.value, it.total_bytes) == ("h2d", "model_weights", 1 << 20)
    assert it.ranges[0] == {"src_offset": 0, "dst_offset": 1 << 20, "bytes": 1 << 20}
    ml.wait("embed")
    assert ml.bucket_info("embed").state is BlockState.GPU
    ml.mark_unloaded(["embed"])
    assert ml.bucket_info("embed").state is BlockState.CPU and len(c.intents) == 1, "marking copies nothing"
    assert ml.transfer_stats("embed") is None, "the transfer state is reset"


def test_packed_model_buckets_load_as_one_intent_and_batches_are_objects():
    c = Client()
    ml = ModelWeightLoader(c, ctx(WorkloadKind.MODEL_WEIGHTS))
    ml.add_packed_buckets("w", Tensor(8 << 20), Tensor(8 << 20), bucket_bytes=1 << 20, bucket_count=8)
    batch = ml.load_batch([f"w{i}" for i in range(8)])
    assert len(c.intents) == 1 and len(c.intents[0].ranges) == 8 and batch.operation == "prefetch"
    batch.wait()
    assert all(ml.bucket_info(f"w{i}").state is BlockState.GPU for i in range(8))
    assert batch.transfer_stats().bytes == 8 << 20 and len(batch.as_dict()["blocks"]) == 8
    with pytest.raises(ValueError):
        ml.add_packed_buckets("x", Tensor(8), Tensor(8), bucket_bytes=0, bucket_count=1)


def test_training_buckets_move_both_ways_as_range_intents():
    c = Client()
    tm = TrainingOffloadManager(c, ctx(WorkloadKind.OPTIMIZER_STATE))
    tm.add_packed_buckets("opt", Tensor(4 << 20), Tensor(4 << 20), bucket_bytes=1 << 20, bucket_count=4,
                          start_offset=0)
    names = [f"opt{i}" for i in range(4)]
    pre = tm.prefetch_batch(names)
    pre.wait()
    off = tm.offload_batch(names[::-1])
    off.wait()
    p, o = c.intents
    assert (p.direction, o.direction) == ("h2d", "d2h") and p.workload_kind.value == "optimizer_state"
    assert [r["src_offset"] for r in o.ranges] == [3 << 20, 2 << 20, 1 << 20, 0]
    assert all(tm.bucket_info(n).state is BlockState.CPU for n in names)
    tm.mark_on_gpu(names[:2])
    assert [tm.bucket_info(n).state for n in names[:2]] == [BlockState.GPU] * 2 and len(c.intents) == 2
    tm.mark_on_cpu()
    assert all(tm.bucket_info(n).state is BlockState.CPU for n in names)
