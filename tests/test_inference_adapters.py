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
