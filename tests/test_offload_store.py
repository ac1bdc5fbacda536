"""Offload store over a recording intent client: registry rules, batched
and unbatched submissions, intent shape (direction, buffers, ranges,
policy, metadata), receipt checks, wait semantics (live receipts, terminal
failures), block state transitions, stats and bucket helpers.  Behaviours
follow unit/test_offload_store.py of the reference with independent fakes."""

from __future__ import annotations

import pytest

from pcie_pool_b200.offload_store import (AdapterTransferContext, BlockState, BucketStoreMixin, OffloadStore,
                                          ReceiptTransferHandle, TransferStats, summarize_transfer_handles,
                                          transfer_stats_from_receipt)
from pcie_pool_b200.schema import TransferReceipt, TransferStatusState, WorkloadKind


class Tensor:
    def __init__(self, n: int, elem: int = 1) -> None:
        self.n, self.elem = n, elem

    def numel(self) -> int:
        return self.n

    def element_size(self) -> int:
        return self.elem


def receipt(it, state, relay_share: float = 0.25, error=None, intent_id=None):
    done = it.total_bytes if state is TransferStatusState.COMPLETE else 0
    relay = int(it.total_bytes * relay_share)
    return TransferReceipt(receipt_id="r-" + it.intent_id, ticket_id="t", intent_id=intent_id or it.intent_id,
                           decision_id="d", topology_snapshot_id="s", job_id=it.job_id, session_id=it.session_id,
                           state=state, bytes_total=it.total_bytes, bytes_completed=done, error=error,
                           path_stats=({"kind": "direct", "bytes": it.total_bytes - relay, "chunk_count": 3},
                                       {"kind": "relay", "bytes": relay, "chunk_count": 1}))


class Client:
    """Records intents; ``final`` decides the receipt a wait returns;
    ``live_waits`` makes the first N waits return a running receipt."""

    def __init__(self, final=TransferStatusState.COMPLETE, live_waits: int = 0, bad_id: bool = False):
        self.intents, self.waits = [], []
        self.final, self.live_waits, self.bad_id = final, live_waits, bad_id

    def submit_transfer_intent(self, it):
        self.intents.append(it)
        return receipt(it, TransferStatusState.RUNNING, intent_id="other" if self.bad_id else None)

    def wait_transfer_receipt(self, intent_id, timeout_seconds=None):
        self.waits.append((intent_id, timeout_seconds))
        it = next(i for i in self.intents if i.intent_id == intent_id)
        if self.live_waits:
            self.live_waits -= 1
            return receipt(it, TransferStatusState.RUNNING)
        err = None if self.final is TransferStatusState.COMPLETE else "lane lost"
        return receipt(it, self.final, error=err)


def ctx(**over):
    kw = dict(job_id="j", session_id="s", cpu_buffer_id="cpu", gpu_buffer_id="gpu", intent_prefix="t")
    kw.update(over)
    return AdapterTransferContext(**kw)


def store(client=None, **over):
    s = OffloadStore(client or Client(), ctx(**over))
    cpu, gpu = Tensor(8192), Tensor(8192)
    for i in range(4):
        s.add(f"b{i}", cpu, gpu, cpu_offset=i * 2048, gpu_offset=(3 - i) * 2048, byte_count=2048)
    return s


def test_context_validation():
    with pytest.raises(ValueError):
        ctx(job_id=" ")
    with pytest.raises(ValueError, match="physical"):
        ctx(policy_hints={"relay_gpus": [1]})
    with pytest.raises(ValueError, match="non-negative"):
        ctx(wait_timeout_seconds=-1)
    c = ctx(workload_kind="kv_cache", intent_prefix=None)
    assert c.workload_kind is WorkloadKind.KV_CACHE and c.intent_prefix.startswith("adapter-")


def test_registry_rules():
    s = store()
    with pytest.raises(ValueError, match="already exists"):
        s.add("b0", Tensor(1))
    with pytest.raises(ValueError, match="non-negative"):
        s.add("x", Tensor(1), cpu_offset=-1)
    with pytest.raises(ValueError, match="positive"):
        s.add("x", Tensor(1), byte_count=0)
    with pytest.raises(ValueError, match="non-empty"):
        s.add("", Tensor(1))
    with pytest.raises(KeyError, match="unknown offload block"):
        s.block("nope")
    assert s.names() == ["b0", "b1", "b2", "b3"] and s.block_ids() == ["b0", "b1", "b2", "b3"]
    assert s.remove("b3").name == "b3" and "b3" not in s.names()


def test_batched_prefetch_is_one_multi_range_intent():
    c = Client()
    s = store(c, priority=2, metadata={"owner": "test"}, workload_kind="training_state")
    batch = s.submit_prefetch_many(["b0", "b2"])
    assert len(c.intents) == 1
    it = c.intents[0]
    assert it.intent_id == "t-prefetch-1" and it.direction == "h2d"
    assert (it.source_buffer_id, it.destination_buffer_id) == ("cpu", "gpu")
    assert [dict(r) for r in it.ranges] == [{"src_offset": 0, "dst_offset": 6144, "bytes": 2048},
                                            {"src_offset": 4096, "dst_offset": 2048, "bytes": 2048}]
    assert it.priority == 2 and it.workload_kind is WorkloadKind.TRAINING_STATE
    assert it.metadata["owner"] == "test" and it.metadata["block_names"] == ["b0", "b2"]
    assert batch.handles[0] is batch.handles[1]
    assert s.block("b0").state is BlockState.PREFETCHING
    batch.wait()
    assert s.block("b0").state is BlockState.GPU and s.block("b1").state is BlockState.CPU
    assert len(c.waits) == 1, "one shared handle is waited once"


def test_evict_swaps_source_and_destination():
    c = Client()
    s = store(c)
    s.evict("b1")
    it = c.intents[0]
    assert it.direction == "d2h" and (it.source_buffer_id, it.destination_buffer_id) == ("gpu", "cpu")
    assert dict(it.ranges[0]) == {"src_offset": 4096, "dst_offset": 2048, "bytes": 2048}
    assert s.block("b1").state is BlockState.EVICTING
    s.wait("b1")
    assert s.block("b1").state is BlockState.CPU


def test_blocks_over_different_tensors_are_submitted_one_by_one():
    c = Client()
    s = OffloadStore(c, ctx())
    s.add("x", Tensor(100), Tensor(100))
    s.add("y", Tensor(300, elem=2), Tensor(300, elem=2))
    handles = s.prefetch_many(["x", "y"])
    assert len(c.intents) == 2 and handles[0] is not handles[1]
    assert [it.total_bytes for it in c.intents] == [100, 600], "bytes come from the tensor size"


def test_live_receipt_does_not_end_the_wait():
    c = Client(live_waits=1)
    s = store(c, wait_timeout_seconds=0.5)
    h = s.prefetch("b0")
    h.wait()
    assert h.receipt.state is TransferStatusState.RUNNING and h.wait_calls == 1
    h.wait()
    assert h.receipt.state is TransferStatusState.COMPLETE and h.wait_calls == 2
    h.wait()
    assert h.wait_calls == 2, "a terminal handle is not waited again"
    assert c.waits[0][1] == 0.5, "the context's timeout is passed through"


def test_failed_transfer_raises_on_wait():
    s = store(Client(final=TransferStatusState.FAILED))
    s.prefetch("b0")
    with pytest.raises(RuntimeError, match="lane lost"):
        s.wait("b0")


def test_mismatched_receipt_is_rejected():
    with pytest.raises(ValueError, match="does not match"):
        store(Client(bad_id=True)).prefetch("b0")


def test_stats_and_infos():
    s = store()
    assert s.transfer_stats("b0") is None and s.stats("b0") is None
    s.prefetch_many(["b0", "b1"])
    s.wait_all() if isinstance(s, BucketStoreMixin) else s.wait_many(["b0", "b1"])
    st = s.transfer_stats_many(["b0", "b1"])
    assert st == TransferStats(bytes=4096, direct_chunks=3, relay_chunks=1), "a shared handle counts once"
    info = s.block_info("b0").as_dict()
    assert info["state"] == "gpu" and info["last_operation"] == "prefetch" and info["bytes"] == 2048
    assert info["transfer_stats"]["bytes"] == 4096


def test_set_state_and_clear():
    s = store()
    s.prefetch("b0")
    s.set_block_state("b0", BlockState.CPU, clear_transfer_state=True)
    b = s.block("b0")
    assert b.state is BlockState.CPU and b.last_handle is None and b.last_operation is None
    s.wait("b0")  # nothing in flight: a no-op
    assert s.block("b0").state is BlockState.CPU


def test_receipt_helpers():
    class It:
        intent_id, job_id, session_id, total_bytes = "i", "j", "s", 1000

    r = receipt(It(), TransferStatusState.COMPLETE, relay_share=0.4)
    assert transfer_stats_from_receipt(r) == TransferStats(bytes=1000, direct_chunks=3, relay_chunks=1)

    class H:
        stats = {"bytes": 10, "direct_chunks": 1, "relay_chunks": 2}

    h = H()
    assert summarize_transfer_handles([h, h, object()]) == TransferStats(10, 1, 2)
    assert isinstance(ReceiptTransferHandle(Client(), None, r).stats, TransferStats)


def test_bucket_helpers():
    from pcie_pool_b200.adapters.training_offload import TrainingOffloadStore

    s = TrainingOffloadStore(Client(), ctx())
    got = s.add_packed_buckets("p", Tensor(4096), Tensor(4096), bucket_bytes=1024, bucket_count=4, start_offset=0)
    assert [b.cpu_offset for b in got] == [0, 1024, 2048, 3072] and s.bucket("p2").block_id == 2
    with pytest.raises(ValueError, match="bucket_bytes"):
        s.add_packed_buckets("q", Tensor(1), Tensor(1), bucket_bytes=0, bucket_count=1)
    assert [i.name for i in s.bucket_infos()] == ["p0", "p1", "p2", "p3"]


# ---- further rules: empty batches, waits before any transfer, handle summaries ---------------------------

def test_an_empty_batch_submits_nothing_and_waits_for_nothing():
    c = Client()
    s = store(c)
    batch = s.submit_prefetch_many([])
    assert batch.names == () and batch.handles == () and c.intents == []
    batch.wait()
    assert batch.transfer_stats().bytes == 0 and batch.as_dict()["blocks"] == []
    assert s.prefetch_many([]) == [] and s.evict_many([]) == []


def test_waiting_before_any_transfer_is_a_no_op():
    c = Client()
    s = store(c)
    s.wait("b0")
    s.wait_many(["b1", "b2"])
    assert c.waits == [] and s.transfer_stats("b0") is None
    assert s.block_info("b0").state == s.block("b0").state


def test_packed_evict_reverses_each_range_and_keeps_block_order():
    c = Client()
    s = store(c)
    s.evict_many(["b3", "b1"])
    (it,) = c.intents
    assert it.direction == "d2h" and it.source_buffer_id == "gpu" and it.destination_buffer_id == "cpu"
    assert [(r["src_offset"], r["dst_offset"]) for r in it.ranges] == [(0, 3 * 2048), (2 * 2048, 2048)]
    assert it.metadata["block_names"] == ["b3", "b1"] and it.metadata["operation"] == "evict"


def test_blocks_carry_connector_fields_into_their_infos():
    s = OffloadStore(Client(), ctx())
    cpu, gpu = Tensor(4096), Tensor(4096)
    s.add("kv", cpu, gpu, block_id=("req", 0, 7), cpu_slot=3, gpu_slot=7, cpu_offset=1024, gpu_offset=2048,
          byte_count=512)
    info = s.block_info("kv").as_dict()
    assert (info["block_id"], info["cpu_slot"], info["gpu_slot"]) == (("req", 0, 7), 3, 7)
    assert [i.name for i in s.block_infos(["kv"])] == ["kv"] and s.block_ids() == [("req", 0, 7)]
    for bad in ({"cpu_offset": -1}, {"gpu_offset": -8}, {"byte_count": 0}):
        with pytest.raises(ValueError):
            s.add("other", cpu, gpu, **bad)
    with pytest.raises(ValueError, match="already exists"):
        s.add("kv", cpu, gpu)
    with pytest.raises(ValueError, match="non-empty"):
        s.add("", cpu, gpu)


def test_handle_summaries_count_a_shared_handle_once_and_accept_dict_stats():
    from types import SimpleNamespace

    from pcie_pool_b200.offload_store import summarize_transfer_handles, transfer_stats_from_receipt

    c = Client()
    s = store(c)
    batch = s.submit_prefetch_many(["b0", "b1", "b2"])
    assert len({id(h) for h in batch.handles}) == 1
    one = summarize_transfer_handles(batch.handles)
    assert one == transfer_stats_from_receipt(batch.handles[0].receipt)
    d = SimpleNamespace(stats={"bytes": 10, "direct_chunks": 1, "relay_chunks": 2})
    both = summarize_transfer_handles([*batch.handles, d, object()])
    assert (both.bytes, both.direct_chunks, both.relay_chunks) == (one.bytes + 10, one.direct_chunks + 1,
                                                                   one.relay_chunks + 2)
