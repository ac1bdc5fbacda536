"""vLLM KV block mapping on CPU tensors shaped like vLLM's caches: block
bytes from the block stride, block refs across layers, byte-range refs per
K/V lane with contiguous block runs merged (and non-contiguous runs kept
apart), the CPU backing order, the per-unit address table of the fused
kernels for both cache layouts, and the slot adapter's transfers: one intent
per layer group, every layer submitted before any wait, a wait failure
surfacing, and statistics summed over groups.  Behaviours follow
e2e/test_inference_adapters.py (vLLM cases) of the reference with
independent fakes."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from test_inference_adapters import Client, ctx

from pcie_pool_b200.adapters.vllm import (VllmKVBlockRef, VllmKVSlotAdapter, block_bytes_from_vllm_kv_tensor,
                                          block_table_units, contiguous_runs, kv_layout,
                                          make_vllm_block_refs_from_ids, make_vllm_layer_block_refs_from_ids,
                                          make_vllm_layer_groups_from_kv_caches, make_vllm_layer_range_refs_from_ids,
                                          vllm_block_name)
from pcie_pool_b200.schema import TransferStatusState, WorkloadKind

BLOCKS, BLOCK, HEADS, DIM = 8, 16, 2, 8  # one block of one lane: 16 * 2 * 8 * 2 bytes (bf16) = 512 B


def caches(layers=2, layout="kv_first"):
    shape = (2, BLOCKS, BLOCK, HEADS, DIM) if layout == "kv_first" else (BLOCKS, 2, BLOCK, HEADS, DIM)
    return [torch.zeros(shape, dtype=torch.bfloat16) for _ in range(layers)]


UNIT = BLOCK * HEADS * DIM * 2


def test_block_bytes_follow_the_block_stride():
    kv = caches(1)[0]
    assert block_bytes_from_vllm_kv_tensor(kv) == UNIT
    assert block_bytes_from_vllm_kv_tensor(caches(1, "blocks_first")[0]) == 2 * UNIT
    with pytest.raises(ValueError, match="two dimensions"):
        block_bytes_from_vllm_kv_tensor(torch.zeros(4))


def test_range_refs_of_a_blocks_first_cache_cover_whole_blocks():
    kv = caches(1, "blocks_first")
    refs = make_vllm_layer_range_refs_from_ids("r", [1, 2, 6], kv)
    assert [(r.lane_id, r.gpu_offset, r.cpu_offset, r.byte_count) for r in refs] == [
        (None, 2 * UNIT, 0, 4 * UNIT), (None, 12 * UNIT, 4 * UNIT, 2 * UNIT)]


def test_block_refs_expand_across_layers_in_cpu_slot_order():
    refs = make_vllm_layer_block_refs_from_ids("r", [5, 2, 7], layer_count=2, cpu_slot_start=10)
    assert [(r.group_id, r.block_id, r.cpu_slot, r.gpu_slot) for r in refs] == [
        (0, 5, 10, 5), (0, 2, 11, 2), (0, 7, 12, 7), (1, 5, 10, 5), (1, 2, 11, 2), (1, 7, 12, 7)]
    one = make_vllm_block_refs_from_ids("r", 3, [4, 6])
    assert [(r.group_id, r.cpu_slot, r.gpu_slot) for r in one] == [(3, 0, 4), (3, 1, 6)]
    assert vllm_block_name(VllmKVBlockRef("r", 1, 4, 0, 4, lane_id=1, byte_count=64)) == "r:g1:b4:l1:bytes64"


def test_contiguous_runs():
    assert contiguous_runs([3, 4, 5, 9, 10, 2]) == [(0, [3, 4, 5]), (3, [9, 10]), (5, [2])]
    assert contiguous_runs([]) == []


def test_range_refs_merge_contiguous_blocks_per_lane():
    kv = caches(1)
    refs = make_vllm_layer_range_refs_from_ids("r", [2, 3, 4], kv)
    assert len(refs) == 2, "one ref per lane for one contiguous run"
    k, v = refs
    lane_bytes = kv[0].stride(0) * 2
    assert (k.lane_id, k.gpu_offset, k.cpu_offset, k.byte_count) == (0, 2 * UNIT, 0, 3 * UNIT)
    assert (v.lane_id, v.gpu_offset, v.cpu_offset, v.byte_count) == (1, lane_bytes + 2 * UNIT, 3 * UNIT, 3 * UNIT)


def test_range_refs_keep_noncontiguous_runs_apart_and_cover_every_layer():
    kv = caches(2)
    refs = make_vllm_layer_range_refs_from_ids("r", [6, 1, 2], kv, cpu_slot_start=4)
    assert len(refs) == 2 * 2 * 2  # layers x lanes x runs
    layer0 = [(r.lane_id, r.block_id, r.cpu_slot, r.byte_count) for r in refs if r.group_id == 0]
    assert layer0 == [(0, 6, 4, UNIT), (0, 1, 5, 2 * UNIT), (1, 6, 7, UNIT), (1, 1, 8, 2 * UNIT)]
    assert sum(r.byte_count for r in refs) == 2 * 2 * 3 * UNIT


def test_kv_layouts_and_the_unit_address_table():
    a = caches(2, "kv_first")
    lay = kv_layout(a[0])
    assert (lay.lanes, lay.unit_bytes, lay.num_blocks) == (2, UNIT, BLOCKS)
    addrs, unit = block_table_units(a, [3, 0])
    assert unit == UNIT and addrs.dtype == np.uint64 and addrs.size == 2 * 2 * 2
    base0, lane = a[0].data_ptr(), a[0].stride(0) * 2
    assert addrs[:4].tolist() == [base0 + 3 * UNIT, base0, base0 + lane + 3 * UNIT, base0 + lane]
    assert addrs[4] == a[1].data_ptr() + 3 * UNIT
    b = caches(1, "blocks_first")
    lay = kv_layout(b[0])
    assert (lay.lanes, lay.unit_bytes) == (1, 2 * UNIT)
    addrs, unit = block_table_units(b, [5])
    assert unit == 2 * UNIT and addrs.tolist() == [b[0].data_ptr() + 5 * 2 * UNIT]
    with pytest.raises(ValueError, match="one block size"):
        block_table_units([a[0], b[0]], [0])
    with pytest.raises(ValueError, match="no KV caches"):
        block_table_units([], [0])


# ---- the slot adapter over layer groups ------------------------------------------------------------------

class Recording(Client):
    """Intent client that logs the order of submits and waits; ``fail``
    names an intent prefix whose wait reports a failed receipt."""

    def __init__(self, fail=None):
        super().__init__()
        self.log, self.fail = [], fail

    def submit_transfer_intent(self, it):
        self.log.append(("submit", it.intent_id))
        return super().submit_transfer_intent(it)

    def wait_transfer_receipt(self, intent_id, timeout_seconds=None):
        self.log.append(("wait", intent_id))
        r = super().wait_transfer_receipt(intent_id, timeout_seconds)
        if self.fail and intent_id.startswith(self.fail):
            from dataclasses import replace

            r = replace(r, state=TransferStatusState.FAILED, bytes_completed=0, error="lane lost")
        return r


def adapter(client, layers=3):
    kv = caches(layers)
    cpu = [torch.zeros(2 * BLOCKS * UNIT, dtype=torch.uint8) for _ in range(layers)]
    groups = make_vllm_layer_groups_from_kv_caches(cpu, kv)
    assert [g.block_bytes for g in groups] == [UNIT] * layers and [g.layer_id for g in groups] == list(range(layers))
    return VllmKVSlotAdapter(client, ctx(WorkloadKind.KV_CACHE, metadata={"chunk_bytes": 4096}), groups), kv


def test_restore_submits_every_layer_before_waiting_and_groups_by_layer():
    c = Recording()
    ad, kv = adapter(c)
    refs = make_vllm_layer_range_refs_from_ids("req", [1, 2, 5], kv)
    handles = ad.restore_prefix(refs)
    kinds = [k for k, _ in c.log]
    assert kinds == ["submit"] * 3 + ["wait"] * 3, "all layers are in flight before the first wait"
    assert len(handles) == len(refs) and len(c.intents) == 3  # one handle per ref, one intent per layer
    for gid, it in enumerate(c.intents):
        assert it.direction == "h2d" and it.workload_kind == "kv_cache"
        assert it.metadata["group_id"] == gid and it.intent_id.startswith(f"a-g{gid}")
        assert it.total_bytes == 2 * 3 * UNIT and len(it.ranges) == 4  # 2 lanes x 2 runs


def test_save_moves_gpu_ranges_to_the_cpu_backing_layout():
    c = Recording()
    ad, kv = adapter(c, layers=1)
    refs = make_vllm_layer_range_refs_from_ids("req", [4, 5], kv)
    ad.save_prefix(refs)
    (it,) = c.intents
    assert it.direction == "d2h"
    lane = kv[0].stride(0) * 2
    got = sorted((r["src_offset"], r["dst_offset"], r["bytes"]) for r in it.ranges)
    assert got == [(4 * UNIT, 0, 2 * UNIT), (lane + 4 * UNIT, 2 * UNIT, 2 * UNIT)]


def test_transfer_stats_sum_over_groups_and_failures_surface():
    c = Recording()
    ad, kv = adapter(c, layers=2)
    refs = make_vllm_layer_range_refs_from_ids("req", [0, 1], kv)
    ad.restore_prefix(refs)
    st = ad.transfer_stats(refs)
    assert st.bytes == 2 * 2 * 2 * UNIT and st.relay_chunks == 2 * 2
    bad = Recording(fail="a-g1")
    ad2, kv2 = adapter(bad, layers=2)
    with pytest.raises(RuntimeError):
        ad2.restore_prefix(make_vllm_layer_range_refs_from_ids("req", [0], kv2))
    assert [k for k, _ in bad.log][:2] == ["submit", "submit"], "both layers were submitted before the failure"


def test_registering_the_same_refs_twice_is_idempotent():
    c = Recording()
    ad, kv = adapter(c, layers=1)
    refs = make_vllm_layer_range_refs_from_ids("req", [3], kv)
    assert ad.register_blocks(refs) == ad.register_blocks(refs)
    ad.restore_prefix(refs)
    ad.restore_prefix(refs)
    assert len(c.intents) == 2 and c.intents[0].ranges == c.intents[1].ranges
