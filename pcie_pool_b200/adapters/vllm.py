"""vLLM KV-cache block mapping.

vLLM keeps one KV tensor per attention layer shaped ``[2, num_blocks, block,
heads, dim]``: K and V are separate "lanes" in dimension 0 and the block id
is dimension 1, so one logical block is two byte ranges
(``lane * stride(0) + block * stride(1)``).  On the CPU side a saved prefix of
``n`` blocks is laid out ``[K blocks 0..n-1][V blocks 0..n-1]``, i.e. CPU
slot ``start + lane * n + index`` (turbobus/adapters/vllm.py:258-304).

``block_table_units`` is new: instead of coalescing ranges per contiguous run
(a permuted block table coalesces nothing: 131,072 ranges of 32 KiB per 32k-
token request), it returns the per-unit device address table the fused
landing kernel scatters through, so a whole request moves as a few large
host-contiguous chunks.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from collections.abc import Mapping
from typing import Iterable

import numpy as np

from ..offload_store import AdapterTransferContext, TransferStats
from .inference import InferenceKVSlot, InferenceKVSlotAdapter


@dataclass(frozen=True)
class VllmKVBlockRef:
    """One vLLM KV block mapped to saved CPU backing and a GPU KV slot."""

    request_id: str
    group_id: int
    block_id: int
    cpu_slot: int
    gpu_slot: int
    lane_id: int | None = None
    cpu_offset: int | None = None
    gpu_offset: int | None = None
    byte_count: int | None = None


@dataclass(frozen=True)
class VllmKVGroup:
    """KV backing tensors and block size of one KV cache group (one layer)."""

    group_id: int
    cpu_backing: object
    gpu_kv_backing: object
    block_bytes: int
    layer_id: int | None = None


def _group_context(ctx: AdapterTransferContext, gid: int) -> AdapterTransferContext:
    return AdapterTransferContext(job_id=ctx.job_id, session_id=ctx.session_id, cpu_buffer_id=ctx.cpu_buffer_id,
                                  gpu_buffer_id=ctx.gpu_buffer_id, workload_kind=ctx.workload_kind,
                                  priority=ctx.priority, policy_hints=ctx.policy_hints,
                                  metadata={**ctx.metadata, "group_id": int(gid)},
                                  intent_prefix=f"{ctx.intent_prefix}-g{int(gid)}",
                                  wait_timeout_seconds=ctx.wait_timeout_seconds)


class VllmKVSlotAdapter:
    """vLLM-shaped wrapper: one ``InferenceKVSlotAdapter`` per KV group."""

    def __init__(self, client, transfer_context: AdapterTransferContext, groups: Iterable[VllmKVGroup]) -> None:
        self.client = client
        self.transfer_context = transfer_context
        self.groups: dict[int, VllmKVGroup] = {g.group_id: g for g in groups}
        self.adapters = {gid: InferenceKVSlotAdapter(client, _group_context(transfer_context, gid), g.cpu_backing,
                                                     g.gpu_kv_backing) for gid, g in self.groups.items()}
        self._registered: set[str] = set()

    def register_blocks(self, refs: Iterable[VllmKVBlockRef]) -> list[str]:
        by_group: dict[int, list[InferenceKVSlot]] = {}
        names = []
        for r in refs:
            g = self.groups[r.group_id]
            name = vllm_block_name(r)
            names.append(name)
            if name in self._registered:
                continue
            by_group.setdefault(r.group_id, []).append(InferenceKVSlot(
                name=name, block_id=(r.request_id, r.group_id, r.block_id), cpu_slot=r.cpu_slot,
                gpu_slot=r.gpu_slot,
                cpu_offset=r.cpu_offset if r.cpu_offset is not None else r.cpu_slot * g.block_bytes,
                gpu_offset=r.gpu_offset if r.gpu_offset is not None else r.gpu_slot * g.block_bytes,
                byte_count=r.byte_count if r.byte_count is not None else g.block_bytes))
        for gid, slots in by_group.items():
            self.adapters[gid].register_slots(slots)
            self._registered.update(s.name for s in slots)
        return names

    def restore_prefix(self, refs: Iterable[VllmKVBlockRef]) -> list:
        return self._transfer(refs, "restore")

    def save_prefix(self, refs: Iterable[VllmKVBlockRef]) -> list:
        return self._transfer(refs, "save")

    def transfer_stats(self, refs: Iterable[VllmKVBlockRef]) -> TransferStats:
        tot = TransferStats()
        for gid, names in self._group_names(refs).items():
            s = self.adapters[gid].transfer_stats(names)
            tot = TransferStats(tot.bytes + s.bytes, tot.direct_chunks + s.direct_chunks,
                                tot.relay_chunks + s.relay_chunks)
        return tot

    def _transfer(self, refs: Iterable[VllmKVBlockRef], op: str) -> list:
        method = "submit_restore_prefix" if op == "restore" else "submit_save_prefix"
        handles, submitted = [], []
        for gid, names in self._group_names(refs).items():
            names, hs = getattr(self.adapters[gid], method)(names)
            submitted.append((gid, names))
            handles.extend(hs)
        for gid, names in submitted:
            self.adapters[gid].wait_prefix(names)
        return handles

    def _group_names(self, refs: Iterable[VllmKVBlockRef]) -> Mapping[int, list[str]]:
        refs = list(refs)
        self.register_blocks(refs)
        out: dict[int, list[str]] = {}
        for r in refs:
            out.setdefault(r.group_id, []).append(vllm_block_name(r))
        return out

    def _batch_size(self, refs: Iterable[VllmKVBlockRef]) -> tuple[int, int]:
        chunk = max(1, int(self.transfer_context.metadata.get("chunk_bytes", 16 << 20)))
        total = chunks = 0
        for r in refs:
            n = int(r.byte_count if r.byte_count is not None else self.groups[r.group_id].block_bytes)
            total += n
            chunks += max(1, math.ceil(n / chunk))
        return total, chunks


def vllm_block_name(ref: VllmKVBlockRef) -> str:
    lane = "" if ref.lane_id is None else f":l{ref.lane_id}"
    nbytes = "" if ref.byte_count is None else f":bytes{ref.byte_count}"
    return f"{ref.request_id}:g{ref.group_id}:b{ref.block_id}{lane}{nbytes}"


def make_vllm_block_refs_from_ids(request_id: str, group_id: int, block_ids: Iterable[int],
                                  cpu_slot_start: int = 0) -> list[VllmKVBlockRef]:
    return [VllmKVBlockRef(request_id, group_id, int(b), cpu_slot_start + i, int(b))
            for i, b in enumerate(block_ids)]


def block_bytes_from_vllm_kv_tensor(tensor) -> int:
    """Bytes of one addressable KV unit: one block of one K/V plane for
    ``[2, blocks, ...]`` tensors (``stride(1)``, as turbobus/adapters/vllm.py:
    206-211 computes it), the whole block for ``[blocks, ...]`` layouts."""
    return kv_layout(tensor).unit_bytes


def make_vllm_layer_groups_from_kv_caches(cpu_backings: Iterable, kv_caches: Iterable, *,
                                          group_id_start: int = 0) -> list[VllmKVGroup]:
    return [VllmKVGroup(group_id=group_id_start + i, layer_id=i, cpu_backing=c, gpu_kv_backing=kv,
                        block_bytes=block_bytes_from_vllm_kv_tensor(kv))
            for i, (c, kv) in enumerate(zip(cpu_backings, kv_caches))]


def make_vllm_layer_block_refs_from_ids(request_id: str, block_ids: Iterable[int], layer_count: int,
                                        cpu_slot_start: int = 0) -> list[VllmKVBlockRef]:
    ids = [int(b) for b in block_ids]
    return [VllmKVBlockRef(request_id, layer, b, cpu_slot_start + i, b)
            for layer in range(layer_count) for i, b in enumerate(ids)]


def contiguous_runs(block_ids: list[int]) -> list[tuple[int, list[int]]]:
    """(start index, run) for each maximal run of consecutive block ids."""
    runs: list[tuple[int, list[int]]] = []
    for i, b in enumerate(block_ids):
        if runs and b == runs[-1][1][-1] + 1:
            runs[-1][1].append(b)
        else:
            runs.append((i, [b]))
    return runs


def make_vllm_layer_range_refs_from_ids(request_id: str, block_ids: Iterable[int], kv_caches: Iterable,
                                        cpu_slot_start: int = 0) -> list[VllmKVBlockRef]:
    """Byte-range refs: one ref per K/V lane (``[2, blocks, ...]``) or per
    block (``[blocks, ...]``) for each contiguous run of block ids, in the
    CPU backing order ``[lane][index]``."""
    ids = [int(b) for b in block_ids]
    refs = []
    for layer, kv in enumerate(kv_caches):
        lay = kv_layout(kv)
        bb = lay.unit_bytes
        for lane in range(lay.lanes):
            for start, run in contiguous_runs(ids):
                slot = cpu_slot_start + lane * len(ids) + start
                goff = lane * lay.lane_stride + run[0] * lay.block_stride
                refs.append(VllmKVBlockRef(request_id, layer, run[0], slot, run[0],
                                           None if lay.lanes == 1 else lane, slot * bb, int(goff), len(run) * bb))
    return refs


@dataclass(frozen=True)
class KVLayout:
    """How one layer's KV tensor addresses a block: ``lanes`` units per block
    (2 when K and V are separate planes), the byte strides between lanes and
    between blocks, and the bytes of one unit."""

    lanes: int
    lane_stride: int
    block_stride: int
    unit_bytes: int
    num_blocks: int


def kv_layout(kv) -> KVLayout:
    """Layout of a vLLM KV cache tensor.  ``[2, num_blocks, ...]`` (K and V
    planes, e.g. the FlashAttention backend) has two units per block;
    ``[num_blocks, 2, ...]`` (K and V adjacent inside a block, e.g. FlashInfer)
    and ``[num_blocks, ...]`` have one unit covering the whole block."""
    es = kv.element_size()
    shape = tuple(int(d) for d in kv.shape)
    if len(shape) >= 3 and shape[0] == 2 and shape[1] != 2:
        return KVLayout(2, kv.stride(0) * es, kv.stride(1) * es, kv.stride(1) * es, shape[1])
    if len(shape) < 2:
        raise ValueError("vLLM KV tensor must have at least two dimensions")
    return KVLayout(1, 0, kv.stride(0) * es, kv.stride(0) * es, shape[0])


def block_table_units(kv_caches: Iterable, block_ids: Iterable[int]) -> tuple[np.ndarray, int]:
    """Device address of every (layer, lane, block) unit of a request in the
    CPU backing order [layer][lane][index] -> (uint64 addresses, unit bytes).

    The landing kernel scatters a host-contiguous chunk of units through this
    table (paged-KV reload) and the push kernel gathers through it (offload).
    """
    ids = np.asarray(list(block_ids), dtype=np.int64)
    out, unit = [], None
    for kv in kv_caches:
        lay = kv_layout(kv)
        if unit is None:
            unit = lay.unit_bytes
        elif lay.unit_bytes != unit:
            raise ValueError("all layers must share one block size")
        base = int(kv.data_ptr())
        for lane in range(lay.lanes):
            out.append(base + lane * lay.lane_stride + ids * lay.block_stride)
    if unit is None:
        raise ValueError("no KV caches given")
    return np.concatenate(out).astype(np.uint64), int(unit)


block_name = vllm_block_name
make_block_refs_from_ids = make_vllm_block_refs_from_ids
make_layer_groups_from_kv_caches = make_vllm_layer_groups_from_kv_caches
make_layer_block_refs_from_ids = make_vllm_layer_block_refs_from_ids
make_layer_range_refs_from_ids = make_vllm_layer_range_refs_from_ids

__all__ = ["VllmKVBlockRef", "VllmKVGroup", "VllmKVSlotAdapter", "block_bytes_from_vllm_kv_tensor",
           "KVLayout", "block_table_units", "contiguous_runs", "kv_layout", "make_vllm_block_refs_from_ids",
           "make_vllm_layer_block_refs_from_ids", "make_vllm_layer_groups_from_kv_caches",
           "make_vllm_layer_range_refs_from_ids", "vllm_block_name"]
