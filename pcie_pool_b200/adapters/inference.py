"""Framework-neutral KV slots over one CPU backing and one GPU KV backing
(turbobus/adapters/inference.py:9-110)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable

from ..offload_store import AdapterTransferContext, OffloadBatch, OffloadStore, TransferStats


@dataclass(frozen=True)
class InferenceKVSlot:
    """One framework-owned KV block slot."""

    name: str
    block_id: object
    cpu_offset: int
    gpu_offset: int
    byte_count: int
    cpu_slot: object | None = None
    gpu_slot: object | None = None


class InferenceKVSlotAdapter(OffloadStore):
    """Register KV slots, then save (evict) or restore (prefetch) prefixes."""

    def __init__(self, client, transfer_context: AdapterTransferContext, cpu_backing, gpu_kv_backing) -> None:
        super().__init__(client, transfer_context)
        self.cpu_backing = cpu_backing
        self.gpu_kv_backing = gpu_kv_backing

    def register_slots(self, slots: Iterable[InferenceKVSlot]) -> None:
        for s in slots:
            self.add(s.name, self.cpu_backing, self.gpu_kv_backing, block_id=s.block_id, cpu_slot=s.cpu_slot,
                     gpu_slot=s.gpu_slot, cpu_offset=s.cpu_offset, gpu_offset=s.gpu_offset,
                     byte_count=s.byte_count)

    def submit_restore_prefix(self, names: Iterable[str]) -> tuple[list[str], list]:
        names = list(names)
        return names, self.prefetch_many(names)

    def submit_save_prefix(self, names: Iterable[str]) -> tuple[list[str], list]:
        names = list(names)
        return names, self.evict_many(names)

    def restore_prefix(self, names: Iterable[str]) -> list:
        names, handles = self.submit_restore_prefix(names)
        self.wait_prefix(names)
        return handles

    def save_prefix(self, names: Iterable[str]) -> list:
        names, handles = self.submit_save_prefix(names)
        self.wait_prefix(names)
        return handles

    def restore_batch(self, names: Iterable[str]) -> OffloadBatch:
        names = list(names)
        return OffloadBatch("restore", tuple(names), tuple(self.prefetch_many(names)), self)

    def save_batch(self, names: Iterable[str]) -> OffloadBatch:
        names = list(names)
        return OffloadBatch("save", tuple(names), tuple(self.evict_many(names)), self)

    def wait_prefix(self, names: Iterable[str]) -> None:
        self.wait_many(names)

    def transfer_stats(self, names: Iterable[str]) -> TransferStats:  # type: ignore[override]
        return self.transfer_stats_many(names)


def make_contiguous_kv_slots(prefix: str, count: int, block_bytes: int) -> list[InferenceKVSlot]:
    return [InferenceKVSlot(name=f"{prefix}{i}", block_id=i, cpu_slot=i, gpu_slot=i, cpu_offset=i * block_bytes,
                            gpu_offset=i * block_bytes, byte_count=block_bytes) for i in range(count)]


FrameworkKVSlot = InferenceKVSlot
FrameworkKVSlotAdapter = InferenceKVSlotAdapter

__all__ = ["FrameworkKVSlot", "FrameworkKVSlotAdapter", "InferenceKVSlot", "InferenceKVSlotAdapter",
           "make_contiguous_kv_slots"]
