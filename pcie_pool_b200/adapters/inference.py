"""KV slots of any inference framework over one CPU and one GPU backing.

A framework describes each KV block it may offload as a slot: a name, the
framework's block id, and where the block's bytes sit in the CPU backing and
in the GPU KV backing.  Saving a prefix moves its slots GPU -> CPU, restoring
moves them CPU -> GPU; slots that share both backings and have explicit sizes
travel as ONE multi-range intent through ``OffloadStore``.  Class and method
names follow the reference's framework adapter
(turbobus/adapters/inference.py:9-114) so connectors written for it work
unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable

from ..offload_store import AdapterTransferContext, OffloadBatch, OffloadStore, TransferStats

# adapter verb -> store operation
_STORE_OP = {"restore": "prefetch", "save": "evict"}


@dataclass(frozen=True)
class InferenceKVSlot:
    """One framework-owned KV block slot and its byte placement."""

    name: str
    block_id: object
    cpu_offset: int
    gpu_offset: int
    byte_count: int
    cpu_slot: object | None = None
    gpu_slot: object | None = None

    def placement(self) -> dict[str, object]:
        """Keyword arguments of ``OffloadStore.add`` for this slot."""
        return {"block_id": self.block_id, "cpu_slot": self.cpu_slot, "gpu_slot": self.gpu_slot,
                "cpu_offset": self.cpu_offset, "gpu_offset": self.gpu_offset, "byte_count": self.byte_count}


class InferenceKVSlotAdapter(OffloadStore):
    """Register a framework's KV slots, then save or restore prefixes of them."""

    def __init__(self, client, transfer_context: AdapterTransferContext, cpu_backing, gpu_kv_backing) -> None:
        super().__init__(client, transfer_context)
        self.cpu_backing = cpu_backing
        self.gpu_kv_backing = gpu_kv_backing

    def register_slots(self, slots: Iterable[InferenceKVSlot]) -> None:
        for slot in slots:
            self.add(slot.name, self.cpu_backing, self.gpu_kv_backing, **slot.placement())

    # -- one mechanism for both directions -------------------------------------------------
    def _batch(self, verb: str, names: Iterable[str]) -> OffloadBatch:
        b = self._submit_many(list(names), _STORE_OP[verb])
        return OffloadBatch(verb, b.names, b.handles, self)

    def _submit(self, verb: str, names: Iterable[str]) -> tuple[list[str], list]:
        b = self._batch(verb, names)
        return list(b.names), list(b.handles)

    def _run(self, verb: str, names: Iterable[str]) -> list:
        b = self._batch(verb, names)
        self.wait_many(b.names)
        return list(b.handles)

    # -- public verbs --------------------------------------------------------------------------
    def submit_restore_prefix(self, names: Iterable[str]) -> tuple[list[str], list]:
        return self._submit("restore", names)

    def submit_save_prefix(self, names: Iterable[str]) -> tuple[list[str], list]:
        return self._submit("save", names)

    def restore_prefix(self, names: Iterable[str]) -> list:
        return self._run("restore", names)

    def save_prefix(self, names: Iterable[str]) -> list:
        return self._run("save", names)

    def restore_batch(self, names: Iterable[str]) -> OffloadBatch:
        return self._batch("restore", names)

    def save_batch(self, names: Iterable[str]) -> OffloadBatch:
        return self._batch("save", names)

    def wait_prefix(self, names: Iterable[str]) -> None:
        self.wait_many(names)

    def transfer_stats(self, names: Iterable[str]) -> TransferStats:  # type: ignore[override]
        return self.transfer_stats_many(names)


def make_contiguous_kv_slots(prefix: str, count: int, block_bytes: int) -> list[InferenceKVSlot]:
    """``count`` slots of ``block_bytes`` laid out back to back in both backings."""
    return [InferenceKVSlot(f"{prefix}{i}", i, i * block_bytes, i * block_bytes, block_bytes, i, i)
            for i in range(count)]


FrameworkKVSlot = InferenceKVSlot
FrameworkKVSlotAdapter = InferenceKVSlotAdapter

__all__ = ["FrameworkKVSlot", "FrameworkKVSlotAdapter", "InferenceKVSlot", "InferenceKVSlotAdapter",
           "make_contiguous_kv_slots"]
