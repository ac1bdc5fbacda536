"""Parameter / optimizer-state buckets: prefetch (H2D) and offload (D2H)
(turbobus/adapters/training_offload.py:15-131)."""

from __future__ import annotations

from typing import Iterable

from ..offload_store import AdapterTransferContext, BlockState, BucketStoreMixin, OffloadBatch, OffloadStore


class TrainingOffloadManager(BucketStoreMixin, OffloadStore):
    def __init__(self, client, transfer_context: AdapterTransferContext) -> None:
        super().__init__(client, transfer_context)

    def prefetch_bucket(self, name: str):
        return self.prefetch(name)

    def prefetch_buckets(self, names: Iterable[str]) -> list:
        return self.prefetch_many(names)

    def submit_prefetch_buckets(self, names: Iterable[str]) -> OffloadBatch:
        return self.submit_prefetch_many(names)

    def prefetch_batch(self, names: Iterable[str]) -> OffloadBatch:
        return self.submit_prefetch_buckets(names)

    def prefetch_all(self) -> list:
        return self.prefetch_buckets(self.names())

    def offload_bucket(self, name: str):
        return self.evict(name)

    def offload_buckets(self, names: Iterable[str]) -> list:
        return self.evict_many(names)

    def submit_offload_buckets(self, names: Iterable[str]) -> OffloadBatch:
        return self.submit_evict_many(names)

    def offload_batch(self, names: Iterable[str]) -> OffloadBatch:
        return self.submit_offload_buckets(names)

    def offload_all(self) -> list:
        return self.evict_many(self.names())

    def mark_on_cpu(self, names: Iterable[str] | None = None) -> None:
        self._mark(names, BlockState.CPU)

    def mark_on_gpu(self, names: Iterable[str] | None = None) -> None:
        self._mark(names, BlockState.GPU)


TrainingOffloadStore = TrainingOffloadManager

__all__ = ["TrainingOffloadManager", "TrainingOffloadStore"]
