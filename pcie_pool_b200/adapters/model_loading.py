"""Model-weight buckets loaded host->device as ``model_weights`` intents
(turbobus/adapters/model_loading.py:15-111)."""

from __future__ import annotations

from typing import Iterable

from ..offload_store import AdapterTransferContext, BlockState, BucketStoreMixin, OffloadBatch, OffloadStore


class ModelWeightLoader(BucketStoreMixin, OffloadStore):
    def __init__(self, client, transfer_context: AdapterTransferContext) -> None:
        super().__init__(client, transfer_context)

    def load_bucket(self, name: str):
        return self.prefetch(name)

    def load_buckets(self, names: Iterable[str]) -> list:
        return self.prefetch_many(names)

    def submit_load_buckets(self, names: Iterable[str]) -> OffloadBatch:
        return self.submit_prefetch_many(names)

    def load_batch(self, names: Iterable[str]) -> OffloadBatch:
        return self.submit_load_buckets(names)

    def load_all(self) -> list:
        return self.prefetch_many(self.names())

    def mark_unloaded(self, names: Iterable[str] | None = None) -> None:
        self._mark(names, BlockState.CPU)


ModelLoader = ModelWeightLoader

__all__ = ["ModelLoader", "ModelWeightLoader"]
