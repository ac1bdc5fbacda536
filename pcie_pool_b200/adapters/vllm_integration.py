"""Observation hooks for a running vLLM (V1) process.

``VllmTurboBusIntegration.install()`` wraps ``GPUModelRunner.initialize_kv_cache``
(to see the KV tensors) and ``KVCacheManager.allocate_slots`` (to see each
request's block ids); vLLM keeps owning scheduling and KV allocation.  The
observed tensors and ids feed the KV slot adapter (intent path) or the
paged-KV offloader (engine path).  API as turbobus/adapters/vllm_integration.py.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass, field
from typing import Callable, Iterable

from ..offload_store import AdapterTransferContext, TransferIntentClient
from .vllm import (VllmKVBlockRef, VllmKVSlotAdapter, block_bytes_from_vllm_kv_tensor,
                   make_vllm_layer_block_refs_from_ids, make_vllm_layer_groups_from_kv_caches)


def _dedup(ids: Iterable[int]) -> tuple[int, ...]:
    seen: set[int] = set()
    out = []
    for b in ids:
        if b not in seen:
            seen.add(b)
            out.append(b)
    return tuple(out)


@dataclass(frozen=True)
class VllmAllocationEvent:
    """Block ids vLLM allocated for one request, per KV cache group."""

    request_id: str
    block_ids_by_group: tuple[tuple[int, ...], ...]
    event_count: int = 1

    @property
    def block_ids(self) -> tuple[int, ...]:
        return _dedup(b for g in self.block_ids_by_group for b in g)

    def merge(self, other: "VllmAllocationEvent") -> "VllmAllocationEvent":
        if other.request_id != self.request_id:
            raise ValueError("cannot merge allocation events for different requests")
        n = max(len(self.block_ids_by_group), len(other.block_ids_by_group))

        def grp(ev, i):
            return ev.block_ids_by_group[i] if i < len(ev.block_ids_by_group) else ()

        return VllmAllocationEvent(self.request_id, tuple(_dedup((*grp(self, i), *grp(other, i))) for i in range(n)),
                                   event_count=self.event_count + other.event_count)


AllocationCallback = Callable[["VllmTurboBusIntegration", object, object, VllmAllocationEvent], None]


@dataclass
class VllmIntegrationState:
    kv_cache_config: object | None = None
    kv_caches: list[object] = field(default_factory=list)
    allocations: dict[str, VllmAllocationEvent] = field(default_factory=dict)
    adapter: VllmKVSlotAdapter | None = None


class VllmTurboBusIntegration:
    def __init__(self, client: TransferIntentClient, transfer_context: AdapterTransferContext,
                 cpu_backings: Iterable | None = None) -> None:
        self.client = client
        self.transfer_context = transfer_context
        self.state = VllmIntegrationState()
        self._cpu_backings = None if cpu_backings is None else list(cpu_backings)
        self._callback: AllocationCallback | None = None

    def install(self) -> None:
        from vllm.v1.core import kv_cache_manager as manager_module
        from vllm.v1.worker import gpu_model_runner as runner_module

        self.install_on_classes(runner_module.GPUModelRunner, manager_module.KVCacheManager)

    def install_on_classes(self, runner_cls, manager_cls) -> None:
        """Wrap the two hook points once per class (idempotent)."""
        runner_cls._turbobus_integration = self
        manager_cls._turbobus_integration = self
        if not hasattr(runner_cls, "_turbobus_original_initialize_kv_cache"):
            orig_init = runner_cls.initialize_kv_cache
            runner_cls._turbobus_original_initialize_kv_cache = orig_init

            @functools.wraps(orig_init)
            def initialize_kv_cache(runner, kv_cache_config, *a, **kw):
                out = orig_init(runner, kv_cache_config, *a, **kw)
                integ = getattr(type(runner), "_turbobus_integration", None)
                if integ is not None:
                    integ.bind_runner(runner, kv_cache_config)
                return out

            runner_cls.initialize_kv_cache = initialize_kv_cache
        if not hasattr(manager_cls, "_turbobus_original_allocate_slots"):
            orig_alloc = manager_cls.allocate_slots
            manager_cls._turbobus_original_allocate_slots = orig_alloc

            @functools.wraps(orig_alloc)
            def allocate_slots(manager, request, *a, **kw):
                out = orig_alloc(manager, request, *a, **kw)
                integ = getattr(type(manager), "_turbobus_integration", None)
                if integ is not None:
                    integ.handle_allocation(request, out)
                return out

            manager_cls.allocate_slots = allocate_slots

    def bind_runner(self, runner, kv_cache_config=None) -> None:
        self.bind_kv_caches(list(getattr(runner, "kv_caches", []) or []), kv_cache_config)

    def bind_kv_caches(self, kv_caches: Iterable, kv_cache_config=None) -> None:
        self.state.kv_cache_config = kv_cache_config
        self.state.kv_caches = list(kv_caches)
        self._refresh()

    def set_cpu_backings(self, cpu_backings: Iterable) -> None:
        self._cpu_backings = list(cpu_backings)
        self._refresh()

    def set_allocation_callback(self, callback: AllocationCallback | None) -> None:
        self._callback = callback

    def allocate_cpu_backings(self, slots_per_layer: int, *, pin_memory: bool = True) -> list:
        import torch

        b = [torch.empty(slots_per_layer * block_bytes_from_vllm_kv_tensor(kv), dtype=torch.uint8,
                         pin_memory=pin_memory) for kv in self.state.kv_caches]
        self.set_cpu_backings(b)
        return b

    def record_allocation(self, request, blocks) -> VllmAllocationEvent | None:
        rid = str(getattr(request, "request_id", "unknown"))
        groups = extract_vllm_block_ids(blocks)
        if not groups:
            return None
        ev = VllmAllocationEvent(rid, groups)
        prev = self.state.allocations.get(rid)
        if prev is not None:
            ev = prev.merge(ev)
        self.state.allocations[rid] = ev
        return ev

    def handle_allocation(self, request, blocks) -> VllmAllocationEvent | None:
        ev = self.record_allocation(request, blocks)
        if ev is not None and self._callback is not None:
            self._callback(self, request, blocks, ev)
        return ev

    def block_ids_for_request(self, request_id: str) -> tuple[int, ...]:
        return self.state.allocations[str(request_id)].block_ids

    def make_refs_for_request(self, request_id: str, *, cpu_slot_start: int = 0) -> list[VllmKVBlockRef]:
        return make_vllm_layer_block_refs_from_ids(str(request_id), self.block_ids_for_request(request_id),
                                                   layer_count=len(self.state.kv_caches),
                                                   cpu_slot_start=cpu_slot_start)

    def restore_request_prefix(self, request_id: str, *, cpu_slot_start: int = 0) -> list:
        return self.require_adapter().restore_prefix(self.make_refs_for_request(request_id, cpu_slot_start=cpu_slot_start))

    def save_request_prefix(self, request_id: str, *, cpu_slot_start: int = 0) -> list:
        return self.require_adapter().save_prefix(self.make_refs_for_request(request_id, cpu_slot_start=cpu_slot_start))

    def _refresh(self) -> None:
        if not self.state.kv_caches or self._cpu_backings is None:
            self.state.adapter = None
            return
        if len(self._cpu_backings) != len(self.state.kv_caches):
            raise ValueError("cpu_backings must match the number of vLLM KV cache tensors")
        self.state.adapter = VllmKVSlotAdapter(self.client, self.transfer_context,
                                               make_vllm_layer_groups_from_kv_caches(self._cpu_backings,
                                                                                     self.state.kv_caches))

    def require_adapter(self) -> VllmKVSlotAdapter:
        if self.state.adapter is None:
            raise RuntimeError("vLLM KV caches and CPU backings must be bound before restore/save")
        return self.state.adapter

    _require_adapter = require_adapter


def extract_vllm_block_ids(blocks) -> tuple[tuple[int, ...], ...]:
    """Block ids from a vLLM ``KVCacheBlocks`` (or ids / groups of ids)."""
    if blocks is None:
        return ()
    get = getattr(blocks, "get_block_ids", None)
    if get is None:
        raw = getattr(blocks, "block_ids", blocks)
    else:
        try:
            raw = get(allow_none=True)
        except TypeError:
            raw = get()
    return normalize_block_id_groups(raw)


def normalize_block_id_groups(raw) -> tuple[tuple[int, ...], ...]:
    if raw is None:
        return ()
    if isinstance(raw, (tuple, list)):
        if all(isinstance(x, int) or x is None for x in raw):
            ids = tuple(int(x) for x in raw if x is not None)
            return (ids,) if ids else ()
        groups = []
        for g in raw:
            if g is None:
                continue
            if isinstance(g, int):
                groups.append((int(g),))
                continue
            ids = []
            for b in g:
                if b is None:
                    continue
                ids.append(int(getattr(b, "block_id", b)))
            groups.append(tuple(ids))
        return tuple(groups)
    if isinstance(raw, int):
        return ((int(raw),),)
    return ()


__all__ = ["AllocationCallback", "VllmAllocationEvent", "VllmIntegrationState", "VllmTurboBusIntegration",
           "extract_vllm_block_ids", "normalize_block_id_groups"]
