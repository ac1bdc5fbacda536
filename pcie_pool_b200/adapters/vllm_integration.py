"""Observe a running vLLM (V1) process without taking anything over.

Two vLLM methods are wrapped so that their results are also reported here:
``GPUModelRunner.initialize_kv_cache`` (the KV tensors, once they exist) and
``KVCacheManager.allocate_slots`` (every request's block ids, as vLLM hands
them out).  vLLM keeps scheduling and allocating; this module only records
what it sees and turns a request's blocks into the KV slot adapter's block
references.  The public surface (class names, methods, the
``_turbobus_integration`` class attribute) follows the reference's module
turbobus/adapters/vllm_integration.py so existing deployments keep working.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass, field
from itertools import zip_longest
from typing import Callable, Iterable

from ..offload_store import AdapterTransferContext, TransferIntentClient
from .vllm import (VllmKVBlockRef, VllmKVSlotAdapter, block_bytes_from_vllm_kv_tensor,
                   make_vllm_layer_block_refs_from_ids, make_vllm_layer_groups_from_kv_caches)

_HOOK_ATTR = "_turbobus_integration"


def _unique(ids: Iterable[int]) -> tuple[int, ...]:
    """Ids in first-seen order, each once."""
    return tuple(dict.fromkeys(ids))


@dataclass(frozen=True)
class VllmAllocationEvent:
    """Everything vLLM has allocated to one request so far, per KV cache
    group; ``event_count`` counts the allocations folded in."""

    request_id: str
    block_ids_by_group: tuple[tuple[int, ...], ...]
    event_count: int = 1

    @property
    def block_ids(self) -> tuple[int, ...]:
        return _unique(b for group in self.block_ids_by_group for b in group)

    def merge(self, other: "VllmAllocationEvent") -> "VllmAllocationEvent":
        """Fold a later allocation of the same request into this one."""
        if other.request_id != self.request_id:
            raise ValueError(f"allocation events of {self.request_id!r} and {other.request_id!r} do not merge")
        groups = tuple(_unique((*mine, *theirs)) for mine, theirs in
                       zip_longest(self.block_ids_by_group, other.block_ids_by_group, fillvalue=()))
        return VllmAllocationEvent(self.request_id, groups, self.event_count + other.event_count)


AllocationCallback = Callable[["VllmTurboBusIntegration", object, object, VllmAllocationEvent], None]


@dataclass
class VllmIntegrationState:
    kv_cache_config: object | None = None
    kv_caches: list[object] = field(default_factory=list)
    allocations: dict[str, VllmAllocationEvent] = field(default_factory=dict)
    adapter: VllmKVSlotAdapter | None = None


def _wrap_once(cls, method: str, report: Callable) -> None:
    """Replace ``cls.method`` (once) by a wrapper that calls the original and
    then ``report(integration, instance, args, kwargs, result)`` when an
    integration is attached to the instance's class."""
    saved = f"_turbobus_original_{method}"
    if hasattr(cls, saved):
        return
    original = getattr(cls, method)
    setattr(cls, saved, original)

    @functools.wraps(original)
    def hooked(obj, *args, **kwargs):
        result = original(obj, *args, **kwargs)
        integration = getattr(type(obj), _HOOK_ATTR, None)
        if integration is not None:
            report(integration, obj, args, kwargs, result)
        return result

    setattr(cls, method, hooked)


class VllmTurboBusIntegration:
    def __init__(self, client: TransferIntentClient, transfer_context: AdapterTransferContext,
                 cpu_backings: Iterable | None = None) -> None:
        self.client = client
        self.transfer_context = transfer_context
        self.state = VllmIntegrationState()
        self._cpu_backings = None if cpu_backings is None else list(cpu_backings)
        self._callback: AllocationCallback | None = None

    # ---- hooking ------------------------------------------------------------------------
    def install(self) -> None:
        from vllm.v1.core import kv_cache_manager
        from vllm.v1.worker import gpu_model_runner

        self.install_on_classes(gpu_model_runner.GPUModelRunner, kv_cache_manager.KVCacheManager)

    def install_on_classes(self, runner_cls, manager_cls) -> None:
        """Attach to these two classes; repeated installs wrap nothing twice."""
        for cls in (runner_cls, manager_cls):
            setattr(cls, _HOOK_ATTR, self)
        _wrap_once(runner_cls, "initialize_kv_cache",
                   lambda integ, runner, args, kw, _r: integ.bind_runner(runner, args[0] if args else
                                                                        kw.get("kv_cache_config")))
        _wrap_once(manager_cls, "allocate_slots",
                   lambda integ, _mgr, args, kw, blocks: integ.handle_allocation(
                       args[0] if args else kw.get("request"), blocks))

    # ---- what vLLM reports --------------------------------------------------------------------
    def bind_runner(self, runner, kv_cache_config=None) -> None:
        self.bind_kv_caches(list(getattr(runner, "kv_caches", None) or ()), kv_cache_config)

    def bind_kv_caches(self, kv_caches: Iterable, kv_cache_config=None) -> None:
        self.state.kv_cache_config = kv_cache_config
        self.state.kv_caches = list(kv_caches)
        self._rebuild_adapter()

    def record_allocation(self, request, blocks) -> VllmAllocationEvent | None:
        groups = extract_vllm_block_ids(blocks)
        if not groups:
            return None
        rid = str(getattr(request, "request_id", "unknown"))
        event = VllmAllocationEvent(rid, groups)
        if rid in self.state.allocations:
            event = self.state.allocations[rid].merge(event)
        self.state.allocations[rid] = event
        return event

    def handle_allocation(self, request, blocks) -> VllmAllocationEvent | None:
        event = self.record_allocation(request, blocks)
        if event is not None and self._callback is not None:
            self._callback(self, request, blocks, event)
        return event

    def set_allocation_callback(self, callback: AllocationCallback | None) -> None:
        self._callback = callback

    # ---- CPU side and transfers -----------------------------------------------------------------
    def set_cpu_backings(self, cpu_backings: Iterable) -> None:
        self._cpu_backings = list(cpu_backings)
        self._rebuild_adapter()

    def allocate_cpu_backings(self, slots_per_layer: int, *, pin_memory: bool = True) -> list:
        """One page-locked CPU backing per KV tensor, ``slots_per_layer`` units each."""
        import torch

        backings = [torch.empty(int(slots_per_layer) * block_bytes_from_vllm_kv_tensor(kv), dtype=torch.uint8,
                                pin_memory=pin_memory) for kv in self.state.kv_caches]
        self.set_cpu_backings(backings)
        return backings

    def block_ids_for_request(self, request_id: str) -> tuple[int, ...]:
        return self.state.allocations[str(request_id)].block_ids

    def make_refs_for_request(self, request_id: str, *, cpu_slot_start: int = 0) -> list[VllmKVBlockRef]:
        return make_vllm_layer_block_refs_from_ids(str(request_id), self.block_ids_for_request(request_id),
                                                   layer_count=len(self.state.kv_caches), cpu_slot_start=cpu_slot_start)

    def restore_request_prefix(self, request_id: str, *, cpu_slot_start: int = 0) -> list:
        refs = self.make_refs_for_request(request_id, cpu_slot_start=cpu_slot_start)
        return self.require_adapter().restore_prefix(refs)

    def save_request_prefix(self, request_id: str, *, cpu_slot_start: int = 0) -> list:
        refs = self.make_refs_for_request(request_id, cpu_slot_start=cpu_slot_start)
        return self.require_adapter().save_prefix(refs)

    def _rebuild_adapter(self) -> None:
        caches, backings = self.state.kv_caches, self._cpu_backings
        if not caches or backings is None:
            self.state.adapter = None
            return
        if len(backings) != len(caches):
            raise ValueError(f"{len(backings)} CPU backings for {len(caches)} vLLM KV cache tensors")
        self.state.adapter = VllmKVSlotAdapter(self.client, self.transfer_context,
                                               make_vllm_layer_groups_from_kv_caches(backings, caches))

    def require_adapter(self) -> VllmKVSlotAdapter:
        if self.state.adapter is None:
            raise RuntimeError("bind the vLLM KV caches and the CPU backings before saving or restoring")
        return self.state.adapter

    _require_adapter = require_adapter


def extract_vllm_block_ids(blocks) -> tuple[tuple[int, ...], ...]:
    """Block ids from a vLLM ``KVCacheBlocks`` (or plain ids / id groups)."""
    if blocks is None:
        return ()
    getter = getattr(blocks, "get_block_ids", None)
    if getter is None:
        return normalize_block_id_groups(getattr(blocks, "block_ids", blocks))
    try:
        return normalize_block_id_groups(getter(allow_none=True))
    except TypeError:  # older vLLM: no allow_none
        return normalize_block_id_groups(getter())


def _block_id(b) -> int:
    return int(getattr(b, "block_id", b))


def normalize_block_id_groups(raw) -> tuple[tuple[int, ...], ...]:
    """``ids``, ``[ids, ...]`` or ``[[block, ...], ...]`` -> tuple of id groups
    (``None`` entries dropped; a flat list is one group)."""
    if isinstance(raw, int):
        return ((raw,),)
    if not isinstance(raw, (tuple, list)):
        return ()
    if all(x is None or isinstance(x, int) for x in raw):
        flat = tuple(int(x) for x in raw if x is not None)
        return (flat,) if flat else ()
    groups = []
    for g in raw:
        if g is None:
            continue
        groups.append((int(g),) if isinstance(g, int) else tuple(_block_id(b) for b in g if b is not None))
    return tuple(groups)


__all__ = ["AllocationCallback", "VllmAllocationEvent", "VllmIntegrationState", "VllmTurboBusIntegration",
           "extract_vllm_block_ids", "normalize_block_id_groups"]
