"""Named CPU<->GPU blocks over daemon transfer intents.

A block is a byte range of a CPU backing and a GPU backing.  ``prefetch``
moves it host->device, ``evict`` device->host.  Blocks that share both
backings and carry explicit byte counts travel as ONE multi-range intent;
other blocks get one intent each.  Every intent returns a
``ReceiptTransferHandle``; waiting on it raises on a failed or canceled
receipt and flips the block state (cpu / prefetching / gpu / evicting).
API and semantics follow turbobus/offload_store.py:284-612.
"""

from __future__ import annotations

import uuid
from dataclasses import dataclass, field
from enum import Enum
from collections.abc import Mapping
from typing import Iterable, Protocol

from .schema import (FORBIDDEN_POLICY_KEYS, TERMINAL_STATES, TransferIntent, TransferReceipt, TransferStatusState,
                     WorkloadKind)


class BlockState(str, Enum):
    CPU = "cpu"
    GPU = "gpu"
    PREFETCHING = "prefetching"
    EVICTING = "evicting"
    UNKNOWN = "unknown"


OPERATIONS = {"prefetch": ("h2d", BlockState.PREFETCHING, BlockState.GPU),
              "evict": ("d2h", BlockState.EVICTING, BlockState.CPU)}


@dataclass(frozen=True)
class TransferStats:
    """Bytes and chunk counts of one or more transfers, split by path kind.
    Stats add, so a batch's figure is the sum of its transfers'."""

    bytes: int = 0
    direct_chunks: int = 0
    relay_chunks: int = 0

    def __add__(self, other: "TransferStats") -> "TransferStats":
        return TransferStats(self.bytes + other.bytes, self.direct_chunks + other.direct_chunks,
                             self.relay_chunks + other.relay_chunks)

    @classmethod
    def of_path(cls, path: Mapping[str, object]) -> "TransferStats":
        """One receipt path record (``kind``, ``bytes``, ``chunk_count``)."""
        nbytes = int(path.get("bytes", 0) or 0)
        chunks = int(path.get("chunk_count", path.get("chunks", 0)) or 0)
        relay = str(path.get("kind", "")).lower() == "relay"
        return cls(nbytes, 0 if relay else chunks, chunks if relay else 0)

    @classmethod
    def coerce(cls, value) -> "TransferStats":
        """A stats object, mapping or anything with the three attributes."""
        if isinstance(value, TransferStats):
            return value
        get = value.get if isinstance(value, Mapping) else (lambda k, d=0: getattr(value, k, d))
        return cls(*(int(get(k, 0) or 0) for k in ("bytes", "direct_chunks", "relay_chunks")))

    def as_dict(self) -> dict[str, int]:
        return {"bytes": self.bytes, "direct_chunks": self.direct_chunks, "relay_chunks": self.relay_chunks}


class TransferIntentClient(Protocol):
    def submit_transfer_intent(self, intent: TransferIntent) -> TransferReceipt:
        ...

    def wait_transfer_receipt(self, intent_id: str, timeout_seconds: float | None = None) -> TransferReceipt:
        ...


def check_policy_hints(hints: Mapping[str, object]) -> dict[str, object]:
    """Adapters state intent, not routing: hints naming relays, lanes or
    paths are refused (the daemon alone chooses physical paths)."""
    h = dict(hints)
    routing = sorted(k for k in map(str, h) if k.lower() in FORBIDDEN_POLICY_KEYS)
    if routing:
        raise ValueError(f"policy_hints may not pick physical paths ({', '.join(routing)}); the daemon does")
    return h


def _text(name: str):
    def norm(v) -> str:
        if not str(v).strip():
            raise ValueError(f"AdapterTransferContext.{name} must be non-empty")
        return str(v)
    return norm


def _timeout(v):
    if v is None:
        return None
    t = float(v)
    if t < 0:
        raise ValueError(f"wait_timeout_seconds must be non-negative, got {t}")
    return t


@dataclass(frozen=True)
class AdapterTransferContext:
    """What every intent of one adapter shares: job, session, the CPU and GPU
    backing buffers, workload class, priority, hints, metadata, the intent-id
    prefix and the wait timeout."""

    job_id: str
    session_id: str
    cpu_buffer_id: str
    gpu_buffer_id: str
    workload_kind: WorkloadKind | str = WorkloadKind.GENERIC
    priority: int = 0
    policy_hints: Mapping[str, object] = field(default_factory=dict)
    metadata: Mapping[str, object] = field(default_factory=dict)
    intent_prefix: str | None = None
    wait_timeout_seconds: float | None = None

    _NORMALIZE = {
        "job_id": _text("job_id"), "session_id": _text("session_id"),
        "cpu_buffer_id": _text("cpu_buffer_id"), "gpu_buffer_id": _text("gpu_buffer_id"),
        "workload_kind": WorkloadKind, "priority": int, "policy_hints": check_policy_hints,
        "metadata": dict, "wait_timeout_seconds": _timeout,
        "intent_prefix": lambda v: _text("intent_prefix")(v or f"adapter-{uuid.uuid4()}"),
    }

    def __post_init__(self) -> None:
        for name, norm in self._NORMALIZE.items():
            object.__setattr__(self, name, norm(getattr(self, name)))


def transfer_stats_from_receipt(receipt: TransferReceipt) -> TransferStats:
    return sum((TransferStats.of_path(p) for p in receipt.path_stats), TransferStats())


def summarize_transfer_handles(handles: Iterable) -> TransferStats:
    """Stats of distinct handles (a handle shared by several blocks counts once)."""
    distinct = {id(h): h for h in handles if getattr(h, "stats", None) is not None}
    return sum((TransferStats.coerce(h.stats) for h in distinct.values()), TransferStats())


_FAILED = (TransferStatusState.FAILED, TransferStatusState.CANCELED)


@dataclass
class ReceiptTransferHandle:
    """The receipt of one submitted intent.  ``wait`` asks the daemon until it
    sees a terminal receipt, then answers from it; a failed or canceled
    transfer raises."""

    client: TransferIntentClient
    intent: TransferIntent
    receipt: TransferReceipt
    wait_timeout_seconds: float | None = None
    wait_calls: int = 0
    _final: TransferReceipt | None = field(default=None, init=False, repr=False)

    @property
    def stats(self) -> TransferStats:
        return transfer_stats_from_receipt(self.receipt)

    @property
    def done(self) -> bool:
        return self._final is not None

    def _accept(self, r) -> TransferReceipt:
        if not isinstance(r, TransferReceipt):
            raise TypeError(f"the daemon client returned {type(r).__name__}, not a TransferReceipt")
        if r.intent_id != self.intent.intent_id:
            raise ValueError(f"receipt for {r.intent_id!r} does not match intent {self.intent.intent_id!r}")
        return r

    def wait(self) -> TransferReceipt:
        if self._final is not None:
            return self._final
        r = self._accept(self.client.wait_transfer_receipt(self.intent.intent_id,
                                                           timeout_seconds=self.wait_timeout_seconds))
        self.receipt = r
        self.wait_calls += 1
        state = TransferStatusState(r.state)
        if state in TERMINAL_STATES:  # a timed-out wait may still return a live receipt
            self._final = r
        if state in _FAILED:
            raise RuntimeError(r.error or f"transfer {self.intent.intent_id} {state.value}")
        return r


@dataclass(frozen=True)
class OffloadBlockInfo:
    name: str
    block_id: object
    cpu_slot: object | None
    gpu_slot: object | None
    cpu_offset: int
    gpu_offset: int
    bytes: int
    state: BlockState
    last_operation: str | None
    transfer_stats: TransferStats | None

    def as_dict(self) -> dict[str, object]:
        return {"name": self.name, "block_id": self.block_id, "cpu_slot": self.cpu_slot,
                "gpu_slot": self.gpu_slot, "cpu_offset": self.cpu_offset, "gpu_offset": self.gpu_offset,
                "bytes": self.bytes, "state": self.state.value, "last_operation": self.last_operation,
                "transfer_stats": None if self.transfer_stats is None else self.transfer_stats.as_dict()}


@dataclass(frozen=True)
class OffloadBatch:
    operation: str
    names: tuple[str, ...]
    handles: tuple[object, ...]
    store: "OffloadStore" = field(repr=False, compare=False)

    def wait(self) -> None:
        self.store.wait_many(self.names)

    def transfer_stats(self) -> TransferStats:
        return self.store.transfer_stats_many(self.names)

    def block_infos(self) -> list[OffloadBlockInfo]:
        return self.store.block_infos(self.names)

    def as_dict(self) -> dict[str, object]:
        return {"operation": self.operation, "names": list(self.names),
                "transfer_stats": self.transfer_stats().as_dict(),
                "blocks": [i.as_dict() for i in self.block_infos()]}


@dataclass
class OffloadBlock:
    name: str
    cpu_tensor: object
    gpu_tensor: object
    block_id: object | None = None
    cpu_slot: object | None = None
    gpu_slot: object | None = None
    cpu_offset: int = 0
    gpu_offset: int = 0
    byte_count: int | None = None
    state: BlockState = BlockState.CPU
    last_prefetch: object | None = None
    last_evict: object | None = None
    last_handle: object | None = None
    last_operation: str | None = None

    def __post_init__(self) -> None:
        if self.block_id is None:
            self.block_id = self.name

    @property
    def bytes(self) -> int:
        if self.byte_count is not None:
            return int(self.byte_count)
        return int(self.cpu_tensor.numel() * self.cpu_tensor.element_size())

    @property
    def last_stats(self):
        return None if self.last_handle is None else self.last_handle.stats

    @property
    def last_transfer_stats(self) -> TransferStats | None:
        return None if self.last_handle is None else summarize_transfer_handles([self.last_handle])

    def info(self) -> OffloadBlockInfo:
        return OffloadBlockInfo(self.name, self.block_id, self.cpu_slot, self.gpu_slot, self.cpu_offset,
                                self.gpu_offset, self.bytes, self.state, self.last_operation,
                                self.last_transfer_stats)


class OffloadStore:
    """Connector-shaped named-block layer over daemon transfer intents."""

    def __init__(self, client: TransferIntentClient, transfer_context: AdapterTransferContext) -> None:
        if not isinstance(transfer_context, AdapterTransferContext):
            raise TypeError("transfer_context must be an AdapterTransferContext")
        self.client = client
        self.transfer_context = transfer_context
        self._blocks: dict[str, OffloadBlock] = {}
        self._intent_counter = 0

    # -- registry ---------------------------------------------------------------------------
    def add(self, name: str, cpu_tensor, gpu_tensor=None, *, block_id=None, cpu_slot=None, gpu_slot=None,
            cpu_offset: int = 0, gpu_offset: int = 0, byte_count: int | None = None) -> OffloadBlock:
        if not isinstance(name, str) or not name:
            raise ValueError("offload block name must be a non-empty string")
        if cpu_offset < 0 or gpu_offset < 0:
            raise ValueError("block offsets must be non-negative")
        if byte_count is not None and byte_count <= 0:
            raise ValueError("byte_count must be positive")
        if name in self._blocks:
            raise ValueError(f"offload block already exists: {name}")
        b = OffloadBlock(name, cpu_tensor, object() if gpu_tensor is None else gpu_tensor, block_id=block_id,
                         cpu_slot=cpu_slot, gpu_slot=gpu_slot, cpu_offset=int(cpu_offset),
                         gpu_offset=int(gpu_offset), byte_count=None if byte_count is None else int(byte_count))
        self._blocks[name] = b
        return b

    add_block = add

    def remove(self, name: str) -> OffloadBlock:
        return self._blocks.pop(name)

    remove_block = remove

    def block(self, name: str) -> OffloadBlock:
        try:
            return self._blocks[name]
        except KeyError as exc:
            raise KeyError(f"unknown offload block: {name}") from exc

    get_block = block

    def names(self) -> list[str]:
        return list(self._blocks)

    def block_ids(self) -> list[object]:
        return [b.block_id for b in self._blocks.values()]

    def blocks(self) -> Iterable[OffloadBlock]:
        return self._blocks.values()

    def block_info(self, name: str) -> OffloadBlockInfo:
        return self.block(name).info()

    def block_infos(self, names: Iterable[str] | None = None) -> list[OffloadBlockInfo]:
        return [b.info() for b in (self._blocks.values() if names is None else map(self.block, names))]

    # -- movement ------------------------------------------------------------------------------
    def prefetch(self, name: str):
        return self.submit_prefetch_many([name]).handles[0]

    def evict(self, name: str):
        return self.submit_evict_many([name]).handles[0]

    def prefetch_many(self, names: Iterable[str]) -> list:
        return list(self.submit_prefetch_many(names).handles)

    def evict_many(self, names: Iterable[str]) -> list:
        return list(self.submit_evict_many(names).handles)

    def submit_prefetch_many(self, names: Iterable[str]) -> OffloadBatch:
        return self._submit_many(names, "prefetch")

    def submit_evict_many(self, names: Iterable[str]) -> OffloadBatch:
        return self._submit_many(names, "evict")

    def _submit_many(self, names: Iterable[str], op: str) -> OffloadBatch:
        if op not in OPERATIONS:
            raise ValueError(f"unknown offload operation: {op}")
        blocks = [self.block(n) for n in names]
        if not blocks:
            return OffloadBatch(op, (), (), self)
        in_flight = OPERATIONS[op][1]
        if self._batchable(blocks):
            h = self._submit_transfer(blocks, op, self._ranges(blocks, op))
            handles = tuple(h for _ in blocks)
            self._record(blocks, h, op, in_flight)
        else:
            handles = tuple(self._submit_transfer([b], op, self._ranges([b], op)) for b in blocks)
            for b, h in zip(blocks, handles):
                self._record([b], h, op, in_flight)
        return OffloadBatch(op, tuple(b.name for b in blocks), handles, self)

    def wait(self, name: str) -> None:
        b = self.block(name)
        if b.last_handle is None:
            return
        b.last_handle.wait()
        self._settle(b)

    def wait_many(self, names: Iterable[str]) -> None:
        """Wait for the blocks' last transfers (a shared batch handle once) and
        move each to where its transfer put it; a block that never moved
        keeps its state, as with :meth:`wait`."""
        done = set()
        for n in names:
            b = self.block(n)
            if b.last_handle is None:
                continue
            if id(b.last_handle) not in done:
                b.last_handle.wait()
                done.add(id(b.last_handle))
            self._settle(b)

    def stats(self, name: str):
        return self.block(name).last_stats

    def transfer_stats(self, name: str) -> TransferStats | None:
        return self.block(name).last_transfer_stats

    def transfer_stats_many(self, names: Iterable[str]) -> TransferStats:
        return summarize_transfer_handles(b.last_handle for b in map(self.block, names) if b.last_handle is not None)

    def set_block_state(self, name: str, state: BlockState, *, clear_transfer_state: bool = False) -> OffloadBlock:
        b = self.block(name)
        b.state = state
        if clear_transfer_state:
            self.clear_block_transfer_state(name)
        return b

    def clear_block_transfer_state(self, name: str) -> OffloadBlock:
        b = self.block(name)
        b.last_prefetch = b.last_evict = b.last_handle = None
        b.last_operation = None
        return b

    # -- internals --------------------------------------------------------------------------------
    @staticmethod
    def _settle(b: OffloadBlock) -> None:
        b.state = OPERATIONS[b.last_operation][2] if b.last_operation in OPERATIONS else BlockState.UNKNOWN

    @staticmethod
    def _batchable(blocks: list[OffloadBlock]) -> bool:
        first = blocks[0]
        return first.byte_count is not None and all(
            b.cpu_tensor is first.cpu_tensor and b.gpu_tensor is first.gpu_tensor and b.byte_count is not None
            for b in blocks)

    @staticmethod
    def _ranges(blocks: list[OffloadBlock], op: str) -> list[dict]:
        h2d = OPERATIONS[op][0] == "h2d"
        return [{"src_offset": b.cpu_offset if h2d else b.gpu_offset,
                 "dst_offset": b.gpu_offset if h2d else b.cpu_offset, "bytes": b.bytes} for b in blocks]

    @staticmethod
    def _record(blocks: list[OffloadBlock], handle, op: str, state: BlockState) -> None:
        for b in blocks:
            if op == "prefetch":
                b.last_prefetch = handle
            else:
                b.last_evict = handle
            b.last_handle, b.last_operation, b.state = handle, op, state

    def _submit_transfer(self, blocks: list[OffloadBlock], op: str, ranges) -> ReceiptTransferHandle:
        direction = OPERATIONS[op][0]
        rs = tuple(dict(r) for r in ranges)
        ctx = self.transfer_context
        src, dst = (ctx.cpu_buffer_id, ctx.gpu_buffer_id) if direction == "h2d" else (ctx.gpu_buffer_id,
                                                                                      ctx.cpu_buffer_id)
        self._intent_counter += 1
        intent = TransferIntent(
            intent_id=f"{ctx.intent_prefix}-{op}-{self._intent_counter}", job_id=ctx.job_id,
            session_id=ctx.session_id, source_buffer_id=src, destination_buffer_id=dst, direction=direction,
            total_bytes=sum(r["bytes"] for r in rs), ranges=rs, workload_kind=ctx.workload_kind,
            priority=ctx.priority, policy_hints=ctx.policy_hints,
            metadata={**ctx.metadata, "operation": op, "block_names": [b.name for b in blocks]})
        receipt = self.client.submit_transfer_intent(intent)
        if not isinstance(receipt, TransferReceipt):
            raise TypeError("submit_transfer_intent must return a TransferReceipt")
        if receipt.intent_id != intent.intent_id:
            raise ValueError("receipt intent_id does not match transfer intent")
        return ReceiptTransferHandle(self.client, intent, receipt, ctx.wait_timeout_seconds)


class BucketStoreMixin:
    """Packed fixed-size buckets over one backing pair (weights, params,
    optimizer state)."""

    def add_bucket(self, name: str, cpu_tensor, gpu_tensor=None, *, bucket_id=None, cpu_offset: int = 0,
                   gpu_offset: int = 0, byte_count: int | None = None) -> OffloadBlock:
        return self.add(name, cpu_tensor, gpu_tensor, block_id=name if bucket_id is None else bucket_id,
                        cpu_slot=bucket_id, gpu_slot=bucket_id, cpu_offset=cpu_offset, gpu_offset=gpu_offset,
                        byte_count=byte_count)

    def add_packed_buckets(self, prefix: str, cpu_tensor, gpu_tensor, *, bucket_bytes: int, bucket_count: int,
                           start_offset: int = 0) -> list[OffloadBlock]:
        if bucket_bytes <= 0:
            raise ValueError("bucket_bytes must be positive")
        if bucket_count <= 0:
            raise ValueError("bucket_count must be positive")
        if start_offset < 0:
            raise ValueError("start_offset must be non-negative")
        return [self.add_bucket(f"{prefix}{i}", cpu_tensor, gpu_tensor, bucket_id=i,
                                cpu_offset=start_offset + i * bucket_bytes, gpu_offset=start_offset + i * bucket_bytes,
                                byte_count=bucket_bytes) for i in range(bucket_count)]

    def bucket(self, name: str) -> OffloadBlock:
        return self.get_block(name)

    def bucket_info(self, name: str) -> OffloadBlockInfo:
        return self.block_info(name)

    def bucket_infos(self, names: Iterable[str] | None = None) -> list[OffloadBlockInfo]:
        return self.block_infos(names)

    def wait_all(self) -> None:
        self.wait_many(self.names())

    def _mark(self, names, state: BlockState) -> None:
        for n in (self.names() if names is None else list(names)):
            self.set_block_state(n, state, clear_transfer_state=True)


OffloadManager = OffloadStore
KVBlockStore = OffloadStore

__all__ = ["AdapterTransferContext", "BlockState", "BucketStoreMixin", "KVBlockStore", "OffloadBatch",
           "OffloadBlock", "OffloadBlockInfo", "OffloadManager", "OffloadStore", "ReceiptTransferHandle",
           "TransferIntentClient", "TransferStats", "summarize_transfer_handles", "transfer_stats_from_receipt"]
