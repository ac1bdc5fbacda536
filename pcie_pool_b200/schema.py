"""Contract objects shared by every layer (client, daemon, scheduler, worker).

Names, fields and wire shapes follow the reference's contract module
(turbobus/schema.py:1-1420) so that plans, receipts, tickets and worker
envelopes serialise to the same JSON (``dataclasses.asdict``).  The
implementation is declarative: every frozen contract lists how each field is
coerced and checked (``_FIELDS``), and a shared ``__post_init__`` applies the
table before the class-specific cross-field rules run.

Bandwidth fields named ``*_gbps`` carry GiB/s, as in the reference
(cpp/src/executor_cuda.cu:28-35 divides by 1024**3).
"""

from __future__ import annotations

from dataclasses import dataclass, field, fields, is_dataclass
from enum import Enum
from collections.abc import Mapping
from typing import Any, Callable


# ---- enums -------------------------------------------------------------------------

class TransferMode(str, Enum):
    AUTO = "auto"
    POOL = "pool"
    DIRECT = "direct"
    RELAY = "relay"


class RequestType(str, Enum):
    REGISTER_JOB = "REGISTER_JOB"
    REGISTER_SESSION = "REGISTER_SESSION"
    REGISTER_BUFFER = "REGISTER_BUFFER"
    GET_INVENTORY = "GET_INVENTORY"
    DISCOVER_RELAYS = "DISCOVER_RELAYS"
    REAP_EXPIRED_LEASES = "REAP_EXPIRED_LEASES"
    PROFILE = "PROFILE"
    GET_PROFILE = "GET_PROFILE"
    PUT_PROFILE = "PUT_PROFILE"
    INVALIDATE_PROFILE = "INVALIDATE_PROFILE"
    INVALIDATE_TOPOLOGY = "INVALIDATE_TOPOLOGY"
    PLAN_TRANSFER = "PLAN_TRANSFER"
    SUBMIT_TRANSFER_INTENT = "SUBMIT_TRANSFER_INTENT"
    WAIT_TRANSFER_RECEIPT = "WAIT_TRANSFER_RECEIPT"
    RESCHEDULE_TRANSFER = "RESCHEDULE_TRANSFER"
    TRANSFER_STATUS = "TRANSFER_STATUS"
    RESERVE_TRANSFER = "RESERVE_TRANSFER"
    ISSUE_LEASE = "ISSUE_LEASE"
    VALIDATE_LEASE = "VALIDATE_LEASE"
    AUTHORIZE_WORKER_TRANSFER = "AUTHORIZE_WORKER_TRANSFER"
    RELEASE_TRANSFER = "RELEASE_TRANSFER"
    CLEANUP = "CLEANUP"
    CLOSE_SESSION = "CLOSE_SESSION"


class TransferStatusState(str, Enum):
    SUBMITTED = "submitted"
    RUNNING = "running"
    COMPLETE = "complete"
    FAILED = "failed"
    CANCELED = "canceled"


TERMINAL_STATES = frozenset({TransferStatusState.COMPLETE, TransferStatusState.FAILED,
                             TransferStatusState.CANCELED})


class BufferKind(str, Enum):
    CPU = "cpu"
    CPU_PINNED = "cpu_pinned"
    GPU = "gpu"
    RELAY_STAGING = "relay_staging"


class WorkloadKind(str, Enum):
    GENERIC = "generic"
    KV_CACHE = "kv_cache"
    MODEL_WEIGHTS = "model_weights"
    TRAINING_STATE = "training_state"
    OPTIMIZER_STATE = "optimizer_state"


class SchedulingDecisionState(str, Enum):
    PLANNED = "planned"
    FALLBACK = "fallback"
    REJECTED = "rejected"


# ---- record conversion ----------------------------------------------------------------

def contract_asdict(obj: Any) -> dict[str, Any]:
    """Dict of a contract for responses: nested contracts are converted, the
    top-level containers are copied, but their contents (plan chunk lists,
    ranges) are shared rather than deep-copied.  Contracts are immutable once
    issued, and a plan of N chunks would otherwise be copied N-deep on every
    response (``dataclasses.asdict`` dominated the per-intent control cost)."""
    cls = type(obj)
    names = _FIELD_NAMES.get(cls)
    if names is None:
        names = _FIELD_NAMES[cls] = tuple(f.name for f in fields(obj))
    out: dict[str, Any] = {}
    for name in names:
        v = getattr(obj, name)
        t = type(v)
        if t is dict:
            v = dict(v)
        elif t is list:
            v = list(v)
        elif hasattr(t, "__dataclass_fields__"):
            v = contract_asdict(v)
        elif isinstance(v, dict):
            v = dict(v)
        elif isinstance(v, list):
            v = list(v)
        out[name] = v
    return out


_FIELD_NAMES: dict[type, tuple[str, ...]] = {}


# ---- field coercers ------------------------------------------------------------------

def nonempty(value: Any, name: str) -> str:
    text = str(value)
    if not text.strip():
        raise ValueError(f"{name} must be non-empty")
    return text


def opt(fn: Callable[[Any, str], Any]) -> Callable[[Any, str], Any]:
    def inner(value: Any, name: str) -> Any:
        return None if value is None else fn(value, name)

    return inner


def nonneg_int(value: Any, name: str) -> int:
    v = int(value)
    if v < 0:
        raise ValueError(f"{name} must be non-negative")
    return v


def nonneg_float(value: Any, name: str) -> float:
    v = float(value)
    if v < 0:
        raise ValueError(f"{name} must be non-negative")
    return v


def as_int(value: Any, name: str) -> int:
    return int(value)


def as_float(value: Any, name: str) -> float:
    return float(value)


def as_bool(value: Any, name: str) -> bool:
    return bool(value)


def as_str(value: Any, name: str) -> str:
    return str(value)


def mapping(value: Any, name: str) -> dict[str, Any]:
    if not isinstance(value, Mapping):
        raise TypeError(f"{name} must be a mapping")
    return dict(value)


def mapping_tuple(value: Any, name: str) -> tuple[dict[str, Any], ...]:
    out = []
    for item in value:
        if not isinstance(item, Mapping):
            raise TypeError(f"{name} entries must be mappings")
        out.append(dict(item))
    return tuple(out)


def nonempty_tuple(value: Any, name: str) -> tuple[str, ...]:
    return tuple(nonempty(v, name) for v in value)


def enum_of(cls: type[Enum]) -> Callable[[Any, str], Any]:
    def inner(value: Any, name: str) -> Any:
        return cls(value)

    return inner


def coerce_direction(value: Any, name: str = "direction") -> str:
    d = str(value).lower()
    if d not in ("h2d", "d2h"):
        raise ValueError("direction must be h2d or d2h")
    return d


class ValidatedRanges(tuple):
    """A tuple of byte ranges that ``byte_ranges`` already checked; passing it
    to another contract skips the per-range work (tickets carry every chunk)."""

    __slots__ = ()


def byte_ranges(value: Any, name: str = "ranges") -> tuple[dict[str, int], ...]:
    if type(value) is ValidatedRanges:
        return value
    out = []
    append = out.append
    for item in value:
        src, dst, n = item["src_offset"], item["dst_offset"], item["bytes"]
        if type(src) is not int or type(dst) is not int or type(n) is not int:  # noqa: E721 - exact ints pass as is
            src, dst, n = int(src), int(dst), int(n)
        if src < 0 or dst < 0:
            raise ValueError("range offsets must be non-negative")
        if n <= 0:
            raise ValueError("range bytes must be positive")
        append({"src_offset": src, "dst_offset": dst, "bytes": n})
    return ValidatedRanges(out)


FORBIDDEN_POLICY_KEYS = frozenset({
    "mode", "path", "paths", "route", "routes", "relay", "relays", "relay_gpu", "relay_gpus",
    "target_device", "target_gpu",
})


def coerce_policy_hints(value: Any, name: str = "policy_hints") -> dict[str, Any]:
    """Intents state what they need, never which physical path to take."""
    hints = mapping(value, name)
    bad = sorted(str(k) for k in hints if str(k).lower() in FORBIDDEN_POLICY_KEYS)
    if bad:
        raise ValueError("policy_hints must not choose physical paths: " + ", ".join(bad))
    return hints


def cuda_ipc_handle(value: Any) -> str:
    if not isinstance(value, str):
        raise ValueError("cuda_ipc_handle must be a hex string")
    try:
        raw = bytes.fromhex(value)
    except ValueError as exc:
        raise ValueError("cuda_ipc_handle must be hex encoded") from exc
    if len(raw) != 64:
        raise ValueError("cuda_ipc_handle must decode to 64 bytes")
    return raw.hex()


def buffer_handle_metadata(*, kind: str, pinned: bool, device_index: int | None,
                           size_bytes: int, handle_type: str, metadata: Any) -> dict[str, Any]:
    """Validate the per-handle-type metadata of a buffer registration.

    ``shared_pinned_cpu``: cpu_pinned + pinned, and the shm name / offset /
    size must cover the buffer.  ``cuda_ipc_device``: gpu with a device index
    and a 64-byte legacy IPC handle (hex).
    """
    if not handle_type.strip():
        raise ValueError("handle_type must be non-empty")
    if not isinstance(metadata, Mapping):
        raise TypeError("metadata must be a dict")
    md = dict(metadata)
    if handle_type == "shared_pinned_cpu":
        if kind != "cpu_pinned":
            raise ValueError("shared_pinned_cpu handles require cpu_pinned buffers")
        if not pinned:
            raise ValueError("shared_pinned_cpu handles require pinned buffers")
        for key in ("shared_memory_name", "offset_bytes", "shared_memory_size_bytes"):
            if key not in md:
                raise ValueError(f"shared_pinned_cpu metadata requires {key}")
        if int(md["offset_bytes"]) < 0:
            raise ValueError("shared_pinned_cpu offset_bytes must be non-negative")
        if int(md["shared_memory_size_bytes"]) < int(md["offset_bytes"]) + int(size_bytes):
            raise ValueError("shared_pinned_cpu shared_memory_size_bytes is smaller than buffer span")
    elif handle_type == "cuda_ipc_device":
        if kind != "gpu":
            raise ValueError("cuda_ipc_device handles require gpu buffers")
        if device_index is None:
            raise ValueError("cuda_ipc_device handles require device_index")
        if "cuda_ipc_handle" not in md:
            raise ValueError("cuda_ipc_device metadata requires cuda_ipc_handle")
        md["cuda_ipc_handle"] = cuda_ipc_handle(md["cuda_ipc_handle"])
        if "cuda_ipc_offset" in md:
            off = md["cuda_ipc_offset"]
            if isinstance(off, bool) or not isinstance(off, int) or off < 0:
                raise ValueError("cuda_ipc_offset must be a non-negative integer")
    elif handle_type == "cuda_vmm_fd":
        # a CUDA VMM allocation exported as a POSIX file descriptor; the
        # descriptor itself travels beside the request (SCM_RIGHTS on the
        # daemon socket) and the daemon records its own copy as ``vmm_fd``
        if kind != "gpu" or device_index is None:
            raise ValueError("cuda_vmm_fd handles require gpu buffers with a device_index")
        mapped = md.get("vmm_mapped_bytes")
        if isinstance(mapped, bool) or not isinstance(mapped, int) or mapped < int(size_bytes):
            raise ValueError("cuda_vmm_fd metadata requires vmm_mapped_bytes covering the buffer")
        if "vmm_fd" in md and (isinstance(md["vmm_fd"], bool) or not isinstance(md["vmm_fd"], int)
                               or md["vmm_fd"] < 0):
            raise ValueError("vmm_fd must be a descriptor number")
    return md


# ---- declarative frozen contracts -------------------------------------------------------

class _Contract:
    """Mixin: apply ``_FIELDS`` coercers, then ``_check`` cross-field rules."""

    _FIELDS: dict[str, Callable[[Any, str], Any]] = {}

    def __post_init__(self) -> None:
        for name, fn in self._FIELDS.items():
            object.__setattr__(self, name, fn(getattr(self, name), name))
        self._check()

    def _check(self) -> None:  # pragma: no cover - overridden
        pass


def _check_ranges_total(total: int, ranges: tuple[dict[str, int], ...], label: str) -> None:
    if sum(r["bytes"] for r in ranges) != total:
        raise ValueError(f"{label} must equal the sum of range bytes")


@dataclass(frozen=True)
class AutoTransferDecision:
    requested_mode: TransferMode
    resolved_mode: TransferMode
    request_bytes: int
    request_chunks: int
    direct_h2d_bw_gbps: float
    relay_effective_bw_gbps: float
    eligible_relay_devices: tuple[int, ...]
    reason: str


@dataclass(frozen=True)
class PeerIdentity(_Contract):
    authenticated: bool
    source: str
    user_id: str | None = None
    process_id: int | None = None
    group_id: int | None = None
    container_id: str | None = None
    unsupported_reason: str | None = None

    _FIELDS = {
        "authenticated": as_bool, "source": nonempty, "user_id": opt(nonempty),
        "process_id": opt(nonneg_int), "group_id": opt(nonneg_int),
        "container_id": opt(nonempty),
    }

    def _check(self) -> None:
        if self.authenticated and self.user_id is None:
            raise ValueError("authenticated peer identity requires user_id")
        if not self.authenticated and self.unsupported_reason is not None:
            object.__setattr__(self, "unsupported_reason",
                               nonempty(self.unsupported_reason, "unsupported_reason"))


@dataclass(frozen=True)
class JobIdentity(_Contract):
    job_id: str
    user_id: str | None = None
    session_id: str | None = None
    container_id: str | None = None
    process_id: int | None = None
    weight: float = 1.0

    _FIELDS = {
        "job_id": nonempty, "user_id": opt(nonempty), "session_id": opt(nonempty),
        "container_id": opt(nonempty), "process_id": opt(nonneg_int), "weight": as_float,
    }

    def _check(self) -> None:
        if self.weight <= 0.0:
            raise ValueError("job weight must be positive")


@dataclass(frozen=True)
class BufferHandle(_Contract):
    buffer_id: str
    job_id: str
    session_id: str
    kind: BufferKind | str
    size_bytes: int
    device_index: int | None = None
    address: int | None = None
    pinned: bool = False
    handle_type: str = "registered_buffer"
    metadata: Mapping[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "buffer_id": nonempty, "job_id": nonempty, "session_id": nonempty,
        "kind": enum_of(BufferKind), "size_bytes": nonneg_int, "device_index": opt(nonneg_int),
        "address": opt(nonneg_int), "pinned": as_bool,
        "handle_type": lambda v, n: nonempty(v, n).lower(), "metadata": mapping,
    }

    def _check(self) -> None:
        if self.kind is BufferKind.GPU and self.device_index is None:
            raise ValueError("gpu buffer handles require device_index")
        if self.kind is BufferKind.CPU_PINNED and not self.pinned:
            raise ValueError("cpu_pinned buffer handles require pinned=True")
        object.__setattr__(self, "metadata", buffer_handle_metadata(
            kind=self.kind.value, pinned=self.pinned, device_index=self.device_index,
            size_bytes=self.size_bytes, handle_type=self.handle_type, metadata=self.metadata))


@dataclass(frozen=True)
class TransferIntent(_Contract):
    intent_id: str
    job_id: str
    session_id: str
    source_buffer_id: str
    destination_buffer_id: str
    direction: str
    total_bytes: int
    ranges: tuple[Mapping[str, int], ...]
    workload_kind: WorkloadKind | str = WorkloadKind.GENERIC
    priority: int = 0
    policy_hints: Mapping[str, Any] = field(default_factory=dict)
    metadata: Mapping[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "intent_id": nonempty, "job_id": nonempty, "session_id": nonempty,
        "source_buffer_id": nonempty, "destination_buffer_id": nonempty, "direction": coerce_direction,
        "total_bytes": as_int, "ranges": byte_ranges, "workload_kind": enum_of(WorkloadKind),
        "priority": as_int, "policy_hints": coerce_policy_hints, "metadata": mapping,
    }

    def _check(self) -> None:
        if self.total_bytes <= 0:
            raise ValueError("total_bytes must be positive")
        if not self.ranges:
            raise ValueError("transfer intent requires at least one byte range")
        _check_ranges_total(self.total_bytes, self.ranges, "total_bytes")
        if self.source_buffer_id == self.destination_buffer_id:
            raise ValueError("source and destination buffers must be different")


@dataclass(frozen=True)
class TopologySnapshot(_Contract):
    snapshot_id: str
    source: str
    discovered_at: float
    version: int = 0
    devices: tuple[Mapping[str, Any], ...] = field(default_factory=tuple)
    pcie_links: tuple[Mapping[str, Any], ...] = field(default_factory=tuple)
    fabric_links: tuple[Mapping[str, Any], ...] = field(default_factory=tuple)
    numa_nodes: tuple[Mapping[str, Any], ...] = field(default_factory=tuple)
    metadata: Mapping[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "snapshot_id": nonempty, "source": nonempty, "discovered_at": nonneg_float,
        "version": nonneg_int, "devices": mapping_tuple, "pcie_links": mapping_tuple,
        "fabric_links": mapping_tuple, "numa_nodes": mapping_tuple, "metadata": mapping,
    }


@dataclass(frozen=True)
class SchedulingDecision(_Contract):
    decision_id: str
    intent_id: str
    topology_snapshot_id: str
    job_id: str
    session_id: str
    state: SchedulingDecisionState | str
    plan: Mapping[str, Any] = field(default_factory=dict)
    path_summary: tuple[Mapping[str, Any], ...] = field(default_factory=tuple)
    fallback_reason: str | None = None
    rejection_reason: str | None = None
    issued_at: float = 0.0
    metadata: Mapping[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "decision_id": nonempty, "intent_id": nonempty, "topology_snapshot_id": nonempty,
        "job_id": nonempty, "session_id": nonempty, "state": enum_of(SchedulingDecisionState),
        "plan": mapping, "path_summary": mapping_tuple, "fallback_reason": opt(nonempty),
        "rejection_reason": opt(nonempty), "issued_at": nonneg_float, "metadata": mapping,
    }

    def _check(self) -> None:
        if self.state is SchedulingDecisionState.REJECTED:
            if self.plan:
                raise ValueError("rejected scheduling decisions must not include a plan")
            if self.rejection_reason is None:
                raise ValueError("rejected scheduling decisions require rejection_reason")
        else:
            if not self.plan:
                raise ValueError("planned scheduling decisions require a plan")
            if self.state is SchedulingDecisionState.FALLBACK and self.fallback_reason is None:
                raise ValueError("fallback scheduling decisions require fallback_reason")


@dataclass(frozen=True)
class ExecutionTicket(_Contract):
    ticket_id: str
    decision_id: str
    intent_id: str
    topology_snapshot_id: str
    job_id: str
    session_id: str
    source_buffer_id: str
    destination_buffer_id: str
    direction: str
    total_bytes: int
    ranges: tuple[Mapping[str, int], ...]
    plan: Mapping[str, Any]
    issued_at: float
    expires_at: float
    lease_ids: tuple[str, ...] = field(default_factory=tuple)
    metadata: Mapping[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "ticket_id": nonempty, "decision_id": nonempty, "intent_id": nonempty,
        "topology_snapshot_id": nonempty, "job_id": nonempty, "session_id": nonempty,
        "source_buffer_id": nonempty, "destination_buffer_id": nonempty, "direction": coerce_direction,
        "total_bytes": as_int, "ranges": byte_ranges, "plan": mapping,
        "issued_at": nonneg_float, "expires_at": as_float, "lease_ids": nonempty_tuple,
        "metadata": mapping,
    }

    def _check(self) -> None:
        if self.total_bytes <= 0:
            raise ValueError("ticket total_bytes must be positive")
        if not self.ranges:
            raise ValueError("execution ticket requires at least one byte range")
        _check_ranges_total(self.total_bytes, self.ranges, "ticket total_bytes")
        if not self.plan:
            raise ValueError("execution ticket requires daemon-issued plan")
        if self.expires_at <= self.issued_at:
            raise ValueError("expires_at must be later than issued_at")
        if self.source_buffer_id == self.destination_buffer_id:
            raise ValueError("source and destination buffers must be different")


@dataclass(frozen=True)
class TransferReceipt(_Contract):
    receipt_id: str
    ticket_id: str
    intent_id: str
    decision_id: str
    topology_snapshot_id: str
    job_id: str
    session_id: str
    state: TransferStatusState | str
    bytes_total: int
    bytes_completed: int
    started_at: float = 0.0
    completed_at: float | None = None
    path_stats: tuple[Mapping[str, Any], ...] = field(default_factory=tuple)
    error: str | None = None
    metadata: Mapping[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "receipt_id": nonempty, "ticket_id": nonempty, "intent_id": nonempty,
        "decision_id": nonempty, "topology_snapshot_id": nonempty, "job_id": nonempty,
        "session_id": nonempty, "state": enum_of(TransferStatusState),
        "bytes_total": nonneg_int, "bytes_completed": nonneg_int, "started_at": nonneg_float,
        "completed_at": opt(as_float), "path_stats": mapping_tuple, "error": opt(as_str),
        "metadata": mapping,
    }

    def _check(self) -> None:
        if self.bytes_completed > self.bytes_total:
            raise ValueError("bytes_completed cannot exceed bytes_total")
        if self.state is TransferStatusState.COMPLETE:
            if self.bytes_completed != self.bytes_total:
                raise ValueError("complete receipt must report all bytes completed")
            if self.error is not None:
                raise ValueError("complete receipt cannot include error")
        if self.state in (TransferStatusState.FAILED, TransferStatusState.CANCELED):
            if self.error is None or not self.error.strip():
                raise ValueError("failed or canceled receipt requires error")
        if self.completed_at is not None and self.completed_at < self.started_at:
            raise ValueError("completed_at must not be earlier than started_at")


@dataclass(frozen=True)
class BufferRegistration(_Contract):
    buffer_id: str
    job_id: str
    kind: str
    size_bytes: int
    device_index: int | None = None
    address: int | None = None
    pinned: bool = False
    handle_type: str = "registered_buffer"
    metadata: dict[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "buffer_id": nonempty, "job_id": nonempty, "kind": nonempty, "size_bytes": nonneg_int,
        "device_index": opt(nonneg_int), "address": opt(nonneg_int), "pinned": as_bool,
        "handle_type": lambda v, n: str(v).lower(),
    }

    def _check(self) -> None:
        object.__setattr__(self, "metadata", buffer_handle_metadata(
            kind=self.kind, pinned=self.pinned, device_index=self.device_index,
            size_bytes=self.size_bytes, handle_type=self.handle_type, metadata=self.metadata))


@dataclass(frozen=True)
class LeaseToken(_Contract):
    lease_id: str
    session_id: str
    relay_gpu: int
    token: str
    buffer_ids: tuple[str, ...] = field(default_factory=tuple)
    job_id: str | None = None
    issued_at: float = 0.0
    expires_at: float = 0.0

    _FIELDS = {
        "lease_id": nonempty, "session_id": nonempty, "relay_gpu": nonneg_int,
        "token": nonempty, "buffer_ids": nonempty_tuple, "job_id": opt(as_str),
        "issued_at": as_float, "expires_at": as_float,
    }

    def _check(self) -> None:
        if self.expires_at and self.expires_at < self.issued_at:
            raise ValueError("expires_at must not be earlier than issued_at")


@dataclass(frozen=True)
class TransferStatus(_Contract):
    transfer_id: str
    job_id: str
    state: TransferStatusState
    bytes_total: int
    bytes_completed: int = 0
    session_id: str | None = None
    error: str | None = None

    _FIELDS = {
        "transfer_id": nonempty, "job_id": nonempty, "state": enum_of(TransferStatusState),
        "bytes_total": nonneg_int, "bytes_completed": nonneg_int, "session_id": opt(as_str),
        "error": opt(as_str),
    }

    def _check(self) -> None:
        if self.bytes_completed > self.bytes_total:
            raise ValueError("bytes_completed cannot exceed bytes_total")
        if self.state is TransferStatusState.COMPLETE and self.bytes_completed != self.bytes_total:
            raise ValueError("complete transfer must report bytes_total completed")


@dataclass(frozen=True)
class WorkerTransferAuthorizationRequest(_Contract):
    transfer_id: str
    lease_id: str
    token: str
    session_id: str
    job_id: str
    src_buffer_id: str
    dst_buffer_id: str
    direction: str
    ranges: tuple[dict[str, int], ...] = field(default_factory=tuple)
    relay_gpu: int | None = None

    _FIELDS = {
        "transfer_id": nonempty, "lease_id": nonempty, "token": nonempty,
        "session_id": nonempty, "job_id": nonempty, "src_buffer_id": nonempty,
        "dst_buffer_id": nonempty, "direction": coerce_direction, "ranges": byte_ranges,
        "relay_gpu": opt(nonneg_int),
    }


@dataclass(frozen=True)
class WorkerTransferAuthorization(_Contract):
    transfer_id: str
    lease_id: str
    session_id: str
    job_id: str
    src_buffer: BufferRegistration
    dst_buffer: BufferRegistration
    direction: str
    ranges: tuple[dict[str, int], ...] = field(default_factory=tuple)
    relay_gpu: int | None = None
    plan: dict[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "transfer_id": nonempty, "lease_id": nonempty, "session_id": nonempty,
        "job_id": nonempty, "direction": coerce_direction, "ranges": byte_ranges,
        "relay_gpu": opt(nonneg_int), "plan": mapping,
    }

    def _check(self) -> None:
        if self.src_buffer.job_id != self.job_id:
            raise ValueError("src buffer job does not match authorization job")
        if self.dst_buffer.job_id != self.job_id:
            raise ValueError("dst buffer job does not match authorization job")


@dataclass(frozen=True)
class WorkerBufferHandle(_Contract):
    buffer_id: str
    job_id: str
    kind: str
    size_bytes: int
    access: str
    device_index: int | None = None
    address: int | None = None
    pinned: bool = False
    handle_type: str = "registered_buffer"
    metadata: dict[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "buffer_id": nonempty, "job_id": nonempty, "kind": nonempty, "size_bytes": nonneg_int,
        "access": lambda v, n: str(v).lower(), "device_index": opt(nonneg_int),
        "address": opt(nonneg_int), "pinned": as_bool,
        "handle_type": lambda v, n: nonempty(str(v).lower(), n),
    }

    @classmethod
    def from_buffer_registration(cls, buffer: BufferRegistration, access: str) -> "WorkerBufferHandle":
        if not isinstance(buffer, BufferRegistration):
            raise TypeError("buffer must be a BufferRegistration")
        return cls(buffer_id=buffer.buffer_id, job_id=buffer.job_id, kind=buffer.kind,
                   size_bytes=buffer.size_bytes, access=access, device_index=buffer.device_index,
                   address=buffer.address, pinned=buffer.pinned, handle_type=buffer.handle_type,
                   metadata=buffer.metadata)

    def _check(self) -> None:
        if self.access not in ("read", "write", "read_write"):
            raise ValueError("access must be read, write, or read_write")
        object.__setattr__(self, "metadata", buffer_handle_metadata(
            kind=self.kind, pinned=self.pinned, device_index=self.device_index,
            size_bytes=self.size_bytes, handle_type=self.handle_type, metadata=self.metadata))


@dataclass(frozen=True)
class WorkerStagingBufferRequirement(_Contract):
    relay_gpu: int
    total_bytes: int
    max_chunk_bytes: int
    chunk_count: int
    alignment_bytes: int = 256
    buffer_kind: str = "relay_staging"
    metadata: dict[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "relay_gpu": nonneg_int, "total_bytes": as_int, "max_chunk_bytes": as_int,
        "chunk_count": as_int, "alignment_bytes": as_int, "buffer_kind": nonempty,
        "metadata": mapping,
    }

    def _check(self) -> None:
        if self.total_bytes <= 0:
            raise ValueError("staging total_bytes must be positive")
        if self.max_chunk_bytes <= 0:
            raise ValueError("staging max_chunk_bytes must be positive")
        if self.max_chunk_bytes > self.total_bytes:
            raise ValueError("staging max_chunk_bytes cannot exceed total_bytes")
        if self.chunk_count <= 0:
            raise ValueError("staging chunk_count must be positive")
        if self.alignment_bytes <= 0:
            raise ValueError("staging alignment_bytes must be positive")


def _check_worker_handle_direction(d: str, src: WorkerBufferHandle, dst: WorkerBufferHandle) -> None:
    """h2d moves shared pinned host memory into a device buffer; d2h the reverse."""
    want_src, want_dst = (("shared_pinned_cpu", "cuda_ipc_device") if d == "h2d"
                          else ("cuda_ipc_device", "shared_pinned_cpu"))
    if src.handle_type != want_src:
        raise ValueError(f"{d} worker source must be {want_src}")
    if dst.handle_type != want_dst:
        raise ValueError(f"{d} worker destination must be {want_dst}")


def check_plan_chunk_bounds(plan: Mapping[str, Any], src_size: int, dst_size: int) -> None:
    for asg in plan.get("assignments", ()) or ():
        if not isinstance(asg, Mapping):
            raise ValueError("daemon plan assignment must be a mapping")
        runs = asg.get("chunk_runs")
        spans = ([(r[0], r[1], r[2]) for r in runs if isinstance(r, (list, tuple)) and len(r) == 4]
                 if runs else asg.get("chunks", ()) or ())
        if runs and len(spans) != len(runs):
            raise ValueError("daemon plan chunk run must be [src_offset, dst_offset, bytes, chunk_bytes]")
        for ch in spans:
            if not isinstance(ch, (Mapping, tuple)):
                raise ValueError("daemon plan chunk must be a mapping")
            s, d, n = ((int(ch["src_offset"]), int(ch["dst_offset"]), int(ch["bytes"])) if isinstance(ch, Mapping)
                       else (int(ch[0]), int(ch[1]), int(ch[2])))
            if s < 0 or d < 0:
                raise ValueError("daemon plan chunk offsets must be non-negative")
            if n <= 0:
                raise ValueError("daemon plan chunk bytes must be positive")
            if s + n > src_size:
                raise ValueError("daemon plan chunk exceeds src buffer size")
            if d + n > dst_size:
                raise ValueError("daemon plan chunk exceeds dst buffer size")


@dataclass(frozen=True)
class WorkerDataPlaneRequest(_Contract):
    transfer_id: str
    lease_id: str
    session_id: str
    job_id: str
    relay_gpu: int
    direction: str
    src_handle: WorkerBufferHandle
    dst_handle: WorkerBufferHandle
    staging: WorkerStagingBufferRequirement
    ranges: tuple[dict[str, int], ...] = field(default_factory=tuple)
    plan: dict[str, Any] = field(default_factory=dict)
    metadata: dict[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "transfer_id": nonempty, "lease_id": nonempty, "session_id": nonempty,
        "job_id": nonempty, "relay_gpu": nonneg_int, "direction": coerce_direction,
        "ranges": byte_ranges, "plan": mapping, "metadata": mapping,
    }

    @classmethod
    def from_authorization(cls, authorization: WorkerTransferAuthorization, *,
                           staging_alignment_bytes: int = 256,
                           metadata: dict[str, Any] | None = None) -> "WorkerDataPlaneRequest":
        if not isinstance(authorization, WorkerTransferAuthorization):
            raise TypeError("authorization must be a WorkerTransferAuthorization")
        if authorization.relay_gpu is None:
            raise ValueError("relay_gpu is required for worker data-plane request")
        ranges = tuple(authorization.ranges)
        if not ranges:
            raise ValueError("worker data-plane request requires chunk ranges")
        return cls(
            transfer_id=authorization.transfer_id, lease_id=authorization.lease_id,
            session_id=authorization.session_id, job_id=authorization.job_id,
            relay_gpu=authorization.relay_gpu, direction=authorization.direction,
            src_handle=WorkerBufferHandle.from_buffer_registration(authorization.src_buffer, "read"),
            dst_handle=WorkerBufferHandle.from_buffer_registration(authorization.dst_buffer, "write"),
            staging=WorkerStagingBufferRequirement(
                relay_gpu=authorization.relay_gpu, total_bytes=sum(r["bytes"] for r in ranges),
                max_chunk_bytes=max(r["bytes"] for r in ranges), chunk_count=len(ranges),
                alignment_bytes=staging_alignment_bytes),
            ranges=ranges, plan=authorization.plan, metadata=metadata or {})

    def _check(self) -> None:
        for name, typ in (("src_handle", WorkerBufferHandle), ("dst_handle", WorkerBufferHandle),
                          ("staging", WorkerStagingBufferRequirement)):
            if not isinstance(getattr(self, name), typ):
                raise TypeError(f"{name} must be a {typ.__name__}")
        if not self.ranges:
            raise ValueError("worker data-plane request requires chunk ranges")
        if sum(r["bytes"] for r in self.ranges) > self.staging.total_bytes:
            raise ValueError("ranges exceed staging total_bytes")
        if max(r["bytes"] for r in self.ranges) > self.staging.max_chunk_bytes:
            raise ValueError("ranges exceed staging max_chunk_bytes")
        if self.staging.chunk_count < len(self.ranges):
            raise ValueError("staging chunk_count cannot be smaller than range count")
        if self.src_handle.job_id != self.job_id:
            raise ValueError("src handle job does not match request job")
        if self.dst_handle.job_id != self.job_id:
            raise ValueError("dst handle job does not match request job")
        if self.staging.relay_gpu != self.relay_gpu:
            raise ValueError("staging relay does not match request relay")
        _check_worker_handle_direction(self.direction, self.src_handle, self.dst_handle)
        for r in self.ranges:
            if r["src_offset"] + r["bytes"] > self.src_handle.size_bytes:
                raise ValueError("worker range exceeds src buffer size")
            if r["dst_offset"] + r["bytes"] > self.dst_handle.size_bytes:
                raise ValueError("worker range exceeds dst buffer size")
        check_plan_chunk_bounds(self.plan, self.src_handle.size_bytes, self.dst_handle.size_bytes)


@dataclass(frozen=True)
class WorkerDataPlaneCompletion(_Contract):
    transfer_id: str
    lease_id: str
    state: TransferStatusState
    bytes_completed: int
    error: str | None = None
    metadata: dict[str, Any] = field(default_factory=dict)

    _FIELDS = {
        "transfer_id": nonempty, "lease_id": nonempty, "state": enum_of(TransferStatusState),
        "bytes_completed": nonneg_int, "error": opt(as_str), "metadata": mapping,
    }

    def _check(self) -> None:
        if self.state not in (TransferStatusState.COMPLETE, TransferStatusState.FAILED):
            raise ValueError("worker completion state must be complete or failed")
        if self.state is TransferStatusState.FAILED and self.error is None:
            raise ValueError("failed worker completion requires error")
        if self.state is TransferStatusState.COMPLETE and self.error is not None:
            raise ValueError("complete worker completion cannot include error")


@dataclass(frozen=True)
class CleanupRequest(_Contract):
    target_kind: str
    target_id: str
    reason: str
    force: bool = False

    _FIELDS = {"target_kind": nonempty, "target_id": nonempty, "reason": nonempty}


# ---- mutable daemon records -------------------------------------------------------------

@dataclass
class Session:
    session_id: str
    target_gpu: int
    relay_gpus: list[int]
    max_inflight_chunks: int
    active_chunks: int = 0
    active: bool = True
    created_at: float = 0.0
    last_seen: float = 0.0
    closed_at: float | None = None


@dataclass
class RelayQuota:
    relay_gpu: int
    max_sessions: int = 1
    max_inflight_chunks: int = 8
    sessions: set[str] = field(default_factory=set)
    active_chunks: int = 0

    def can_attach(self) -> bool:
        return len(self.sessions) < self.max_sessions

    def can_reserve(self, chunks: int) -> bool:
        return self.active_chunks + chunks <= self.max_inflight_chunks


@dataclass
class TransferReservation:
    reservation_id: str
    session_id: str
    relay_gpu: int
    chunks: int
    bytes: int = 0
    direction: str = "unknown"


@dataclass
class DaemonRequest:
    request_type: RequestType
    session_id: str | None = None
    payload: dict[str, Any] = field(default_factory=dict)
    peer_identity: PeerIdentity | None = None

    def __post_init__(self) -> None:
        if self.peer_identity is not None and not isinstance(self.peer_identity, PeerIdentity):
            self.peer_identity = PeerIdentity(**self.peer_identity)


@dataclass
class DaemonResponse:
    ok: bool
    payload: dict[str, Any] = field(default_factory=dict)
    error: str | None = None


__all__ = [
    "AutoTransferDecision", "BufferHandle", "BufferKind", "BufferRegistration", "CleanupRequest",
    "DaemonRequest", "DaemonResponse", "ExecutionTicket", "JobIdentity", "LeaseToken",
    "PeerIdentity", "RelayQuota", "RequestType", "SchedulingDecision", "SchedulingDecisionState",
    "Session", "TopologySnapshot", "TransferIntent", "TransferMode", "TransferReceipt",
    "TransferReservation", "TransferStatus", "TransferStatusState", "WorkloadKind",
    "WorkerTransferAuthorization", "WorkerTransferAuthorizationRequest", "WorkerBufferHandle",
    "WorkerDataPlaneCompletion", "WorkerDataPlaneRequest", "WorkerStagingBufferRequirement",
]
