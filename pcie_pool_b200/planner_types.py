"""Immutable plan records.  ``PlannerTransferPlan.as_dict()`` defines the plan
JSON shared with the reference (turbobus/planner_types.py:8-141,
turbobus/plan_trace.py:43-47):

    {"total_bytes", "chunk_bytes", "assignments": [
        {"path": {"kind", "direction", "target_device", "relay_device",
                  "h2d_bw_gbps", "d2h_bw_gbps", "p2p_bw_gbps",
                  "effective_bw_gbps", "enabled", "fabric_kind"},
         "chunks": [{"src_offset", "dst_offset", "bytes", "relay_device"}],
         "bytes", "chunk_count"}]}
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field

from .schema import TransferMode

DEFAULT_CHUNK_BYTES = 16 * 1024 * 1024


class _AsDict:
    def as_dict(self) -> dict[str, object]:
        return asdict(self)


@dataclass(frozen=True)
class PlannerDevice(_AsDict):
    device_id: int
    kind: str = "gpu"
    memory_bytes: int = 0
    numa_node: int | None = None
    pci_bus_id: str | None = None
    name: str | None = None


@dataclass(frozen=True)
class PlannerLink(_AsDict):
    src_device: int
    dst_device: int
    kind: str
    bandwidth_gbps: float = 0.0
    latency_ns: float = 0.0
    enabled: bool = True
    fabric_kind: str | None = None


@dataclass(frozen=True)
class PlannerChunk(_AsDict):
    src_offset: int
    dst_offset: int
    bytes: int
    relay_device: int | None = None


@dataclass(frozen=True)
class PlannerPath(_AsDict):
    kind: str
    direction: str
    target_device: int
    relay_device: int = -1
    h2d_bw_gbps: float = 0.0
    d2h_bw_gbps: float = 0.0
    p2p_bw_gbps: float = 0.0
    effective_bw_gbps: float = 0.0
    enabled: bool = True
    fabric_kind: str | None = None

    @property
    def lane_device(self) -> int:
        """GPU whose PCIe link carries this path."""
        return self.target_device if self.kind == "direct" else self.relay_device

    def as_dict(self) -> dict[str, object]:
        # built field by field: every plan conversion calls this once per path
        return {"kind": self.kind, "direction": self.direction, "target_device": self.target_device,
                "relay_device": self.relay_device, "h2d_bw_gbps": self.h2d_bw_gbps,
                "d2h_bw_gbps": self.d2h_bw_gbps, "p2p_bw_gbps": self.p2p_bw_gbps,
                "effective_bw_gbps": self.effective_bw_gbps, "enabled": self.enabled,
                "fabric_kind": self.fabric_kind}


@dataclass(frozen=True)
class PlannerPathAssignment:
    path: PlannerPath
    chunks: tuple[PlannerChunk, ...] = field(default_factory=tuple)

    @property
    def bytes(self) -> int:
        return sum(c.bytes for c in self.chunks)

    def as_dict(self) -> dict[str, object]:
        # flat records: built directly (dataclasses.asdict per chunk dominated
        # the cost of converting plans with thousands of chunks)
        chunks = [{"src_offset": c.src_offset, "dst_offset": c.dst_offset, "bytes": c.bytes,
                   "relay_device": c.relay_device} for c in self.chunks]
        return {"path": self.path.as_dict(), "chunks": chunks,
                "bytes": sum(c["bytes"] for c in chunks), "chunk_count": len(chunks)}


@dataclass(frozen=True)
class PlannerTransferPlan:
    total_bytes: int = 0
    chunk_bytes: int = DEFAULT_CHUNK_BYTES
    assignments: tuple[PlannerPathAssignment, ...] = field(default_factory=tuple)

    def as_dict(self) -> dict[str, object]:
        return {"total_bytes": self.total_bytes, "chunk_bytes": self.chunk_bytes,
                "assignments": [a.as_dict() for a in self.assignments]}

    @property
    def chunk_count(self) -> int:
        return sum(len(a.chunks) for a in self.assignments)


@dataclass(frozen=True)
class PlannerLease(_AsDict):
    lease_id: str
    session_id: str
    relay_device: int
    chunk_limit: int
    bytes_limit: int = 0
    direction: str = "unknown"
    granted_at: float = 0.0
    expires_at: float = 0.0
    active: bool = True
    job_id: str | None = None
    reason: str | None = None


@dataclass(frozen=True)
class PlannerStats:
    bytes: int = 0
    direct_bytes: int = 0
    relay_bytes: int = 0
    direct_chunks: int = 0
    relay_chunks: int = 0
    path_count: int = 0
    relay_path_count: int = 0
    fallback_reason: str | None = None
    requested_mode: TransferMode | str = TransferMode.POOL
    resolved_mode: TransferMode | str = TransferMode.POOL

    def as_dict(self) -> dict[str, object]:
        data = asdict(self)
        for key in ("requested_mode", "resolved_mode"):
            if isinstance(data[key], TransferMode):
                data[key] = data[key].value
        return data


__all__ = ["DEFAULT_CHUNK_BYTES", "PlannerChunk", "PlannerDevice", "PlannerLease", "PlannerLink",
           "PlannerPath", "PlannerPathAssignment", "PlannerStats", "PlannerTransferPlan"]
