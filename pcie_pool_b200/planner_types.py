"""Immutable plan records.  ``PlannerTransferPlan.as_dict()`` defines the plan
JSON shared with the reference (turbobus/planner_types.py:8-141,
turbobus/plan_trace.py:43-47):

    {"total_bytes", "chunk_bytes", "assignments": [
        {"path": {"kind", "direction", "target_device", "relay_device",
                  "h2d_bw_gbps", "d2h_bw_gbps", "p2p_bw_gbps",
                  "effective_bw_gbps", "enabled", "fabric_kind"},
         "chunks": [{"src_offset", "dst_offset", "bytes", "relay_device"}],
         "bytes", "chunk_count"}]}

Compact form (this framework's addition).  An assignment whose chunks form a
few contiguous spans carries ``"chunk_runs": [[src, dst, bytes, chunk], ...]``
instead of ``"chunks"``: one run stands for ``ceil(bytes / chunk)`` chunks at
``src + k*chunk`` / ``dst + k*chunk`` of ``min(chunk, bytes - k*chunk)``
bytes.  A lane that takes one contiguous span of a 4 GiB transfer is then one
record instead of hundreds, so planning, leases, tickets and the executor do
per-lane, not per-chunk, work.  Every reader goes through the accessors
below (``assignment_chunks`` / ``assignment_arrays`` / ...), and
``expand_plan`` turns a compact plan into the reference's chunk-list form
for files and tools that expect it.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import asdict, dataclass, field, fields

from .schema import TransferMode

DEFAULT_CHUNK_BYTES = 16 * 1024 * 1024


_NAMES: dict[type, tuple[str, ...]] = {}


def _plain(v):
    """``dataclasses.asdict`` semantics for these records (nested records to
    dicts, containers rebuilt), without its per-value generic dispatch."""
    t = type(v)
    if t in (int, float, str, bool) or v is None:
        return v
    if hasattr(t, "__dataclass_fields__"):
        return _record_dict(v)
    if t is tuple or t is list:
        return t(_plain(x) for x in v)
    if t is dict:
        return {k: _plain(x) for k, x in v.items()}
    return v


def _record_dict(obj) -> dict[str, object]:
    t = type(obj)
    names = _NAMES.get(t)
    if names is None:
        names = _NAMES[t] = tuple(f.name for f in fields(t))
    return {n: _plain(getattr(obj, n)) for n in names}


class _AsDict:
    def as_dict(self) -> dict[str, object]:
        return _record_dict(self)


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


def run_chunk_count(run) -> int:
    n, c = int(run[2]), int(run[3])
    return -(-n // c) if n > 0 else 0


@dataclass(frozen=True)
class PlannerPathAssignment:
    path: PlannerPath
    chunks: tuple[PlannerChunk, ...] = field(default_factory=tuple)
    # compact form: (src, dst, bytes, chunk) spans; used instead of ``chunks``
    runs: tuple[tuple[int, int, int, int], ...] = field(default_factory=tuple)

    @property
    def bytes(self) -> int:
        if self.runs:
            return sum(int(r[2]) for r in self.runs)
        return sum(c.bytes for c in self.chunks)

    @property
    def chunk_count(self) -> int:
        if self.runs:
            return sum(run_chunk_count(r) for r in self.runs)
        return len(self.chunks)

    def chunk_list(self) -> tuple[PlannerChunk, ...]:
        """Every chunk as a record (expands runs)."""
        if not self.runs:
            return self.chunks
        dev = None if self.path.kind == "direct" else self.path.relay_device
        return tuple(PlannerChunk(s, d, n, dev) for s, d, n in _expand_runs(self.runs))

    def as_dict(self) -> dict[str, object]:
        if self.runs:
            return {"path": self.path.as_dict(), "chunk_runs": [list(r) for r in self.runs],
                    "bytes": self.bytes, "chunk_count": self.chunk_count}
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
        return sum(a.chunk_count for a in self.assignments)


# ---- plan-dict accessors (both the chunk-list and the compact form) -------------------

def _expand_runs(runs):
    for r in runs:
        s, d, n, c = int(r[0]), int(r[1]), int(r[2]), int(r[3])
        if c <= 0:
            raise ValueError("chunk run needs a positive chunk size")
        for o in range(0, n, c):
            yield s + o, d + o, min(c, n - o)


def _check_run(r) -> None:
    if not isinstance(r, (list, tuple)) or len(r) != 4:
        raise ValueError("transfer plan chunk run must be [src_offset, dst_offset, bytes, chunk_bytes]")
    if min(int(x) for x in r) < 0 or int(r[2]) <= 0 or int(r[3]) <= 0:
        raise ValueError("transfer plan chunk run must have non-negative offsets and positive sizes")


def assignment_has_chunks(a: Mapping) -> bool:
    return bool(a.get("chunk_runs") or a.get("chunks"))


def assignment_chunk_count(a: Mapping) -> int:
    runs = a.get("chunk_runs")
    if runs:
        return sum(run_chunk_count(r) for r in runs)
    return len(a.get("chunks", ()) or ())


def assignment_bytes(a: Mapping) -> int:
    runs = a.get("chunk_runs")
    if runs:
        return sum(int(r[2]) for r in runs)
    return sum(int(c["bytes"]) for c in a.get("chunks", ()) or ())


def assignment_spans(a: Mapping) -> list[tuple[int, int, int]]:
    """(src, dst, bytes) extents of an assignment: one per chunk in the
    chunk-list form, one per run in the compact form (for bounds checks)."""
    runs = a.get("chunk_runs")
    if runs:
        for r in runs:
            _check_run(r)
        return [(int(r[0]), int(r[1]), int(r[2])) for r in runs]
    return [(int(c["src_offset"]), int(c["dst_offset"]), int(c["bytes"])) for c in assignment_chunks(a)]


def assignment_chunks(a: Mapping) -> list[dict]:
    """Chunk records ``{src_offset, dst_offset, bytes, relay_device}`` of one
    assignment, in order, from either form."""
    runs = a.get("chunk_runs")
    if not runs:
        out = []
        for c in a.get("chunks", ()) or ():
            if not isinstance(c, Mapping):
                raise ValueError("transfer plan chunk must be an object")
            out.append(c)
        return out
    path = a.get("path") if isinstance(a.get("path"), Mapping) else {}
    dev = None if str(path.get("kind", "direct")) == "direct" else path.get("relay_device")
    for r in runs:
        _check_run(r)
    return [{"src_offset": s, "dst_offset": d, "bytes": n, "relay_device": dev}
            for s, d, n in _expand_runs(runs)]


def assignment_arrays(a: Mapping):
    """(src, dst, bytes) uint64 arrays of one assignment's chunks; runs expand
    with vector arithmetic, without per-chunk Python objects."""
    import numpy as np

    runs = a.get("chunk_runs")
    if not runs:
        rows = [(int(c["src_offset"]), int(c["dst_offset"]), int(c["bytes"]))
                for c in assignment_chunks(a)]
        arr = np.array(rows, dtype=np.uint64).reshape(-1, 3)
        return arr[:, 0].copy(), arr[:, 1].copy(), arr[:, 2].copy()
    srcs, dsts, sizes = [], [], []
    for r in runs:
        _check_run(r)
        s, d, n, c = (int(x) for x in r)
        o = np.arange(0, n, c, dtype=np.uint64)
        srcs.append(o + np.uint64(s))
        dsts.append(o + np.uint64(d))
        sizes.append(np.minimum(np.uint64(c), np.uint64(n) - o))
    return np.concatenate(srcs), np.concatenate(dsts), np.concatenate(sizes)


def runs_from_chunks(src, dst, nbytes) -> list[list[int]]:
    """Merge consecutive equal-size chunks that are contiguous on both sides
    into runs (a run may end with one shorter chunk)."""
    runs: list[list[int]] = []
    for s, d, n in zip((int(x) for x in src), (int(x) for x in dst), (int(x) for x in nbytes)):
        if runs:
            r = runs[-1]
            full = r[2] % r[3] == 0  # the run so far ends on a whole chunk
            if full and s == r[0] + r[2] and d == r[1] + r[2] and n <= r[3]:
                r[2] += n
                continue
        runs.append([s, d, n, n])
    return runs


def expand_plan(plan: Mapping) -> dict:
    """The plan in the reference's chunk-list form (a new dict)."""
    out = dict(plan)
    asg = []
    for a in plan.get("assignments", ()) or ():
        if isinstance(a, Mapping) and a.get("chunk_runs"):
            b = {k: v for k, v in a.items() if k != "chunk_runs"}
            b["chunks"] = assignment_chunks(a)
            asg.append(b)
        else:
            asg.append(a)
    out["assignments"] = asg
    return out


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
           "PlannerPath", "PlannerPathAssignment", "PlannerStats", "PlannerTransferPlan", "assignment_arrays",
           "assignment_bytes", "assignment_chunk_count", "assignment_chunks", "assignment_has_chunks",
           "assignment_spans",
           "expand_plan", "run_chunk_count", "runs_from_chunks"]
