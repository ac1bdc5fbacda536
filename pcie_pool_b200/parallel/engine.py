"""Python face of the native data plane (``PoolEngine``).

A transfer is described lane by lane: ``Lane(device, src_off, dst_off,
bytes)`` where ``device`` is the GPU whose PCIe link carries the lane (the
target itself for the direct lane).  Plans in the reference's dict format
(``{"assignments": [{"path": {...}, "chunks": [...]}]}``,
turbobus/plan_trace.py:43-47) convert with :func:`lanes_from_plan`.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from collections.abc import Mapping
from typing import Iterable, Sequence

import numpy as np

from .._native import native

H2D = 0
D2H = 1


@dataclass
class Lane:
    device: int
    src_off: np.ndarray
    dst_off: np.ndarray
    bytes: np.ndarray
    unit0: np.ndarray | None = None
    tensor: np.ndarray | None = None
    count: np.ndarray | None = None

    @property
    def total_bytes(self) -> int:
        return int(self.bytes.sum()) if self.bytes.size else 0

    @property
    def num_chunks(self) -> int:
        return int(self.bytes.size)


def make_lane(device: int, chunks: Iterable, **extra) -> Lane:
    """Lane from (src_off, dst_off, bytes) tuples or dicts."""
    rows = [(c["src_offset"], c["dst_offset"], c["bytes"]) if isinstance(c, Mapping) else (c[0], c[1], c[2])
            for c in chunks]
    a = np.array(rows, dtype=np.uint64).reshape(-1, 3)
    return Lane(device, a[:, 0].copy(), a[:, 1].copy(), a[:, 2].copy(), **extra)


def lanes_from_plan(plan: Mapping, target: int) -> list[Lane]:
    """Convert a plan dict (chunk-list or compact chunk-run form) into engine
    lanes; runs expand with vector arithmetic."""
    from ..planner_types import assignment_arrays, assignment_has_chunks

    lanes: list[Lane] = []
    for asg in plan.get("assignments", []) or []:
        path = asg["path"]
        if not path.get("enabled", True):
            raise ValueError("plan contains a disabled path")
        kind = str(path.get("kind", "direct"))
        dev = target if kind == "direct" else int(path["relay_device"])
        if assignment_has_chunks(asg):
            src, dst, nbytes = assignment_arrays(asg)
            lanes.append(Lane(dev, src, dst, nbytes))
    return lanes


@dataclass
class LaneResult:
    device: int
    direct: bool
    bytes: int
    chunks: int
    cuda_ms: float


@dataclass
class TransferResult:
    id: int
    ok: bool
    status_code: int
    error: str
    bytes: int
    cuda_ms: float
    submit_to_complete_ms: float
    gib_per_s: float
    lanes: list[LaneResult] = field(default_factory=list)
    checksums: np.ndarray | None = None  # shape [chunks, 2] in lane order
    error_lane: int = -1
    error_chunk: int = -1
    trace: np.ndarray | None = None  # [chunks, 4] device ns: wait begin, ready, done, CTAs (lane order)

    @property
    def gb_per_s(self) -> float:
        return self.bytes / 1e9 / (self.cuda_ms / 1e3) if self.cuda_ms > 0 else 0.0

    def raise_for_status(self) -> "TransferResult":
        if not self.ok:
            raise RuntimeError(f"transfer {self.id} failed: {self.error} "
                               f"(lane {self.error_lane}, chunk {self.error_chunk})")
        return self


class PoolEngine:
    """Persistent multi-GPU data plane (one per process)."""

    def __init__(self, devices: Sequence[int], slot_bytes: int = 16 << 20, slots: int = 3,
                 ctas_per_lane: int = 4, timeout_s: float = 10.0,
                 enable_peer_access: bool = True, coalesce_bytes: int = 64 << 20) -> None:
        C = native()
        opt = C.EngineOptions()
        opt.slot_bytes = int(slot_bytes)
        opt.slots = int(slots)
        opt.ctas_per_lane = int(ctas_per_lane)
        opt.timeout_s = float(timeout_s)
        opt.enable_peer_access = bool(enable_peer_access)
        opt.coalesce_bytes = int(coalesce_bytes)
        self._C = C
        self._eng = C.PoolEngine(list(int(d) for d in devices), opt)
        self.devices = list(int(d) for d in devices)
        self.slot_bytes = int(slot_bytes)
        self.slots = int(slots)

    # -- submission -------------------------------------------------------------
    def submit(self, direction: int, target: int, host_ptr: int, host_bytes: int, dev_ptr: int,
               dev_bytes: int, lanes: Sequence[Lane], op: int | None = None,
               checksum: bool = False, stage_direct: bool = False, serialize: bool = False,
               ctas_per_lane: int = 0, timeout_s: float = 0.0,
               unit_bytes: int = 0, unit_addrs: np.ndarray | None = None,
               ranges: tuple[np.ndarray, np.ndarray, np.ndarray] | None = None,
               tensors: Sequence[tuple[int, int, int, int]] = (),
               adam: Mapping | None = None,
               debug_drop_publish: int = -1, trace: bool = False) -> int:
        C = self._C
        spec = C.TransferSpec()
        spec.direction = int(direction)
        spec.target = int(target)
        spec.host_ptr = int(host_ptr)
        spec.host_bytes = int(host_bytes)
        spec.dev_ptr = int(dev_ptr)
        spec.dev_bytes = int(dev_bytes)
        spec.op = C.OP_COPY if op is None else int(op)
        spec.checksum = bool(checksum)
        spec.stage_direct = bool(stage_direct)
        spec.serialize = bool(serialize)
        spec.debug_drop_publish = int(debug_drop_publish)
        spec.trace = bool(trace)
        spec.ctas_per_lane = int(ctas_per_lane)
        spec.timeout_s = float(timeout_s)
        spec.unit_bytes = int(unit_bytes)
        if unit_addrs is not None:
            spec.set_unit_addrs(np.ascontiguousarray(unit_addrs, dtype=np.uint64))
        if ranges is not None:
            addr, nbytes, pos = ranges
            spec.set_ranges(np.ascontiguousarray(addr, dtype=np.uint64),
                            np.ascontiguousarray(nbytes, dtype=np.uint32),
                            np.ascontiguousarray(pos, dtype=np.uint64))
        qts = []
        for q, scales, rows, cols in tensors:
            t = C.QuantTensorSpec()
            t.q, t.scales, t.rows, t.cols = int(q), int(scales), int(rows), int(cols)
            qts.append(t)
        spec.tensors = qts
        if adam is not None:
            a = C.AdamStepSpec()
            for k, v in adam.items():
                setattr(a, k, v)
            spec.adam = a
        nl = []
        for lane in lanes:
            ls = C.LaneSpec()
            ls.device = int(lane.device)
            ls.set_chunks(lane.src_off, lane.dst_off, lane.bytes, lane.unit0, lane.tensor,
                          lane.count)
            nl.append(ls)
        spec.lanes = nl
        self._last_chunks = [lane.num_chunks for lane in lanes]
        return self._eng.submit(spec)

    def wait(self, tid: int, host_timeout_s: float = 0.0) -> TransferResult:
        r = self._eng.wait(tid, host_timeout_s)
        cs = np.array(r.checksums, dtype=np.uint64).reshape(-1, 2)
        tr = np.array(r.trace, dtype=np.uint64).reshape(-1, 4) if len(r.trace) else None
        return TransferResult(
            id=r.id, ok=r.ok, status_code=r.status_code, error=r.error, bytes=r.bytes,
            cuda_ms=r.cuda_ms, submit_to_complete_ms=r.submit_to_complete_ms,
            gib_per_s=r.gib_per_s,
            lanes=[LaneResult(l.device, l.direct, l.bytes, l.chunks, l.cuda_ms) for l in r.lanes],
            checksums=cs, error_lane=r.error_lane, error_chunk=r.error_chunk, trace=tr)

    def query(self, tid: int) -> bool:
        return self._eng.query(tid)

    def run(self, *args, **kwargs) -> TransferResult:
        return self.wait(self.submit(*args, **kwargs))

    # -- introspection ---------------------------------------------------------------
    def max_lane_ctas(self, device: int) -> int:
        return self._eng.max_lane_ctas(device)

    def issued(self, device: int) -> list[int]:
        return list(self._eng.issued(device))


def split_even(total: int, chunk: int, lanes: Sequence[int], start: int = 0,
               dst_start: int = 0) -> list[Lane]:
    """Round-robin ``chunk``-sized pieces of [start, start+total) over lanes."""
    offs = np.arange(0, total, chunk, dtype=np.uint64)
    sizes = np.minimum(chunk, total - offs).astype(np.uint64)
    out = []
    for i, dev in enumerate(lanes):
        sel = slice(i, None, len(lanes))
        out.append(Lane(int(dev), offs[sel] + np.uint64(start), offs[sel] + np.uint64(dst_start),
                        sizes[sel].copy()))
    return [l for l in out if l.num_chunks]
