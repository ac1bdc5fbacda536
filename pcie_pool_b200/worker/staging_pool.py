"""Per-transfer staging-slot records of the worker helper.

A slot is the bookkeeping of one authorized transfer's relay staging
(``staging-N`` ids, requested bytes rounded up to the alignment, 256 by
default), as turbobus/worker/staging_pool.py:13-183.  The device memory
behind it is the worker's persistent PoolEngine rings (allocated once per
relay GPU, not per transfer); ``engine_ring_bytes`` reports them when an
engine is attached.
"""

from __future__ import annotations

import itertools
import threading
from dataclasses import asdict, dataclass
from typing import Callable

from ..schema import WorkerDataPlaneRequest


class WorkerStagingPoolError(RuntimeError):
    pass


def _align_up(n: int, a: int) -> int:
    return (int(n) + a - 1) // a * a


@dataclass(frozen=True)
class WorkerStagingSlot:
    slot_id: str
    transfer_id: str
    lease_id: str
    session_id: str
    job_id: str
    relay_gpu: int
    requested_bytes: int
    allocated_bytes: int
    max_chunk_bytes: int
    chunk_count: int
    alignment_bytes: int
    buffer_kind: str = "relay_staging"
    state: str = "allocated"

    @classmethod
    def from_request(cls, request: WorkerDataPlaneRequest, *, slot_id: str) -> "WorkerStagingSlot":
        if not isinstance(request, WorkerDataPlaneRequest):
            raise TypeError("request must be a WorkerDataPlaneRequest")
        st = request.staging
        return cls(slot_id=slot_id, transfer_id=request.transfer_id, lease_id=request.lease_id,
                   session_id=request.session_id, job_id=request.job_id, relay_gpu=request.relay_gpu,
                   requested_bytes=st.total_bytes, allocated_bytes=_align_up(st.total_bytes, st.alignment_bytes),
                   max_chunk_bytes=st.max_chunk_bytes, chunk_count=st.chunk_count,
                   alignment_bytes=st.alignment_bytes, buffer_kind=st.buffer_kind)

    def __post_init__(self) -> None:
        for name in ("slot_id", "transfer_id", "lease_id", "session_id", "job_id", "buffer_kind"):
            v = str(getattr(self, name))
            if not v.strip():
                raise ValueError(f"{name} must be non-empty")
            object.__setattr__(self, name, v)
        ints = {n: int(getattr(self, n)) for n in ("relay_gpu", "requested_bytes", "allocated_bytes",
                                                   "max_chunk_bytes", "chunk_count", "alignment_bytes")}
        if ints["relay_gpu"] < 0:
            raise ValueError("relay_gpu must be non-negative")
        if ints["requested_bytes"] <= 0:
            raise ValueError("requested_bytes must be positive")
        if ints["allocated_bytes"] < ints["requested_bytes"]:
            raise ValueError("allocated_bytes cannot be smaller than requested_bytes")
        if ints["max_chunk_bytes"] <= 0:
            raise ValueError("max_chunk_bytes must be positive")
        if ints["chunk_count"] <= 0:
            raise ValueError("chunk_count must be positive")
        if ints["alignment_bytes"] <= 0:
            raise ValueError("alignment_bytes must be positive")
        if ints["allocated_bytes"] % ints["alignment_bytes"]:
            raise ValueError("allocated_bytes must be alignment-sized")
        for n, v in ints.items():
            object.__setattr__(self, n, v)

    def as_dict(self) -> dict[str, object]:
        return asdict(self)

    def released(self) -> "WorkerStagingSlot":
        d = self.as_dict()
        d["state"] = "released"
        return WorkerStagingSlot(**d)


class WorkerStagingPool:
    def __init__(self, slot_id_factory: Callable[[], str] | None = None, engine=None) -> None:
        self._factory = slot_id_factory
        self._ids = itertools.count(1)
        self._slots: dict[str, WorkerStagingSlot] = {}
        self._lock = threading.Lock()
        self.engine = engine

    def _new_id(self) -> str:
        return str(self._factory()) if self._factory is not None else f"staging-{next(self._ids)}"

    def allocate(self, request: WorkerDataPlaneRequest) -> WorkerStagingSlot:
        with self._lock:
            sid = self._new_id()
            if sid in self._slots:
                raise WorkerStagingPoolError("staging slot id already exists")
            slot = WorkerStagingSlot.from_request(request, slot_id=sid)
            self._slots[sid] = slot
            return slot

    def describe(self, slot_id: str | None = None) -> dict[str, object]:
        with self._lock:
            if slot_id is not None:
                slot = self._slots.get(str(slot_id))
                if slot is None:
                    raise WorkerStagingPoolError("unknown staging slot")
                return slot.as_dict()
            out: dict[str, object] = {"slots": {k: s.as_dict() for k, s in sorted(self._slots.items())}}
        if self.engine is not None:
            out["engine_ring_bytes"] = int(self.engine.slot_bytes) * int(self.engine.slots)
        return out

    def validate_slot_for_request(self, slot_id: str, request: WorkerDataPlaneRequest) -> WorkerStagingSlot:
        if not isinstance(request, WorkerDataPlaneRequest):
            raise TypeError("request must be a WorkerDataPlaneRequest")
        with self._lock:
            slot = self._slots.get(str(slot_id))
        if slot is None:
            raise WorkerStagingPoolError("unknown staging slot")
        for attr, what in (("transfer_id", "transfer"), ("lease_id", "lease"), ("session_id", "session"),
                           ("job_id", "job"), ("relay_gpu", "relay")):
            if getattr(slot, attr) != getattr(request, attr):
                raise WorkerStagingPoolError(f"staging slot {what} mismatch")
        return slot

    def release(self, slot_id: str, request: WorkerDataPlaneRequest | None = None) -> WorkerStagingSlot:
        if request is not None:
            self.validate_slot_for_request(slot_id, request)
        with self._lock:
            slot = self._slots.pop(str(slot_id), None)
        if slot is None:
            raise WorkerStagingPoolError("unknown staging slot")
        return slot.released()

    def __len__(self) -> int:
        return len(self._slots)


__all__ = ["WorkerStagingPool", "WorkerStagingPoolError", "WorkerStagingSlot"]
