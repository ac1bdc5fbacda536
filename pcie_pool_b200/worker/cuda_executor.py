"""Executes a daemon-ticketed plan on the native PoolEngine.

Unlike the reference executor, which builds and initialises a new native
runtime for every transfer (staging cudaMalloc + memset + peer enable,
turbobus/worker/cuda_executor.py:67-75), one engine per device set lives
for the worker process: its staging rings, streams, mailboxes and peer
mappings are made once.  The plan is narrowed to the ticket's authorized
relays and checked the same way (:174-245); the result carries the path
label ``pool_h2d``/``relay_d2h``/... and per-lane measured stats.
"""

from __future__ import annotations

from ..planner_types import assignment_chunks

import threading
from typing import Any

from .helper import WorkerTransferRequest, WorkerTransferResult, WorkerTransferState, _failed
from .resources import WorkerDataPlaneResources
from .staging_pool import WorkerStagingSlot


def scoped_plan(request: WorkerTransferRequest, target: int) -> dict[str, Any]:
    """The ticketed plan with only authorized relays, re-validated."""
    dp = request.data_plane
    if not dp.plan:
        raise ValueError("CUDA worker executor requires a daemon-issued transfer plan")
    relays = set(request.relay_gpus)
    out, relay_chunks, total = [], [], 0
    for a in dp.plan.get("assignments", ()) or ():
        if not isinstance(a, dict) or not isinstance(a.get("path"), dict):
            raise ValueError("daemon plan assignment must be a mapping with a path")
        p = dict(a["path"])
        kind = str(p.get("kind", "")).lower()
        if kind not in ("direct", "relay"):
            raise ValueError("daemon plan path must be direct or relay")
        if str(p.get("direction", "")).lower() != dp.direction:
            raise ValueError("daemon plan direction does not match worker request")
        if int(p.get("target_device", target)) != target:
            raise ValueError("daemon plan target does not match worker target")
        if not bool(p.get("enabled", True)):
            raise ValueError("daemon plan path is disabled")
        if kind == "relay":
            if int(p.get("relay_device", -1)) not in relays:
                raise ValueError("daemon plan relay is not authorized by worker ticket")
        else:
            p["relay_device"] = -1
        p["enabled"] = True
        chunks = [{"src_offset": int(c["src_offset"]), "dst_offset": int(c["dst_offset"]), "bytes": int(c["bytes"])}
                  for c in assignment_chunks(a)]
        if not chunks:
            continue
        n = sum(c["bytes"] for c in chunks)
        total += n
        if kind == "relay":
            relay_chunks.extend(chunks)
        out.append({"path": p, "chunks": chunks, "bytes": n, "chunk_count": len(chunks)})
    if not out:
        raise ValueError("daemon plan has no authorized relay chunks")
    if int(dp.plan.get("total_bytes", total)) != total:
        raise ValueError("daemon plan total bytes do not match assigned chunks")
    if tuple(relay_chunks) != dp.ranges:
        raise ValueError("authorized ranges do not match daemon plan")
    return {"total_bytes": total, "chunk_bytes": int(dp.plan.get("chunk_bytes", dp.staging.max_chunk_bytes)),
            "assignments": out}


def _validate(request: WorkerTransferRequest, slot: WorkerStagingSlot) -> None:
    if not isinstance(request, WorkerTransferRequest):
        raise TypeError("request must be a WorkerTransferRequest")
    if request.ticket is None:
        raise ValueError("CUDA worker executor requires a daemon-issued ExecutionTicket")
    if not isinstance(slot, WorkerStagingSlot):
        raise TypeError("staging_slot must be a WorkerStagingSlot")
    if slot.transfer_id != request.transfer_id:
        raise ValueError("staging slot transfer does not match request")
    if slot.lease_id != request.authorization.lease_id:
        raise ValueError("staging slot lease does not match request")
    if slot.relay_gpu != request.authorization.relay_gpu:
        raise ValueError("staging slot relay does not match request")


class CudaWorkerExecutor:
    """``execute_bound(request, slot, resources)`` runs the plan; engines are
    cached per sorted device set."""

    def __init__(self, *, engine_factory=None, checksum: bool = True, **engine_kw) -> None:
        self._factory = engine_factory
        self._engine_kw = engine_kw
        self.checksum = checksum
        self._engines: dict[tuple[int, ...], Any] = {}
        self._run_locks: dict[int, threading.Lock] = {}
        self._lock = threading.Lock()

    def engine_for(self, devices) -> Any:
        key = tuple(sorted({int(d) for d in devices}))
        with self._lock:
            eng = self._engines.get(key)
            if eng is None:
                if self._factory is not None:
                    eng = self._factory(list(key))
                else:
                    from ..parallel.engine import PoolEngine

                    eng = PoolEngine(list(key), **self._engine_kw)
                self._engines[key] = eng
                self._run_locks[id(eng)] = threading.Lock()
            return eng

    def execute(self, request: WorkerTransferRequest, staging_slot: WorkerStagingSlot) -> WorkerTransferResult:
        _validate(request, staging_slot)
        return _failed(request, staging_slot, "CUDA worker execution requires bound data-plane resources")

    def execute_bound(self, request: WorkerTransferRequest, staging_slot: WorkerStagingSlot,
                      resources: WorkerDataPlaneResources) -> WorkerTransferResult:
        _validate(request, staging_slot)
        if not isinstance(resources, WorkerDataPlaneResources):
            raise TypeError("resources must be WorkerDataPlaneResources")
        if resources.request != request.data_plane:
            return _failed(request, staging_slot, "bound resources do not match the worker request")
        dp = request.data_plane
        th = dp.dst_handle if dp.direction == "h2d" else dp.src_handle
        if th.device_index is None:
            return _failed(request, staging_slot, "CUDA worker executor requires a GPU device index")
        target = int(th.device_index)
        try:
            from ..parallel.engine import D2H, H2D, lanes_from_plan

            plan = scoped_plan(request, target)
            eng = self.engine_for([target, *request.relay_gpus])
            lanes = lanes_from_plan(plan, target)
            with self._run_locks[id(eng)]:  # one transfer at a time per engine (shared staging rings)
                r = eng.run(H2D if dp.direction == "h2d" else D2H, target, resources.host_ptr, resources.host_bytes,
                            resources.device_ptr, resources.device_bytes, lanes, checksum=self.checksum)
        except Exception as exc:  # noqa: BLE001 - engine failures become failed results
            return _failed(request, staging_slot, str(exc))
        if not r.ok:
            return _failed(request, staging_slot, r.error or "engine transfer failed")
        d_b = sum(l.bytes for l in r.lanes if l.direct)
        d_c = sum(l.chunks for l in r.lanes if l.direct)
        r_b = sum(l.bytes for l in r.lanes if not l.direct)
        r_c = sum(l.chunks for l in r.lanes if not l.direct)
        return WorkerTransferResult(request.transfer_id, WorkerTransferState.COMPLETE, bytes_completed=r.bytes,
                                    metadata={
                                        "executor": "cuda_worker", "path": f"{'pool' if d_c else 'relay'}_{dp.direction}",
                                        "plan_source": "daemon", "relay_gpu": dp.relay_gpu,
                                        "relay_gpus": list(request.relay_gpus), "target_device": target,
                                        "src_buffer_id": dp.src_handle.buffer_id,
                                        "dst_buffer_id": dp.dst_handle.buffer_id,
                                        "staging_slot_id": staging_slot.slot_id, "direct_bytes": d_b,
                                        "direct_chunks": d_c, "relay_bytes": r_b, "relay_chunks": r_c,
                                        "cuda_ms": r.cuda_ms, "gb_per_s": r.gb_per_s,
                                        "lanes": [{"device": l.device, "direct": l.direct, "bytes": l.bytes,
                                                   "chunks": l.chunks, "cuda_ms": l.cuda_ms} for l in r.lanes]})


__all__ = ["CudaWorkerExecutor", "scoped_plan"]
