"""Executes admitted intents: the piece the reference's daemon lacks (its
SUBMIT_TRANSFER_INTENT plans, issues a ticket and returns; nothing consumes
the ticket).

``IntentExecutor`` runs each admitted ticket on a ``DataPlane`` in a worker
thread, outside the daemon lock, and reports RUNNING / COMPLETE / FAILED with
measured per-lane statistics back to the daemon.  Data planes:

* ``EngineDataPlane`` - the native PoolEngine on real GPUs; resolves buffer
  registrations (shared pinned host memory by shm name, CUDA IPC device
  handles, or in-process addresses) and moves the plan's chunks through the
  direct + relay lanes with the fused landing kernel (checksum on);
* ``mock.MockDataPlane`` - a simulated node on the CPU (tests, config 1).
"""

from __future__ import annotations

import threading
from collections import OrderedDict
import time
import traceback
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Protocol

import numpy as np

from ..schema import BufferRegistration, ExecutionTicket, TransferIntent


@dataclass
class ExecutionResult:
    ok: bool
    bytes_completed: int
    error: str | None = None
    measured: dict[str, Any] = field(default_factory=dict)


class DataPlane(Protocol):
    def execute(self, ticket: ExecutionTicket, src: BufferRegistration, dst: BufferRegistration,
                intent: TransferIntent | None) -> ExecutionResult:
        ...


class IntentExecutor:
    """Thread-pool executor bound to one daemon."""

    def __init__(self, data_plane: DataPlane, max_workers: int = 4) -> None:
        self.data_plane = data_plane
        self._pool = ThreadPoolExecutor(max_workers=max_workers, thread_name_prefix="pcie-pool-exec")
        self._canceled: set[str] = set()
        self._lock = threading.Lock()
        self.completed: list[str] = []

    def bind(self, daemon) -> None:
        self._daemon = daemon

    def submit(self, daemon, transfer_id: str, ticket: ExecutionTicket, src: BufferRegistration | None,
               dst: BufferRegistration | None, intent: TransferIntent | None) -> None:
        self._pool.submit(self._run, daemon, transfer_id, ticket, src, dst, intent)

    def cancel(self, transfer_id: str) -> None:
        with self._lock:
            self._canceled.add(transfer_id)

    def _run(self, daemon, tid: str, ticket: ExecutionTicket, src, dst, intent) -> None:
        with self._lock:
            if tid in self._canceled:
                return
        daemon.executor_started(tid)
        t0 = time.perf_counter()
        try:
            if src is None or dst is None:
                raise RuntimeError("ticket buffers are no longer registered")
            extra = daemon.landing_buffers(intent) if hasattr(daemon, "landing_buffers") else {}
            if extra:
                res = self.data_plane.execute(ticket, src, dst, intent, buffers=extra)
            else:
                res = self.data_plane.execute(ticket, src, dst, intent)
        except Exception as exc:  # noqa: BLE001 - every data-plane error fails the transfer
            res = ExecutionResult(ok=False, bytes_completed=0,
                                  error=f"{type(exc).__name__}: {exc}",
                                  measured={"traceback": traceback.format_exc(limit=5)})
        res.measured.setdefault("host_ms", (time.perf_counter() - t0) * 1e3)
        daemon.executor_finished(tid, ok_=res.ok, bytes_completed=res.bytes_completed, error=res.error,
                                 measured=res.measured)
        with self._lock:
            self.completed.append(tid)

    def shutdown(self, wait: bool = True) -> None:
        self._pool.shutdown(wait=wait)


class EngineDataPlane:
    """Runs tickets on the native PoolEngine (all GPUs of the node)."""

    def __init__(self, engine=None, devices=None, *, checksum: bool = True, failover: bool = True,
                 **engine_kw) -> None:
        self.failover = failover
        # tests: the next transfer drops the "ready" publications of this lane
        # (so its landing wait runs out) and runs with this device timeout
        self.debug_drop_publish = -1
        self.failover_timeout_s = 0.0
        self._engine = engine
        self._devices = devices
        self._engine_kw = engine_kw
        self.checksum = checksum
        self._host_maps: dict[str, tuple[Any, int]] = {}
        self._ipc: dict[str, int] = {}
        self._lock = threading.Lock()
        self._lane_cache: OrderedDict = OrderedDict()

    @property
    def engine(self):
        if self._engine is None:
            from ..parallel.engine import PoolEngine

            if self._devices is None:
                import torch

                self._devices = list(range(torch.cuda.device_count()))
            self._engine = PoolEngine(self._devices, **self._engine_kw)
        return self._engine

    def _lanes(self, plan, target: int):
        """Engine lanes of a plan.  The scheduler reuses plan objects for a
        repeated intent shape, so each plan's chunk arrays are kept; every
        call gets fresh ``Lane`` records over them (a fused op annotates its
        lanes with per-chunk fields, which must not leak into the next
        transfer).  The cache holds the plan's assignments so their identity
        stays unique."""
        from ..parallel.engine import Lane, lanes_from_plan

        asg = plan.get("assignments")
        if asg is None:
            return lanes_from_plan(plan, target)
        key = (id(asg), int(target))
        with self._lock:
            hit = self._lane_cache.get(key)
            if hit is not None and hit[0] is asg:
                self._lane_cache.move_to_end(key)
                base = hit[1]
            else:
                base = None
        if base is None:
            base = tuple(lanes_from_plan(plan, target))
            with self._lock:
                self._lane_cache[key] = (asg, base)
                while len(self._lane_cache) > 64:
                    self._lane_cache.popitem(last=False)
        return [Lane(l.device, l.src_off, l.dst_off, l.bytes) for l in base]

    # -- buffer resolution ------------------------------------------------------------------
    def host_pointer(self, buf: BufferRegistration) -> int:
        if buf.handle_type == "shared_pinned_cpu":
            name = str(buf.metadata["shared_memory_name"])
            with self._lock:
                if name not in self._host_maps:
                    from multiprocessing import shared_memory

                    from .._native import native

                    shm = shared_memory.SharedMemory(name=name)
                    import numpy as np

                    base = np.frombuffer(shm.buf, dtype=np.uint8).ctypes.data
                    if not native().is_pinned(base):
                        native().host_register(base, shm.size)
                    self._host_maps[name] = (shm, base)
                _shm, base = self._host_maps[name]
            return base + int(buf.metadata["offset_bytes"])
        if buf.address is None:
            raise ValueError(f"buffer {buf.buffer_id} has no host address")
        return int(buf.address)

    def device_pointer(self, buf: BufferRegistration) -> int:
        if buf.handle_type == "cuda_vmm_fd":
            # import the exporter's VMM allocation once per registration
            key = f"vmm:{buf.buffer_id}:{buf.metadata['vmm_fd']}"
            with self._lock:
                if key not in self._ipc:
                    from .._native import native

                    self._ipc[key] = native().vmm_import(int(buf.metadata["vmm_fd"]), int(buf.device_index or 0),
                                                         int(buf.metadata["vmm_mapped_bytes"]))
                return self._ipc[key]
        if buf.handle_type == "cuda_ipc_device":
            h = str(buf.metadata["cuda_ipc_handle"])
            with self._lock:
                if h not in self._ipc:
                    from .._native import native

                    self._ipc[h] = native().open_ipc_handle(bytes.fromhex(h), int(buf.device_index or 0))
                # the handle maps its allocation's base; the buffer may start inside it
                return self._ipc[h] + int(buf.metadata.get("cuda_ipc_offset", 0) or 0)
        if buf.address is None:
            raise ValueError(f"buffer {buf.buffer_id} has no device address")
        return int(buf.address)

    # -- execution ------------------------------------------------------------------------------
    def execute(self, ticket: ExecutionTicket, src: BufferRegistration, dst: BufferRegistration,
                intent: TransferIntent | None, buffers: dict | None = None) -> ExecutionResult:
        from ..parallel.engine import D2H, H2D, Lane, lanes_from_plan
        from .landing import LandingSpec, annotate_lanes, fp8_table, unit_addresses

        h2d = ticket.direction == "h2d"
        host_buf, dev_buf = (src, dst) if h2d else (dst, src)
        target = int(dev_buf.device_index or 0)
        host_ptr = self.host_pointer(host_buf)
        dev_ptr = self.device_pointer(dev_buf)
        # fused landing op named by the intent (validated by the daemon)
        spec = LandingSpec.from_metadata(intent.metadata) if intent is not None else None
        lanes = self._lanes(ticket.plan, target)
        eng = self.engine
        direction = H2D if h2d else D2H
        op_kw: dict = {}
        if spec is not None and spec.op != "copy":
            from .._native import native

            C = native()
            annotate_lanes(spec, lanes, h2d)
            if spec.op == "adamw":
                a = spec.adam_params
                regs = dict(buffers or {})
                if a["grads_buffer"] not in regs:
                    raise RuntimeError("adamw grads buffer is no longer registered")
                adam = {k: a[k] for k in ("lr", "beta1", "beta2", "eps", "weight_decay", "grad_scale", "step")}
                adam.update(grads=self.device_pointer(regs[a["grads_buffer"]]), params=dev_ptr,
                            nparams=int(a["nparams"]))
                op_kw = {"op": C.OP_ADAMW, "adam": adam}
            elif spec.units_op:
                regs = dict(buffers or {})
                regs.setdefault(dev_buf.buffer_id, dev_buf)
                missing = [b for b in spec.buffer_ids() if b not in regs]
                if missing:
                    raise RuntimeError(f"landing buffers are no longer registered: {missing}")
                op_kw = {"op": C.OP_SCATTER_UNITS if h2d else C.OP_GATHER_UNITS, "unit_bytes": spec.unit_bytes,
                         "unit_addrs": unit_addresses(spec, lambda b: self.device_pointer(regs[b]))}
            else:
                op_kw = {"op": C.OP_FP8_QUANT, "tensors": fp8_table(spec, dev_ptr)}
            if spec.ctas_per_lane:
                op_kw["ctas_per_lane"] = spec.ctas_per_lane

        def run(ls, drop=-1):
            kw = {"debug_drop_publish": drop} if drop >= 0 else {}
            if drop >= 0 and self.failover_timeout_s:
                kw["timeout_s"] = self.failover_timeout_s
            return eng.run(direction, target, host_ptr, host_buf.size_bytes, dev_ptr, dev_buf.size_bytes, ls,
                           checksum=self.checksum, **op_kw, **kw)

        drop, self.debug_drop_publish = self.debug_drop_publish, -1
        r = run(lanes, drop)
        failover = None
        lane_stats = list(r.lanes)
        checksums = None if r.checksums is None else np.array(r.checksums, dtype=np.uint64, copy=True)
        # an optimizer round trip is not idempotent: its lanes are never re-run
        idempotent = spec is None or spec.op != "adamw"
        if not r.ok and self.failover and idempotent and len(lanes) > 1 and 0 <= r.error_lane < len(lanes):
            # Lane failover: the chunks of the lane that failed are moved again
            # over a surviving lane (the direct lane when it survived).  Every
            # op here is a pure data movement, so chunks of the failed lane
            # that did land are simply written again with the same bytes.
            bad = lanes[r.error_lane]
            survivors = [l for i, l in enumerate(lanes) if i != r.error_lane]
            host = next((l for l in survivors if l.device == target), survivors[0])
            redo = Lane(host.device, bad.src_off, bad.dst_off, bad.bytes, unit0=bad.unit0, tensor=bad.tensor,
                        count=bad.count)
            r2 = run([redo])
            failover = {"failed_lane_device": int(bad.device), "rerun_on_device": int(host.device),
                        "rerun_bytes": int(bad.total_bytes), "first_error": r.error, "rerun_ok": bool(r2.ok)}
            if r2.ok:
                first = sum(len(l.bytes) for l in lanes[:r.error_lane])
                if checksums is not None and r2.checksums is not None and len(r2.checksums):
                    checksums[first:first + len(bad.bytes)] = np.asarray(r2.checksums, dtype=np.uint64)
                lane_stats = [l for i, l in enumerate(r.lanes) if i != r.error_lane] + list(r2.lanes)
                r = type(r)(id=r.id, ok=True, status_code=0, error="", bytes=sum(l.total_bytes for l in lanes),
                            cuda_ms=r.cuda_ms + r2.cuda_ms, submit_to_complete_ms=r.submit_to_complete_ms,
                            gib_per_s=r.gib_per_s, lanes=lane_stats, checksums=checksums)
        measured = {
            "cuda_ms": r.cuda_ms, "gib_per_s": r.gib_per_s, "gb_per_s": r.gb_per_s,
            "submit_to_complete_ms": r.submit_to_complete_ms,
            "path_stats": [{"kind": "direct" if l.direct else "relay", "direction": ticket.direction,
                            "target_device": target, "relay_device": -1 if l.direct else l.device,
                            "bytes": int(l.bytes), "chunk_count": int(l.chunks),
                            "cuda_ms": float(l.cuda_ms),
                            "gib_per_second": (l.bytes / (1 << 30)) / (l.cuda_ms / 1e3) if l.cuda_ms > 0 else 0.0}
                           for l in lane_stats],
        }
        measured["landing_op"] = spec.op if spec is not None else "copy"
        if failover is not None:
            measured["failover"] = failover
            measured["fallback_reason"] = (f"lane failover: relay {failover['failed_lane_device']} failed, "
                                           f"re-ran on {failover['rerun_on_device']}")
        if self.checksum and r.checksums is not None and len(r.checksums):
            measured["chunk_checksums"] = np.asarray(r.checksums, dtype=np.uint64).reshape(-1, 2).tolist()
        return ExecutionResult(ok=r.ok, bytes_completed=r.bytes if r.ok else 0,
                               error=None if r.ok else r.error, measured=measured)


__all__ = ["DataPlane", "EngineDataPlane", "ExecutionResult", "IntentExecutor"]
