"""A simulated node for CPU-only runs: N "GPUs" whose memory is host memory,
lanes that are threads, and a data plane with the engine's contract.

Used for BASELINE config 1 (daemon + planner + client end to end on a world
of 4 simulated GPUs), for host-side fault injection (a lane that raises,
stalls past a deadline or corrupts a chunk) and by the tests.  Every chunk's
lane assignment is recorded so a run can prove each chunk moved exactly once
on the lane the plan chose.
"""

from __future__ import annotations

import ctypes
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable

import numpy as np

from ..daemon.executor import ExecutionResult
from ..planner_types import assignment_chunks
from ..schema import BufferRegistration, ExecutionTicket, TransferIntent
from ..utils.checksum import checksum_bytes


class MockLaneError(RuntimeError):
    pass


@dataclass
class FaultPlan:
    """Host-side fault injection for the mock lanes."""

    fail_lane: int | None = None       # lane device that raises on its first chunk
    stall_lane: int | None = None      # lane device that sleeps stall_seconds per chunk
    stall_seconds: float = 0.0
    corrupt_lane: int | None = None    # lane device that flips one byte in its first chunk
    deadline_seconds: float = 30.0     # per-transfer watchdog


@dataclass
class MockWorld:
    """``gpu_count`` simulated devices, each with a bandwidth (GiB/s) used only
    to report modelled lane times."""

    gpu_count: int = 4
    lane_gibps: float = 50.0
    p2p_gibps: float = 600.0
    memory: dict[int, dict[int, np.ndarray]] = field(default_factory=dict)

    def alloc(self, device: int, nbytes: int) -> np.ndarray:
        """Device memory of a simulated GPU (host bytes), kept alive here."""
        if not 0 <= device < self.gpu_count:
            raise ValueError("device index out of range")
        arr = np.zeros(nbytes, dtype=np.uint8)
        self.memory.setdefault(device, {})[arr.ctypes.data] = arr
        return arr

    def profile(self, target: int = 0) -> dict[str, Any]:
        """A daemon profile entry for this world (GiB/s)."""
        return {"target_device": target, "direct_h2d_bw_gbps": self.lane_gibps,
                "direct_d2h_bw_gbps": self.lane_gibps,
                "relays": [{"relay_device": g, "target_device": target, "h2d_bw_gbps": self.lane_gibps,
                            "d2h_bw_gbps": self.lane_gibps, "p2p_bw_gbps": self.p2p_gibps,
                            "effective_bw_gbps": self.lane_gibps, "effective_d2h_bw_gbps": self.lane_gibps,
                            "p2p_enabled": True} for g in range(self.gpu_count) if g != target]}


class MockDataPlane:
    """Moves the bytes of a ticket's plan between in-process buffers, one
    thread per lane, honouring the plan's chunk-to-lane assignment."""

    def __init__(self, world: MockWorld | None = None, faults: FaultPlan | None = None,
                 checksum: bool = True) -> None:
        self.world = world or MockWorld()
        self.faults = faults or FaultPlan()
        self.checksum = checksum
        self.trace: list[dict[str, Any]] = []
        self._lock = threading.Lock()

    def execute(self, ticket: ExecutionTicket, src: BufferRegistration, dst: BufferRegistration,
                intent: TransferIntent | None, buffers: dict | None = None) -> ExecutionResult:
        from ..daemon.landing import LandingSpec

        if src.address is None or dst.address is None:
            raise MockLaneError("mock data plane needs in-process buffer addresses")
        plan = ticket.plan
        lanes = []
        for asg in plan.get("assignments", []) or []:
            p = asg["path"]
            dev = int(p["target_device"]) if p["kind"] == "direct" else int(p["relay_device"])
            lanes.append((dev, p["kind"], [(int(c["src_offset"]), int(c["dst_offset"]), int(c["bytes"]))
                                            for c in assignment_chunks(asg)]))
        spec = LandingSpec.from_metadata(intent.metadata) if intent is not None else None
        landing = None
        if spec is not None and spec.op != "copy":
            landing = _MockLanding(spec, ticket.direction == "h2d", src, dst, dict(buffers or {}))
        return self.run_lanes(ticket.direction, int(src.address), int(src.size_bytes),
                              int(dst.address), int(dst.size_bytes), lanes,
                              transfer_id=str(ticket.metadata.get("transfer_id", ticket.ticket_id)),
                              landing=landing)

    def run_lanes(self, direction: str, src: int, src_bytes: int, dst: int, dst_bytes: int,
                  lanes: list[tuple[int, str, list[tuple[int, int, int]]]],
                  transfer_id: str = "", landing: "_MockLanding | None" = None) -> ExecutionResult:
        f = self.faults
        results: dict[int, dict[str, Any]] = {}
        errors: list[str] = []
        sums: dict[tuple[int, int], tuple[int, int]] = {}

        def lane_worker(idx: int, dev: int, kind: str, chunks: list[tuple[int, int, int]]) -> None:
            t0 = time.perf_counter()
            moved = 0
            for k, (so, do, n) in enumerate(chunks):
                if landing is not None:
                    try:
                        landing.move(so, do, n)
                    except (ValueError, IndexError) as exc:
                        errors.append(f"lane {dev}: chunk {k}: {exc}")
                        return
                    moved += n
                    with self._lock:
                        self.trace.append({"transfer_id": transfer_id, "lane": dev, "kind": kind,
                                           "src_offset": so, "dst_offset": do, "bytes": n, "op": landing.spec.op})
                    continue
                if so < 0 or do < 0 or so + n > src_bytes or do + n > dst_bytes:
                    errors.append(f"lane {dev}: chunk {k} out of bounds")
                    return
                if f.fail_lane == dev:
                    errors.append(f"lane {dev}: injected failure")
                    return
                if f.stall_lane == dev and f.stall_seconds:
                    time.sleep(f.stall_seconds)
                if time.perf_counter() - t0 > f.deadline_seconds:
                    errors.append(f"lane {dev}: deadline exceeded")
                    return
                ctypes.memmove(dst + do, src + so, n)
                if f.corrupt_lane == dev and k == 0:
                    b = ctypes.c_uint8.from_address(dst + do)
                    b.value ^= 0xFF
                if self.checksum:
                    landed = np.ctypeslib.as_array((ctypes.c_uint8 * n).from_address(dst + do))
                    sent = np.ctypeslib.as_array((ctypes.c_uint8 * n).from_address(src + so))
                    sums[(idx, k)] = checksum_bytes(landed)
                    if checksum_bytes(sent) != sums[(idx, k)]:
                        errors.append(f"lane {dev}: checksum mismatch on chunk {k}")
                        return
                moved += n
                with self._lock:
                    self.trace.append({"transfer_id": transfer_id, "lane": dev, "kind": kind,
                                       "src_offset": so, "dst_offset": do, "bytes": n})
            results[idx] = {"device": dev, "kind": kind, "bytes": moved, "chunks": len(chunks),
                            "host_ms": (time.perf_counter() - t0) * 1e3}

        ths = [threading.Thread(target=lane_worker, args=(i, d, k, c)) for i, (d, k, c) in enumerate(lanes)]
        t0 = time.perf_counter()
        for t in ths:
            t.start()
        for t in ths:
            t.join(timeout=f.deadline_seconds + 5)
        host_ms = (time.perf_counter() - t0) * 1e3
        total = sum(r["bytes"] for r in results.values())
        gib = self.world.lane_gibps
        path_stats = [{"kind": r["kind"], "direction": direction,
                       "relay_device": -1 if r["kind"] == "direct" else r["device"],
                       "bytes": r["bytes"], "chunk_count": r["chunks"],
                       "model_ms": r["bytes"] / (gib * (1 << 30)) * 1e3, "host_ms": r["host_ms"]}
                      for _, r in sorted(results.items())]
        measured = {"host_ms": host_ms, "path_stats": path_stats, "simulated": True}
        if errors:
            return ExecutionResult(ok=False, bytes_completed=total, error="; ".join(errors), measured=measured)
        return ExecutionResult(ok=True, bytes_completed=total, measured=measured)


class _MockLanding:
    """The fused landing ops on host memory, chunk by chunk, with the same
    addressing rules as the GPU kernels: unit scatter / gather through the
    KV layout and bf16 -> e4m3 block quantisation (the OCP oracle)."""

    def __init__(self, spec, h2d: bool, src: BufferRegistration, dst: BufferRegistration,
                 buffers: dict) -> None:
        from ..daemon.landing import unit_addresses

        self.spec, self.h2d = spec, h2d
        self.host, self.dev = (src, dst) if h2d else (dst, src)
        buffers.setdefault(self.dev.buffer_id, self.dev)
        if spec.units_op:
            self.units = unit_addresses(spec, lambda b: int(buffers[b].address))
        if spec.op == "adamw":
            self.grads = int(buffers[spec.adam_params["grads_buffer"]].address)

    def move(self, so: int, do: int, n: int) -> None:
        spec = self.spec
        hbase = int(self.host.address)
        if spec.op == "adamw":
            self._adamw(hbase, so, n)
            return
        if spec.units_op:
            u = spec.unit_bytes
            host_off, pos = (so, do) if self.h2d else (do, so)
            if pos % u or n % u:
                raise ValueError("chunk is not a whole number of units")
            for k in range(n // u):
                ua = int(self.units[pos // u + k])
                h = hbase + host_off + k * u
                if self.h2d:
                    ctypes.memmove(ua, h, u)
                else:
                    ctypes.memmove(h, ua, u)
            return
        from ..utils.fp8 import block_quant

        ts = sorted(spec.tensors, key=lambda t: t.host_offset)
        t = next(t for t in reversed(ts) if t.host_offset <= so)
        rb = 2 * t.cols
        row0, rows = (so - t.host_offset) // rb, n // rb
        raw = np.ctypeslib.as_array((ctypes.c_uint16 * (n // 2)).from_address(hbase + so)).copy()
        x = (raw.astype(np.uint32) << 16).view(np.float32).reshape(rows, t.cols)
        q, sc = block_quant(x)
        dbase = int(self.dev.address)
        ctypes.memmove(dbase + t.q_offset + row0 * t.cols, q.ctypes.data, q.nbytes)
        ctypes.memmove(dbase + t.scales_offset + (row0 // 128) * (t.cols // 128) * 4, sc.ctypes.data, sc.nbytes)


    def _adamw(self, hbase: int, so: int, n: int) -> None:
        """The kernel's AdamW (float32, same operation order) on host tiles."""
        from ..daemon.landing import ADAM_TILE_BYTES, ADAM_TILE_PARAMS

        a = self.spec.adam_params
        f32 = np.float32
        lr, b1, b2, eps, wd, gs = (float(a[k]) for k in ("lr", "beta1", "beta2", "eps", "weight_decay",
                                                          "grad_scale"))
        t = int(a["step"])
        # factors formed in double and rounded once, as the kernel's host side does
        decay, fb2, omb1, omb2 = f32(1.0 - lr * wd), f32(b2), f32(1.0 - b1), f32(1.0 - b2)
        step_size = f32(lr / (1.0 - b1 ** t))
        sqrt_bc2 = f32(np.sqrt(1.0 - b2 ** t))
        eps, gs = f32(eps), f32(gs)
        nparams = int(a["nparams"])
        tiles = n // ADAM_TILE_BYTES
        st = np.ctypeslib.as_array((ctypes.c_float * (n // 4)).from_address(hbase + so)).reshape(tiles, 3,
                                                                                               ADAM_TILE_PARAMS)
        p0 = so // ADAM_TILE_BYTES * ADAM_TILE_PARAMS
        cnt = max(0, min(tiles * ADAM_TILE_PARAMS, nparams - p0))
        graw = np.ctypeslib.as_array((ctypes.c_uint16 * cnt).from_address(self.grads + 2 * p0))
        g = (graw.astype(np.uint32) << 16).view(np.float32) * gs
        flat = st.transpose(1, 0, 2).reshape(3, -1)[:, :cnt].copy()
        mast, m, v = flat
        p = mast * decay
        m = m + omb1 * (g - m)
        v = v * fb2 + (g * g) * omb2
        p = p - step_size * (m / (np.sqrt(v) / sqrt_bc2 + eps))
        full = st.transpose(1, 0, 2).reshape(3, -1).copy()
        full[0, :cnt], full[1, :cnt], full[2, :cnt] = p, m, v
        st[:] = full.reshape(3, tiles, ADAM_TILE_PARAMS).transpose(1, 0, 2)
        bits = p.astype(np.float32).view(np.uint32)
        rounded = ((bits + np.uint32(0x7FFF) + ((bits >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
        out = np.ctypeslib.as_array((ctypes.c_uint16 * cnt).from_address(int(self.dev.address) + 2 * p0))
        out[:] = rounded


def chunk_lane_map(trace: list[dict[str, Any]]) -> dict[int, int]:
    """src_offset -> lane for every traced chunk (raises if a chunk moved twice)."""
    out: dict[int, int] = {}
    for rec in trace:
        if rec["src_offset"] in out:
            raise AssertionError(f"chunk at {rec['src_offset']} moved twice")
        out[rec["src_offset"]] = rec["lane"]
    return out


class MockCudaBackend:
    """Stand-in for the CUDA backend in worker tests: IPC handles are 64
    random bytes mapped to in-process addresses; host registration is
    recorded, not performed.  Like CUDA, a handle names a whole allocation:
    ``allocations`` (base -> bytes) declares them, and a pointer inside one
    exports the allocation's handle (mapped at its base)."""

    def __init__(self) -> None:
        self.handles: dict[bytes, int] = {}
        self.open: dict[int, bytes] = {}
        self.registered: dict[int, int] = {}
        self.allocations: dict[int, int] = {}
        self.device = 0

    def set_device(self, device_index: int) -> None:
        self.device = int(device_index)

    def _base(self, device_ptr: int) -> int:
        for base, size in self.allocations.items():
            if base <= int(device_ptr) < base + size:
                return base
        return int(device_ptr)

    def device_allocation_offset(self, device_ptr: int) -> int:
        return int(device_ptr) - self._base(device_ptr)

    def export_device_ipc_handle(self, device_ptr: int) -> bytes:
        import os

        h = os.urandom(64)
        self.handles[h] = self._base(device_ptr)
        return h

    def open_device_ipc_handle(self, handle, device_index: int = 0) -> int:
        h = bytes.fromhex(handle) if isinstance(handle, str) else bytes(handle)
        if h not in self.handles:
            raise RuntimeError("unknown CUDA IPC handle")
        ptr = self.handles[h]
        self.open[ptr] = h
        return ptr

    def close_device_ipc_handle(self, device_ptr: int) -> None:
        self.open.pop(int(device_ptr), None)

    def register_host_memory(self, host_ptr: int, nbytes: int) -> None:
        self.registered[int(host_ptr)] = int(nbytes)

    def unregister_host_memory(self, host_ptr: int) -> None:
        self.registered.pop(int(host_ptr), None)


class MockWorkerExecutor:
    """Worker executor over the mock lanes: runs the ticket's scoped plan
    (direct + authorized relays) between the bound resources' addresses."""

    def __init__(self, plane: MockDataPlane | None = None) -> None:
        self.plane = plane or MockDataPlane()
        self.calls = 0

    def execute(self, request, staging_slot):
        from ..worker.helper import _failed

        return _failed(request, staging_slot, "mock worker execution requires bound resources")

    def execute_bound(self, request, staging_slot, resources):
        from ..worker.cuda_executor import scoped_plan
        from ..worker.helper import WorkerTransferResult, WorkerTransferState, _failed

        self.calls += 1
        dp = request.data_plane
        h2d = dp.direction == "h2d"
        target = int((dp.dst_handle if h2d else dp.src_handle).device_index or 0)
        plan = scoped_plan(request, target)
        lanes = []
        for a in plan["assignments"]:
            p = a["path"]
            dev = target if p["kind"] == "direct" else int(p["relay_device"])
            lanes.append((dev, p["kind"], [(c["src_offset"], c["dst_offset"], c["bytes"]) for c in assignment_chunks(a)]))
        src, sb, dst, db = ((resources.host_ptr, resources.host_bytes, resources.device_ptr, resources.device_bytes)
                            if h2d else
                            (resources.device_ptr, resources.device_bytes, resources.host_ptr, resources.host_bytes))
        r = self.plane.run_lanes(dp.direction, src, sb, dst, db, lanes, transfer_id=request.transfer_id)
        if not r.ok:
            return _failed(request, staging_slot, r.error)
        d_c = sum(len(c) for _d, k, c in lanes if k == "direct")
        return WorkerTransferResult(request.transfer_id, WorkerTransferState.COMPLETE, bytes_completed=r.bytes_completed,
                                    metadata={"executor": "mock_worker", "staging_slot_id": staging_slot.slot_id,
                                              "path": f"{'pool' if d_c else 'relay'}_{dp.direction}",
                                              "path_stats": r.measured.get("path_stats", [])})


__all__ = ["FaultPlan", "MockCudaBackend", "MockDataPlane", "MockLaneError", "MockWorkerExecutor", "MockWorld",
           "chunk_lane_map"]
