"""Runtime layer between plans and the native engine.

* ``RuntimeOptions`` - the reference's option set (chunk size, staging
  slots, profiling, planner thresholds, daemon hints; turbobus/runtime_engine.py:45-107)
  plus the engine knobs of this implementation (CTAs per lane, checksum,
  adaptive lane weights).
* ``PoolRuntime`` - a persistent runtime with the reference ``Runtime``'s
  method names (``init``, ``profile``, ``fetch_plan_to_gpu``,
  ``offload_plan_to_cpu``, ``wait``, ``stats``, ``run_dummy_compute``) over
  one ``PoolEngine``; created once and reused for every transfer.
* plan / profile converters between the daemon's dict formats and engine lanes.
"""

from __future__ import annotations

from .planner_types import assignment_chunks

import json
import time
from dataclasses import dataclass, field
from pathlib import Path
from collections.abc import Mapping
from typing import Any, Iterable, Sequence

from .plan_trace import transfer_plan_to_dict
from .schema import TransferMode


@dataclass
class RuntimeOptions:
    chunk_bytes: int = 16 * 1024 * 1024
    staging_slots: int = 3
    enable_peer_access: bool = True
    profile_bytes: int = 256 * 1024 * 1024
    profile_on_first_transfer: bool = True
    profile_cache_enabled: bool = True
    transfer_mode: TransferMode | str = TransferMode.POOL
    min_chunks_for_relay: int = 2
    min_pool_bytes: int = 12 * 1024 * 1024
    relay_min_effective_bw_gbps: float = 0.0
    relay_min_direct_ratio: float = 0.0
    enable_dynamic_weights: bool = True
    dynamic_weight_alpha: float = 0.5
    daemon_socket_path: str | None = None
    daemon_max_inflight_chunks: int = 8
    daemon_profile_max_age_seconds: float = 3600.0
    ctas_per_lane: int = 4
    checksum: bool = True
    timeout_s: float = 10.0

    @classmethod
    def from_tuning_json(cls, path: str | Path) -> "RuntimeOptions":
        best = read_json(path).get("best")
        if not isinstance(best, dict):
            raise ValueError("tuning JSON does not contain a 'best' object")
        return cls(chunk_bytes=int(best["chunk_bytes"]), staging_slots=int(best["staging_slots"]))

    @classmethod
    def from_profile_json(cls, path: str | Path) -> "RuntimeOptions":
        cfg = read_json(path).get("config", {})
        if not isinstance(cfg, dict):
            raise ValueError("profile JSON contains an invalid 'config' object")
        d = cls()
        return cls(chunk_bytes=int(cfg.get("chunk_bytes", d.chunk_bytes)),
                   staging_slots=int(cfg.get("staging_slots", d.staging_slots)),
                   profile_bytes=int(cfg.get("profile_bytes", d.profile_bytes)))

    def planner_options(self):
        from .planner_engine import PlannerEngineOptions

        return PlannerEngineOptions(min_chunks_for_relay=self.min_chunks_for_relay,
                                    relay_min_effective_bw_gbps=self.relay_min_effective_bw_gbps,
                                    relay_min_direct_ratio=self.relay_min_direct_ratio)

    def to_native(self):
        """The native engine's options for these settings (``_C.EngineOptions``;
        the reference returns its ``_turbobus.RuntimeOptions``,
        turbobus/runtime_engine.py:87-107).  Planning fields stay on the
        Python side (``planner_options``); the engine takes the staging ring
        geometry, lane-kernel width, device timeout and peer setting."""
        from ._native import native

        o = native().EngineOptions()
        o.slot_bytes = max(int(self.chunk_bytes), 1 << 20)
        o.slots = int(self.staging_slots)
        o.ctas_per_lane = int(self.ctas_per_lane)
        o.timeout_s = float(self.timeout_s)
        o.enable_peer_access = bool(self.enable_peer_access)
        return o


def read_json(path: str | Path) -> dict:
    with Path(path).open("r", encoding="utf-8") as fh:
        data = json.load(fh)
    if not isinstance(data, dict):
        raise ValueError("expected a JSON object")
    return data


# ---- profiles ----------------------------------------------------------------------------

@dataclass(frozen=True)
class SimpleProfileRelay:
    relay_device: int
    target_device: int
    h2d_bw_gbps: float
    d2h_bw_gbps: float
    p2p_bw_gbps: float
    effective_bw_gbps: float
    effective_d2h_bw_gbps: float
    p2p_enabled: bool


@dataclass(frozen=True)
class SimpleProfileResult:
    target_device: int
    direct_h2d_bw_gbps: float
    direct_d2h_bw_gbps: float
    relays: list[SimpleProfileRelay] = field(default_factory=list)
    concurrent: Mapping[str, Any] = field(default_factory=dict)


def _g(o, k, d=None):
    return o.get(k, d) if isinstance(o, Mapping) else getattr(o, k, d)


def profile_to_daemon_dict(profile) -> dict[str, object]:
    out = {
        "target_device": int(_g(profile, "target_device", 0)),
        "direct_h2d_bw_gbps": float(_g(profile, "direct_h2d_bw_gbps", 0.0) or 0.0),
        "direct_d2h_bw_gbps": float(_g(profile, "direct_d2h_bw_gbps", 0.0) or 0.0),
        "relays": [{"relay_device": int(_g(r, "relay_device")),
                    "target_device": int(_g(r, "target_device", 0)),
                    **{k: float(_g(r, k, 0.0) or 0.0) for k in ("h2d_bw_gbps", "d2h_bw_gbps", "p2p_bw_gbps",
                                                                 "effective_bw_gbps", "effective_d2h_bw_gbps")},
                    "p2p_enabled": bool(_g(r, "p2p_enabled", False))} for r in (_g(profile, "relays", []) or [])],
    }
    conc = _g(profile, "concurrent", None)
    if conc:
        out["concurrent"] = dict(conc)
    return out


def profile_from_daemon_entry(entry: Mapping, target_gpu: int) -> SimpleProfileResult:
    prof = entry.get("profile")
    if not isinstance(prof, Mapping):
        raise ValueError("daemon profile entry has no profile object")
    h2d = float(prof.get("direct_h2d_bw_gbps", 0.0) or 0.0)
    if h2d <= 0.0:
        raise ValueError("daemon profile direct_h2d_bw_gbps must be positive")
    relays = []
    for r in prof.get("relays", []) or []:
        if not isinstance(r, Mapping):
            raise ValueError("daemon profile relay must be an object")
        relays.append(SimpleProfileRelay(
            relay_device=int(r["relay_device"]), target_device=int(r.get("target_device", target_gpu)),
            **{k: float(r.get(k, 0.0) or 0.0) for k in ("h2d_bw_gbps", "d2h_bw_gbps", "p2p_bw_gbps",
                                                         "effective_bw_gbps", "effective_d2h_bw_gbps")},
            p2p_enabled=bool(r.get("p2p_enabled", False))))
    return SimpleProfileResult(int(prof.get("target_device", target_gpu)), h2d,
                               float(prof.get("direct_d2h_bw_gbps", 0.0) or 0.0), relays,
                               dict(prof.get("concurrent", {}) or {}))


def daemon_profile_is_fresh(entry: Mapping, max_age_seconds: float) -> bool:
    if max_age_seconds <= 0:
        return True
    updated = float(entry.get("updated_at", 0.0) or 0.0)
    return updated > 0.0 and (time.time() - updated) <= float(max_age_seconds)


# ---- plans -> engine lanes ---------------------------------------------------------------------

def plan_to_lanes(plan, target: int, *, source_bytes: int | None = None,
                  destination_bytes: int | None = None):
    """Validate a plan (dict or object) and convert it into engine lanes:
    no disabled path, chunk bytes summing to ``total_bytes``, chunks inside
    both buffers (reference checks: turbobus/runtime_engine.py:338-410)."""
    from .parallel.engine import make_lane

    payload = dict(plan) if isinstance(plan, Mapping) else transfer_plan_to_dict(plan)
    total = int(payload.get("total_bytes", 0))
    if total < 0:
        raise ValueError("transfer plan total_bytes must be non-negative")
    if int(payload.get("chunk_bytes", 16 << 20)) <= 0:
        raise ValueError("transfer plan chunk_bytes must be positive")
    lanes, seen = [], 0
    for asg in payload.get("assignments", []) or []:
        if not isinstance(asg, Mapping) or not isinstance(asg.get("path"), Mapping):
            raise ValueError("transfer plan assignment must be an object")
        p = asg["path"]
        if not bool(p.get("enabled", True)):
            raise ValueError("transfer plan contains a disabled path")
        kind = str(p.get("kind", "")).lower()
        if kind not in ("direct", "relay"):
            raise ValueError(f"unsupported transfer plan path: {kind}")
        chunks = []
        for c in assignment_chunks(asg):
            s, d, n = int(c.get("src_offset", 0)), int(c.get("dst_offset", 0)), int(c.get("bytes", 0))
            if s < 0 or d < 0 or n <= 0:
                raise ValueError("transfer plan chunk offsets must be non-negative and bytes positive")
            if source_bytes is not None and s + n > source_bytes:
                raise ValueError("range source extends past source buffer")
            if destination_bytes is not None and d + n > destination_bytes:
                raise ValueError("range destination extends past destination buffer")
            chunks.append((s, d, n))
            seen += n
        if chunks:
            dev = int(target) if kind == "direct" else int(p.get("relay_device", -1))
            lanes.append(make_lane(dev, chunks))
    if total > 0 and not lanes:
        raise ValueError("transfer plan has no chunk assignments")
    if lanes and seen != total:
        raise ValueError("transfer plan total_bytes must match assigned chunk bytes")
    return lanes


# ---- stats objects mirroring the reference's native stats ---------------------------------------

@dataclass
class PathStats:
    kind: str
    direction: str
    target_device: int
    relay_device: int
    bytes: int
    chunks: int
    cuda_elapsed_ms: float
    gib_per_second: float


@dataclass
class TransferStats:
    bytes: int = 0
    direct_bytes: int = 0
    relay_bytes: int = 0
    submit_to_complete_ms: float = 0.0
    cuda_elapsed_ms: float = 0.0
    gib_per_second: float = 0.0
    submit_gib_per_second: float = 0.0
    direct_chunks: int = 0
    relay_chunks: int = 0
    relay_devices: list[int] = field(default_factory=list)
    relay_device_bytes: list[int] = field(default_factory=list)
    relay_device_chunks: list[int] = field(default_factory=list)
    path_stats: list[PathStats] = field(default_factory=list)
    checksums: Any = None
    ok: bool = True
    error: str = ""


def stats_from_result(res, direction: str, target: int) -> TransferStats:
    st = TransferStats(bytes=res.bytes, submit_to_complete_ms=res.submit_to_complete_ms,
                       cuda_elapsed_ms=res.cuda_ms, gib_per_second=res.gib_per_s, checksums=res.checksums,
                       ok=res.ok, error=res.error)
    gib = float(1 << 30)
    if res.submit_to_complete_ms > 0:
        st.submit_gib_per_second = (res.bytes / gib) / (res.submit_to_complete_ms / 1e3)
    for l in res.lanes:
        ps = PathStats("direct" if l.direct else "relay", direction, target, -1 if l.direct else l.device,
                       l.bytes, l.chunks, l.cuda_ms, (l.bytes / gib) / (l.cuda_ms / 1e3) if l.cuda_ms > 0 else 0.0)
        st.path_stats.append(ps)
        if l.direct:
            st.direct_bytes += l.bytes
            st.direct_chunks += l.chunks
        else:
            st.relay_bytes += l.bytes
            st.relay_chunks += l.chunks
            st.relay_devices.append(l.device)
            st.relay_device_bytes.append(l.bytes)
            st.relay_device_chunks.append(l.chunks)
    return st


@dataclass
class DummyComputeStats:
    elements: int
    iterations: int
    cuda_elapsed_ms: float


class RuntimeHandle:
    def __init__(self, tid: int, direction: str) -> None:
        self.id = tid
        self.direction = direction
        self.status = "submitted"
        self.error = ""


class PoolRuntime:
    """Persistent runtime over one ``PoolEngine`` (reference Runtime API)."""

    def __init__(self, options: RuntimeOptions | None = None) -> None:
        self.options = options or RuntimeOptions()
        self._engine = None
        self.target_device = -1
        self.relay_devices: list[int] = []
        self._profile = None
        self._last_plan: dict | None = None
        self._results: dict[int, TransferStats] = {}
        self._balancer = None

    def init(self, target_device: int, relay_devices: Sequence[int]) -> None:
        from .parallel.balance import LaneBalancer
        from .parallel.engine import PoolEngine

        self.target_device = int(target_device)
        self.relay_devices = [int(d) for d in relay_devices if int(d) != int(target_device)]
        o = self.options
        self._engine = PoolEngine([self.target_device, *self.relay_devices],
                                  slot_bytes=max(int(o.chunk_bytes), 1 << 20), slots=int(o.staging_slots),
                                  ctas_per_lane=int(o.ctas_per_lane), timeout_s=float(o.timeout_s),
                                  enable_peer_access=bool(o.enable_peer_access))
        self._balancer = LaneBalancer(alpha=o.dynamic_weight_alpha)

    @property
    def engine(self):
        if self._engine is None:
            raise RuntimeError("runtime is not initialized")
        return self._engine

    def profile(self, bytes_: int = 256 << 20, force: bool = False):
        from .parallel.linkprobe import probe_profile

        if self._engine is None:
            raise RuntimeError("runtime is not initialized")
        if force or self._profile is None or not self.options.profile_cache_enabled:
            self._profile = probe_profile(self._engine, self.target_device, self.relay_devices, int(bytes_))
        return self._profile

    def set_cached_profile(self, profile) -> None:
        if self._engine is None:
            raise RuntimeError("runtime is not initialized")
        self._profile = profile

    def cached_profile(self):
        return self._profile

    def planner_profile(self):
        return self._profile

    def last_plan(self) -> dict | None:
        return self._last_plan

    def _submit(self, direction: str, host_ptr: int, host_bytes: int, dev_ptr: int, dev_bytes: int, plan) -> RuntimeHandle:
        from .parallel.engine import D2H, H2D

        h2d = direction == "h2d"
        lanes = plan_to_lanes(plan, self.target_device, source_bytes=host_bytes if h2d else dev_bytes,
                              destination_bytes=dev_bytes if h2d else host_bytes)
        self._last_plan = dict(plan) if isinstance(plan, Mapping) else transfer_plan_to_dict(plan)
        tid = self.engine.submit(H2D if h2d else D2H, self.target_device, host_ptr, host_bytes, dev_ptr,
                                 dev_bytes, lanes, checksum=self.options.checksum)
        return RuntimeHandle(tid, direction)

    def fetch_plan_to_gpu(self, host_ptr: int, host_bytes: int, target_ptr: int, target_bytes: int, plan) -> RuntimeHandle:
        return self._submit("h2d", host_ptr, host_bytes, target_ptr, target_bytes, plan)

    def offload_plan_to_cpu(self, target_ptr: int, target_bytes: int, host_ptr: int, host_bytes: int, plan) -> RuntimeHandle:
        return self._submit("d2h", host_ptr, host_bytes, target_ptr, target_bytes, plan)

    def wait(self, handle: RuntimeHandle) -> None:
        res = self.engine.wait(handle.id)
        st = stats_from_result(res, handle.direction, self.target_device)
        self._results[handle.id] = st
        if self._balancer is not None and res.ok:
            self._balancer.observe(self.target_device, handle.direction, res)
        handle.status = "complete" if res.ok else "failed"
        handle.error = res.error
        if not res.ok:
            raise RuntimeError(f"transfer {handle.id} failed: {res.error}")

    def stats(self, handle: RuntimeHandle) -> TransferStats:
        if handle.id not in self._results:
            raise ValueError("unknown transfer handle (wait first)")
        return self._results[handle.id]

    def run_dummy_compute(self, device_ptr: int, elements: int, iterations: int) -> DummyComputeStats:
        import torch

        from ._native import native

        dev = self.target_device
        s = torch.cuda.Stream(device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.device(dev), torch.cuda.stream(s):
            e0.record(s)
            native().interference(int(device_ptr), int(elements), int(iterations), 0, s.cuda_stream)
            e1.record(s)
        s.synchronize()
        return DummyComputeStats(int(elements), int(iterations), e0.elapsed_time(e1))

    # -- tensor conveniences -------------------------------------------------------------------
    def lane_weights(self, direction: str) -> list[float] | None:
        if self._balancer is None:
            return None
        return self._balancer.weights(self.target_device, direction, [self.target_device, *self.relay_devices])

    def plan_for(self, total_bytes: int, direction: str = "h2d"):
        from .parallel.planning import plan_lanes

        devs = [self.target_device, *self.relay_devices]
        if self.options.transfer_mode in (TransferMode.DIRECT, "direct") or total_bytes < self.options.min_pool_bytes:
            devs = [self.target_device]
        w = self.lane_weights(direction) if self.options.enable_dynamic_weights else None
        if w is not None and len(w) != len(devs):
            w = None
        return plan_lanes(total_bytes, int(self.options.chunk_bytes), devs, self.target_device, bw_gibps=w)

    def fetch(self, cpu_tensor, gpu_tensor) -> TransferStats:
        from .parallel.engine import H2D

        n = validate_transfer_tensors(cpu_tensor, gpu_tensor, self.target_device, "h2d")
        lanes = self.plan_for(n, "h2d")
        res = self.engine.run(H2D, self.target_device, cpu_tensor.data_ptr(), n, gpu_tensor.data_ptr(), n, lanes,
                              checksum=self.options.checksum)
        if self._balancer is not None and res.ok:
            self._balancer.observe(self.target_device, "h2d", res)
        res.raise_for_status()
        return stats_from_result(res, "h2d", self.target_device)

    def offload(self, gpu_tensor, cpu_tensor) -> TransferStats:
        from .parallel.engine import D2H

        n = validate_transfer_tensors(cpu_tensor, gpu_tensor, self.target_device, "d2h")
        lanes = self.plan_for(n, "d2h")
        res = self.engine.run(D2H, self.target_device, cpu_tensor.data_ptr(), n, gpu_tensor.data_ptr(), n, lanes,
                              checksum=self.options.checksum)
        if self._balancer is not None and res.ok:
            self._balancer.observe(self.target_device, "d2h", res)
        res.raise_for_status()
        return stats_from_result(res, "d2h", self.target_device)


def validate_transfer_tensors(cpu_tensor, gpu_tensor, target_gpu: int, direction: str) -> int:
    import torch

    if direction not in ("h2d", "d2h"):
        raise ValueError(f"unsupported transfer direction: {direction}")
    if not isinstance(cpu_tensor, torch.Tensor) or not isinstance(gpu_tensor, torch.Tensor):
        raise TypeError("cpu_tensor and gpu_tensor must be torch.Tensor")
    if cpu_tensor.device.type != "cpu":
        raise ValueError("cpu_tensor must be on CPU")
    if not cpu_tensor.is_pinned():
        raise ValueError("cpu_tensor must be pinned memory")
    if gpu_tensor.device.type != "cuda":
        raise ValueError("gpu_tensor must be on CUDA")
    if gpu_tensor.device.index != target_gpu:
        raise ValueError("gpu_tensor must be on the runtime target_gpu")
    if not cpu_tensor.is_contiguous() or not gpu_tensor.is_contiguous():
        raise ValueError("cpu_tensor and gpu_tensor must be contiguous")
    cb = cpu_tensor.numel() * cpu_tensor.element_size()
    gb = gpu_tensor.numel() * gpu_tensor.element_size()
    if direction == "h2d":
        if gb < cb:
            raise ValueError("gpu_tensor is smaller than cpu_tensor")
        return cb
    if cb < gb:
        raise ValueError("cpu_tensor is smaller than gpu_tensor")
    return gb


class TransferHandle:
    """Handle over a runtime transfer: ``wait()`` then ``stats``."""

    def __init__(self, runtime: PoolRuntime, native_handle: RuntimeHandle,
                 daemon_reservations: list[str] | None = None) -> None:
        self.runtime = runtime
        self.native = native_handle
        self._daemon_reservations = list(daemon_reservations or [])
        self._status = "submitted"
        self._stats = None
        self.error = ""

    @property
    def id(self) -> int:
        return self.native.id

    @property
    def status(self) -> str:
        return self._status

    @property
    def done(self) -> bool:
        return self._status == "complete"

    @property
    def stats(self):
        return self._stats

    def wait(self) -> None:
        if self.done:
            return
        try:
            self.runtime.wait(self.native)
        except Exception as exc:
            self._status, self.error = "failed", str(exc)
            raise
        self._status = "complete"
        self._stats = self.runtime.stats(self.native)

    def __repr__(self) -> str:
        return f"TransferHandle(id={self.id}, status={self.status})"


def range_fields(item) -> tuple[int, int, int]:
    if isinstance(item, Mapping):
        return int(item["src_offset"]), int(item["dst_offset"]), int(item["bytes"])
    if isinstance(item, Sequence) and not isinstance(item, (str, bytes, bytearray)):
        if len(item) != 3:
            raise ValueError("range tuples must be (src_offset, dst_offset, bytes)")
        return int(item[0]), int(item[1]), int(item[2])
    return int(item.src_offset), int(item.dst_offset), int(item.bytes)


def validate_ranges(ranges: Iterable, source_bytes: int, destination_bytes: int) -> list[tuple[int, int, int]]:
    out = []
    for item in ranges:
        s, d, n = range_fields(item)
        if s < 0 or d < 0 or n <= 0:
            raise ValueError("range offsets must be non-negative and bytes must be positive")
        if s + n > source_bytes:
            raise ValueError("range source extends past source tensor")
        if d + n > destination_bytes:
            raise ValueError("range destination extends past destination tensor")
        out.append((s, d, n))
    if not out:
        raise ValueError("at least one non-empty range is required")
    return out


__all__ = ["DummyComputeStats", "PathStats", "PoolRuntime", "RuntimeHandle", "RuntimeOptions", "SimpleProfileRelay",
           "SimpleProfileResult", "TransferHandle", "TransferStats", "daemon_profile_is_fresh", "plan_to_lanes",
           "profile_from_daemon_entry", "profile_to_daemon_dict", "range_fields", "stats_from_result",
           "validate_ranges", "validate_transfer_tensors"]
