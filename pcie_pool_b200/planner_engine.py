"""Chunk planner.

Turns (bytes or ranges, chunk size, bandwidth profile, mode) into a
``PlannerTransferPlan``: the direct lane plus eligible relay lanes, each with
an ordered chunk list.

Path eligibility follows the reference (turbobus/planner_engine.py:96-151):
the direct path when its bandwidth is positive and the mode is not ``relay``;
a relay when peer access is enabled, its effective bandwidth is positive, at
least ``relay_min_effective_bw_gbps`` and at least ``relay_min_direct_ratio``
times the direct bandwidth.  ``pool`` mode with fewer than
``min_chunks_for_relay`` chunks plans direct only.

Assignment policies:
  * ``legacy``           - argmin(assigned_bytes / bw) per chunk, ties to the
                           lower path index (the reference's rule).
  * ``earliest_finish``  - each chunk to the lane that would finish it first,
                           counting a per-chunk lane latency; lanes sharing an
                           uplink are first scaled to the group's concurrent
                           capacity.  This is the default.
The per-chunk loops run in the native planner core when it is built.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from collections.abc import Mapping
from typing import Iterable, Sequence

from .planner_types import (PlannerChunk, PlannerPath, PlannerPathAssignment,
                            PlannerTransferPlan)
from .schema import TransferMode
from .transfer import coerce_range

POLICIES = ("legacy", "earliest_finish")
CHUNK_CANDIDATES = tuple(1 << s for s in range(20, 27))  # 1 .. 64 MiB


@dataclass(frozen=True)
class PlannerEngineOptions:
    min_chunks_for_relay: int = 2
    relay_min_effective_bw_gbps: float = 0.0
    relay_min_direct_ratio: float = 0.0
    policy: str = "earliest_finish"
    # per-lane fixed cost of one chunk (seconds); keyed by lane device, -1 = default
    lane_latency_s: Mapping[int, float] = field(default_factory=dict)
    # lanes sharing a PCIe uplink: device -> group id, group id -> capacity (GiB/s)
    uplink_group: Mapping[int, int] = field(default_factory=dict)
    group_capacity_gbps: Mapping[int, float] = field(default_factory=dict)
    # cut chunks on multiples of this many bytes (fused-op tiles, KV units)
    align_bytes: int = 1
    # use a probed profile's concurrent lane set and rates when present
    use_concurrent_profile: bool = True
    # ``blocked``: each lane takes one contiguous span (after assignment)
    layout: str = "interleaved"

    def __post_init__(self) -> None:
        if self.policy not in POLICIES:
            raise ValueError(f"unknown planner policy {self.policy!r}")
        if self.align_bytes < 1:
            raise ValueError("align_bytes must be >= 1")
        if self.layout not in ("interleaved", "blocked"):
            raise ValueError("layout must be 'interleaved' or 'blocked'")


class PlannerEngine:
    def __init__(self, options: PlannerEngineOptions | None = None) -> None:
        self.options = options or PlannerEngineOptions()

    # ---- public -----------------------------------------------------------------
    def plan(self, total_bytes: int, chunk_bytes: int, profile,
             mode: TransferMode | str = TransferMode.POOL, *,
             direction: str = "h2d") -> PlannerTransferPlan:
        import numpy as np

        total = max(0, int(total_bytes))
        if total == 0:
            return PlannerTransferPlan()
        chunk = int(chunk_bytes)
        if chunk <= 0:
            raise ValueError("chunk_bytes must be greater than zero")
        chunk = self._aligned_chunk(chunk)
        offs = np.arange(0, total, chunk, dtype=np.int64)
        return self._finish(offs, offs, np.minimum(chunk, total - offs), total, chunk, profile, mode,
                            direction)

    def plan_ranges(self, ranges: Iterable, chunk_bytes: int, profile,
                    mode: TransferMode | str = TransferMode.POOL, *,
                    direction: str = "h2d") -> PlannerTransferPlan:
        import numpy as np

        chunk = int(chunk_bytes)
        if chunk <= 0:
            raise ValueError("chunk_bytes must be greater than zero")
        chunk = self._aligned_chunk(chunk)
        srcs, dsts, sizes = [], [], []
        total = 0
        for item in ranges:
            r = _range_tuple(item)
            if r[2] <= 0:
                continue
            total += r[2]
            o = np.arange(0, r[2], chunk, dtype=np.int64)
            srcs.append(o + r[0])
            dsts.append(o + r[1])
            sizes.append(np.minimum(chunk, r[2] - o))
        if not srcs:
            return PlannerTransferPlan()
        return self._finish(np.concatenate(srcs), np.concatenate(dsts), np.concatenate(sizes), total, chunk,
                            profile, mode, direction)

    def auto_chunk_bytes(self, total_bytes: int, profile, *, direction: str = "h2d",
                         candidates: Sequence[int] = CHUNK_CANDIDATES,
                         max_chunk: int | None = None) -> int:
        """Chunk size with the smallest estimated makespan over the lanes the
        profile makes eligible (per-chunk latency vs. pipeline fill)."""
        paths = self.build_paths(profile, TransferMode.POOL, direction)
        if not paths:
            raise RuntimeError("no enabled transfer path is available")
        bw, lat = self._lane_model(paths)
        cands = [self._aligned_chunk(c) for c in candidates if max_chunk is None or c <= max_chunk]
        if not cands:
            raise ValueError("no chunk-size candidate fits")
        C = _native_planner()
        if C is not None:
            return int(C.choose_chunk_bytes(int(total_bytes), cands, bw, lat))
        return min(cands, key=lambda c: _estimate(int(total_bytes), c, bw, lat))

    def build_paths(self, profile, mode: TransferMode | str, direction: str) -> list[PlannerPath]:
        mode = TransferMode(mode)
        paths: list[PlannerPath] = []
        direct_bw = _direct_bw(profile, direction)
        if mode is not TransferMode.RELAY and direct_bw > 0.0:
            paths.append(PlannerPath(
                kind="direct", direction=direction,
                target_device=int(_get(profile, "target_device", 0)), relay_device=-1,
                h2d_bw_gbps=float(_get(profile, "direct_h2d_bw_gbps", 0.0) or 0.0),
                d2h_bw_gbps=float(_get(profile, "direct_d2h_bw_gbps", 0.0) or direct_bw),
                p2p_bw_gbps=0.0, effective_bw_gbps=float(direct_bw), enabled=True))
        if mode is TransferMode.DIRECT:
            return paths
        o = self.options
        conc = None
        if o.use_concurrent_profile and o.policy != "legacy":
            c = (_get(profile, "concurrent", None) or {}).get(direction)
            if isinstance(c, Mapping) and c.get("lanes"):
                conc = ({int(x) for x in c["lanes"]}, {int(k): float(v) for k, v in
                                                       (c.get("lane_gibps") or {}).items()})
        if conc is not None and paths:
            tgt = paths[0].target_device
            if tgt in conc[1]:
                paths[0] = PlannerPath(**{**paths[0].as_dict(), "effective_bw_gbps": conc[1][tgt]})
        for relay in _get(profile, "relays", []) or []:
            dev = int(_get(relay, "relay_device", -1))
            if conc is not None and (dev not in conc[0] or dev not in conc[1]):
                continue
            eff = conc[1][dev] if conc is not None else _relay_bw(relay, direction)
            if not _get(relay, "p2p_enabled", False) or eff <= 0.0:
                continue
            if eff < o.relay_min_effective_bw_gbps:
                continue
            if direct_bw > 0.0 and o.relay_min_direct_ratio > 0.0 and eff < direct_bw * o.relay_min_direct_ratio:
                continue
            paths.append(PlannerPath(
                kind="relay", direction=direction,
                target_device=int(_get(relay, "target_device", _get(profile, "target_device", 0))),
                relay_device=int(_get(relay, "relay_device", -1)),
                h2d_bw_gbps=float(_get(relay, "h2d_bw_gbps", 0.0) or 0.0),
                d2h_bw_gbps=float(_get(relay, "d2h_bw_gbps", 0.0) or _get(relay, "h2d_bw_gbps", 0.0) or 0.0),
                p2p_bw_gbps=float(_get(relay, "p2p_bw_gbps", 0.0) or 0.0),
                effective_bw_gbps=float(eff), enabled=True, fabric_kind=_get(relay, "fabric_kind", None)))
        return paths

    # ---- internals --------------------------------------------------------------------
    def _aligned_chunk(self, chunk: int) -> int:
        a = self.options.align_bytes
        return chunk if a <= 1 else max(a, (chunk // a) * a)

    def _finish(self, src, dst, sizes, total: int, chunk: int, profile, mode,
                direction: str) -> PlannerTransferPlan:
        import numpy as np

        mode = TransferMode(mode)
        if mode is TransferMode.AUTO:
            mode = TransferMode.POOL
        if mode is TransferMode.POOL and sizes.size < self.options.min_chunks_for_relay:
            mode = TransferMode.DIRECT
        paths = self.build_paths(profile, mode, direction)
        if not paths:
            raise RuntimeError("no enabled transfer path is available")
        if sum(p.effective_bw_gbps for p in paths) <= 0.0:
            raise RuntimeError("enabled paths have zero effective bandwidth")
        idx = np.asarray(self._assign(sizes, paths), dtype=np.int64)
        out = []
        if self.options.layout == "blocked":
            # each lane takes one contiguous slice of the chunk sequence, kept
            # as runs (one per lane unless a range boundary splits it)
            counts = np.bincount(idx, minlength=len(paths))
            start = 0
            for p, n in zip(paths, counts):
                n = int(n)
                if n:
                    out.append(PlannerPathAssignment(p, runs=_runs(src[start:start + n], dst[start:start + n],
                                                                   sizes[start:start + n], chunk)))
                start += n
        else:
            for i, p in enumerate(paths):
                sel = np.flatnonzero(idx == i)
                if sel.size:
                    out.append(PlannerPathAssignment(p, tuple(
                        PlannerChunk(s_, d_, n_) for s_, d_, n_ in
                        zip(src[sel].tolist(), dst[sel].tolist(), sizes[sel].tolist()))))
        return PlannerTransferPlan(total_bytes=int(total), chunk_bytes=int(chunk), assignments=tuple(out))

    def _lane_model(self, paths: Sequence[PlannerPath]) -> tuple[list[float], list[float]]:
        o = self.options
        bw = [max(p.effective_bw_gbps, 1e-12) for p in paths]
        if o.uplink_group:
            groups = [int(o.uplink_group.get(p.lane_device, -1)) for p in paths]
            caps: dict[int, float] = dict(o.group_capacity_gbps)
            sums: dict[int, float] = {}
            for g, b in zip(groups, bw):
                if g >= 0:
                    sums[g] = sums.get(g, 0.0) + b
            bw = [b * (caps[g] / sums[g]) if g >= 0 and caps.get(g, 0.0) > 0.0 and sums[g] > caps[g]
                  else b for g, b in zip(groups, bw)]
        default_lat = float(o.lane_latency_s.get(-1, 0.0))
        lat = [float(o.lane_latency_s.get(p.lane_device, default_lat)) for p in paths]
        return bw, lat

    def _assign(self, sizes, paths: Sequence[PlannerPath]):
        import numpy as np

        policy = self.options.policy
        if len(paths) == 1:
            return np.zeros(len(sizes), dtype=np.int64)
        if policy == "legacy":
            bw = [max(p.effective_bw_gbps, 1e-12) for p in paths]
            lat: list[float] = []
        else:
            bw, lat = self._lane_model(paths)
        C = _native_planner()
        if C is None:
            return assign_python([int(x) for x in sizes], bw, lat, policy)
        pol = C.POLICY_LEGACY if policy == "legacy" else C.POLICY_EARLIEST_FINISH
        return np.asarray(C.assign_chunks(np.asarray(sizes, dtype=np.uint64), bw, lat, pol), dtype=np.int64)


def _runs(src, dst, sizes, chunk: int) -> tuple[tuple[int, int, int, int], ...]:
    """Runs of a contiguous slice of the chunk sequence: a new run starts
    where a chunk is not contiguous with the previous one on either side, or
    after a chunk shorter than ``chunk`` (a range's tail)."""
    import numpy as np

    if len(sizes) == 0:
        return ()
    brk = np.flatnonzero((src[1:] != src[:-1] + sizes[:-1]) | (dst[1:] != dst[:-1] + sizes[:-1])
                         | (sizes[:-1] != chunk)) + 1
    starts = np.concatenate(([0], brk))
    ends = np.concatenate((brk, [len(sizes)]))
    csum = np.concatenate(([0], np.cumsum(sizes)))
    return tuple((int(src[a]), int(dst[a]), int(csum[b] - csum[a]), int(chunk))
                 for a, b in zip(starts.tolist(), ends.tolist()))


def _native_planner():
    """The native planner (C++), or None when the extension is not built --
    a host-side computation whose Python twin (``assign_python`` /
    ``_estimate``) gives the same assignment, so planning also works on
    machines that never built the CUDA extension.  Errors inside a native
    call are not caught."""
    from ._native import native

    try:
        return native(build_if_missing=False)
    except RuntimeError:
        return None


def assign_python(sizes: Sequence[int], bw: Sequence[float], lat: Sequence[float],
                  policy: str) -> list[int]:
    """Pure-Python twin of the native assignment loop (same tie rules)."""
    out: list[int] = []
    if policy == "legacy":
        assigned = [0.0] * len(bw)
        for n in sizes:
            best, score = 0, math.inf
            for i, b in enumerate(bw):
                s = assigned[i] / b
                if s < score:
                    best, score = i, s
            out.append(best)
            assigned[best] += float(n)
        return out
    finish = [0.0] * len(bw)
    gib = float(1 << 30)
    for n in sizes:
        best, t_best = 0, math.inf
        for i, b in enumerate(bw):
            t = finish[i] + (lat[i] if lat else 0.0) + (n / gib) / b
            if t < t_best:
                best, t_best = i, t
        out.append(best)
        finish[best] = t_best
    return out


def _estimate(total: int, chunk: int, bw: Sequence[float], lat: Sequence[float]) -> float:
    sizes = [min(chunk, total - o) for o in range(0, total, chunk)]
    idx = assign_python(sizes, bw, lat, "earliest_finish")
    fin = [0.0] * len(bw)
    fill = 0.0
    for n, i in zip(sizes, idx):
        t = (lat[i] if lat else 0.0) + (n / float(1 << 30)) / bw[i]
        fin[i] += t
        fill = max(fill, t)
    return max(fin) + 0.5 * fill


def _get(obj, name: str, default=None):
    if isinstance(obj, Mapping):
        return obj.get(name, default)
    return getattr(obj, name, default)


def _direct_bw(profile, direction: str) -> float:
    key = "direct_h2d_bw_gbps" if direction == "h2d" else "direct_d2h_bw_gbps"
    bw = max(0.0, float(_get(profile, key, 0.0) or 0.0))
    if direction != "h2d" and bw <= 0.0:
        bw = max(0.0, float(_get(profile, "direct_h2d_bw_gbps", 0.0) or 0.0))
    return bw


def _relay_bw(relay, direction: str) -> float:
    key = "effective_bw_gbps" if direction == "h2d" else "effective_d2h_bw_gbps"
    bw = max(0.0, float(_get(relay, key, 0.0) or 0.0))
    if direction != "h2d" and bw <= 0.0:
        bw = max(0.0, float(_get(relay, "effective_bw_gbps", 0.0) or 0.0))
    return bw


def _range_tuple(item) -> tuple[int, int, int]:
    """(src, dst, bytes) of a range; empty ranges pass through to be skipped."""
    if isinstance(item, Mapping):
        t = (int(item["src_offset"]), int(item["dst_offset"]), int(item["bytes"]))
    elif isinstance(item, (tuple, list)):
        if len(item) != 3:
            raise ValueError("range tuples must be (src_offset, dst_offset, bytes)")
        t = (int(item[0]), int(item[1]), int(item[2]))
    else:
        t = (int(item.src_offset), int(item.dst_offset), int(item.bytes))
    if t[2] > 0:
        coerce_range(t)  # validates offsets
    return t


def plan_transfer(total_bytes: int, chunk_bytes: int, profile, mode: TransferMode | str = TransferMode.POOL,
                  *, direction: str = "h2d", options: PlannerEngineOptions | None = None) -> PlannerTransferPlan:
    return PlannerEngine(options).plan(total_bytes, chunk_bytes, profile, mode, direction=direction)


def plan_transfer_ranges(ranges: Iterable, chunk_bytes: int, profile,
                         mode: TransferMode | str = TransferMode.POOL, *, direction: str = "h2d",
                         options: PlannerEngineOptions | None = None) -> PlannerTransferPlan:
    return PlannerEngine(options).plan_ranges(ranges, chunk_bytes, profile, mode, direction=direction)


__all__ = ["CHUNK_CANDIDATES", "POLICIES", "PlannerEngine", "PlannerEngineOptions", "assign_python",
           "plan_transfer", "plan_transfer_ranges"]
