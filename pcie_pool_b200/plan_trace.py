"""Plan <-> dict conversion and plan/trace files.

``transfer_plan_to_dict`` produces the plan JSON of the reference
(turbobus/plan_trace.py:6-47) from any plan-like object; ``plan_from_dict``
is its inverse.  ``write_trace`` stores a plan together with the measured
per-lane result as one versioned JSON document, and ``chrome_trace`` turns
such a record into Chrome-trace events (one row per lane).
"""

from __future__ import annotations

import json
import time
from pathlib import Path
from collections.abc import Mapping
from typing import Any

from .planner_types import (PlannerChunk, PlannerPath, PlannerPathAssignment,
                            PlannerTransferPlan, assignment_chunks, expand_plan)

TRACE_FORMAT = "pcie_pool_b200.plan_trace.v1"

_PATH_KEYS = ("kind", "direction", "target_device", "relay_device", "h2d_bw_gbps",
              "d2h_bw_gbps", "p2p_bw_gbps", "effective_bw_gbps", "enabled")


def transfer_plan_to_dict(plan) -> dict:
    """The plan in the reference's chunk-list form (compact chunk runs are
    expanded, so files written from it read the same in both projects)."""
    if isinstance(plan, Mapping):
        return expand_plan(plan)
    as_dict = getattr(plan, "as_dict", None)
    if callable(as_dict):
        out = as_dict()
        if isinstance(out, dict):
            return expand_plan(out)
    assignments = []
    for asg in plan.assignments:
        path = asg.path
        chunks = [{"src_offset": int(c.src_offset), "dst_offset": int(c.dst_offset),
                   "bytes": int(c.bytes)} for c in asg.chunk_list()]
        assignments.append({
            "path": {k: getattr(path, k) for k in _PATH_KEYS},
            "chunks": chunks,
            "bytes": sum(c["bytes"] for c in chunks),
            "chunk_count": len(chunks),
        })
    return {"total_bytes": int(plan.total_bytes), "chunk_bytes": int(plan.chunk_bytes),
            "assignments": assignments}


def plan_from_dict(data: Mapping[str, Any]) -> PlannerTransferPlan:
    assignments = []
    for asg in data.get("assignments", []) or []:
        p = asg["path"]
        path = PlannerPath(
            kind=str(p["kind"]), direction=str(p.get("direction", "h2d")),
            target_device=int(p.get("target_device", 0)),
            relay_device=int(p.get("relay_device", -1)),
            h2d_bw_gbps=float(p.get("h2d_bw_gbps", 0.0) or 0.0),
            d2h_bw_gbps=float(p.get("d2h_bw_gbps", 0.0) or 0.0),
            p2p_bw_gbps=float(p.get("p2p_bw_gbps", 0.0) or 0.0),
            effective_bw_gbps=float(p.get("effective_bw_gbps", 0.0) or 0.0),
            enabled=bool(p.get("enabled", True)), fabric_kind=p.get("fabric_kind"))
        chunks = tuple(PlannerChunk(int(c["src_offset"]), int(c["dst_offset"]), int(c["bytes"]),
                                    c.get("relay_device")) for c in assignment_chunks(asg))
        assignments.append(PlannerPathAssignment(path, chunks))
    return PlannerTransferPlan(int(data.get("total_bytes", 0)),
                               int(data.get("chunk_bytes", 16 << 20)), tuple(assignments))


def validate_plan_dict(data: Mapping[str, Any]) -> None:
    """Every chunk assigned exactly once and byte totals consistent."""
    total = int(data.get("total_bytes", 0))
    seen = 0
    for asg in data.get("assignments", []) or []:
        if not asg.get("path", {}).get("enabled", True):
            raise ValueError("transfer plan contains a disabled path")
        n = 0
        for c in assignment_chunks(asg):
            if int(c["bytes"]) <= 0 or int(c["src_offset"]) < 0 or int(c["dst_offset"]) < 0:
                raise ValueError("plan chunk offsets must be non-negative and bytes positive")
            n += int(c["bytes"])
        if "bytes" in asg and int(asg["bytes"]) != n:
            raise ValueError("assignment bytes do not match its chunks")
        seen += n
    if seen != total:
        raise ValueError("transfer plan total_bytes must match assigned chunk bytes")


def trace_record(plan, result: Any = None, **extra: Any) -> dict:
    rec: dict[str, Any] = {"format": TRACE_FORMAT, "created_at": time.time(),
                           "plan": transfer_plan_to_dict(plan)}
    if result is not None:
        rec["result"] = {
            "ok": bool(getattr(result, "ok", True)),
            "bytes": int(getattr(result, "bytes", 0)),
            "cuda_ms": float(getattr(result, "cuda_ms", 0.0)),
            "gib_per_s": float(getattr(result, "gib_per_s", 0.0)),
            "lanes": [{"device": l.device, "direct": l.direct, "bytes": l.bytes,
                       "chunks": l.chunks, "cuda_ms": l.cuda_ms}
                      for l in getattr(result, "lanes", [])],
        }
    rec.update(extra)
    return rec


def write_trace(path: str | Path, plan, result: Any = None, **extra: Any) -> Path:
    p = Path(path)
    p.write_text(json.dumps(trace_record(plan, result, **extra), indent=1, sort_keys=True))
    return p


def read_trace(path: str | Path) -> dict:
    rec = json.loads(Path(path).read_text())
    if rec.get("format") != TRACE_FORMAT:
        raise ValueError(f"not a {TRACE_FORMAT} file")
    return rec


def chrome_trace(record: Mapping[str, Any], t0_us: float = 0.0) -> dict:
    """Chrome trace (chrome://tracing) events for a trace record's lanes."""
    events = []
    res = record.get("result") or {}
    for i, lane in enumerate(res.get("lanes", [])):
        name = "direct" if lane.get("direct") else f"relay gpu{lane['device']}"
        events.append({"name": name, "ph": "X", "pid": 0, "tid": i, "ts": t0_us,
                       "dur": float(lane.get("cuda_ms", 0.0)) * 1e3,
                       "args": {"bytes": lane.get("bytes"), "chunks": lane.get("chunks")}})
    return {"traceEvents": events, "displayTimeUnit": "ms"}



def device_trace_events(result, lanes, *, name: str = "transfer", pid: int = 0) -> list[dict]:
    """Chrome-trace events from a transfer run with ``trace=True``: per lane
    (one track per lane device) and chunk, a ``wait`` span (until the chunk
    was published -- H2D -- or its staging slot was free -- D2H) and a
    ``move`` span (until the last CTA finished it).  Times are the device's
    %globaltimer in microseconds relative to the earliest stamp."""
    tr = getattr(result, "trace", None)
    if tr is None or not len(tr):
        return []
    stamps = [int(x) for x in tr[:, 0] if int(x)]
    if not stamps:
        return []
    t0 = min(stamps)
    out, i = [], 0
    for lane in lanes:
        for k in range(len(lane.bytes)):
            a, b, c, ctas = (int(x) for x in tr[i])
            i += 1
            if not a:
                continue
            args = {"chunk": k, "bytes": int(lane.bytes[k]), "ctas": ctas}
            out.append({"name": f"{name}:wait", "ph": "X", "pid": pid, "tid": int(lane.device),
                        "ts": (a - t0) / 1e3, "dur": max(0, b - a) / 1e3, "args": args})
            if c:
                out.append({"name": f"{name}:move", "ph": "X", "pid": pid, "tid": int(lane.device),
                            "ts": (b - t0) / 1e3, "dur": max(0, c - b) / 1e3, "args": args})
    return out


__all__ = ["TRACE_FORMAT", "chrome_trace", "device_trace_events", "plan_from_dict", "read_trace", "trace_record",
           "transfer_plan_to_dict", "validate_plan_dict", "write_trace"]
