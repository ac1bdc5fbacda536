"""Helpers shared by the daemon-first (intent) benchmark CLIs: daemon options,
intent construction, receipt -> trace conversion and the ``daemon_receipt``
/ ``daemon_profile`` / ``daemon_reservation`` key=value lines.  The line
formats and trace fields match turbobus benchmarks/daemon_support.py:88-155
so existing log tooling keeps parsing them; receipts here carry MEASURED
per-lane stats (``cuda_ms``) when the daemon executed the intent."""

from __future__ import annotations

import os
from dataclasses import asdict
from enum import Enum
from collections.abc import Mapping
from typing import Iterable

from ..schema import TransferIntent, TransferReceipt, WorkloadKind


def add_daemon_options(parser) -> None:
    parser.add_argument("--daemon-socket-path")
    parser.add_argument("--daemon-max-inflight-chunks", type=int, default=8)
    parser.add_argument("--daemon-profile-max-age-seconds", type=float, default=3600.0)


def runtime_options_kwargs(args) -> dict[str, object]:
    kw: dict[str, object] = {}
    if getattr(args, "daemon_socket_path", None):
        kw["daemon_socket_path"] = args.daemon_socket_path
    kw["daemon_max_inflight_chunks"] = int(getattr(args, "daemon_max_inflight_chunks", 8))
    kw["daemon_profile_max_age_seconds"] = float(getattr(args, "daemon_profile_max_age_seconds", 3600.0))
    return kw


def collect_daemon_reservation_info(handles: Iterable) -> dict[str, object]:
    ids, relays = [], set()
    for h in handles:
        md = getattr(getattr(h, "receipt", None), "metadata", None) or {}
        for lid in md.get("lease_ids", ()) or ():
            ids.append(str(lid))
        for p in getattr(getattr(h, "receipt", None), "path_stats", ()) or ():
            if str(p.get("kind", "")) == "relay":
                relays.add(int(p.get("relay_device", -1)))
    return {"reservation_count": len(ids), "reservation_ids": ",".join(ids),
            "relay_gpus": ",".join(str(r) for r in sorted(relays))}


def make_benchmark_transfer_intent(*, intent_id: str, workload_kind: WorkloadKind | str, job_id: str,
                                   session_id: str, source_buffer_id: str, destination_buffer_id: str,
                                   direction: str, total_bytes: int, ranges, policy_hints: Mapping | None = None,
                                   metadata: Mapping | None = None, priority: int = 0) -> TransferIntent:
    return TransferIntent(intent_id=intent_id, job_id=job_id, session_id=session_id,
                          source_buffer_id=source_buffer_id, destination_buffer_id=destination_buffer_id,
                          direction=direction, total_bytes=int(total_bytes), ranges=tuple(ranges),
                          workload_kind=WorkloadKind(workload_kind), priority=int(priority),
                          policy_hints=dict(policy_hints or {}), metadata=dict(metadata or {}))


def submit_benchmark_transfer_intent(client, intent: TransferIntent, wait_timeout_seconds: float | None = None):
    receipt = client.submit_transfer_intent(intent)
    if wait_timeout_seconds is not None:
        receipt = client.wait_transfer_receipt(intent.intent_id, timeout_seconds=wait_timeout_seconds)
    return receipt


def _json_ready(v):
    if isinstance(v, Enum):
        return v.value
    if isinstance(v, Mapping):
        return {str(k): _json_ready(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_json_ready(x) for x in v]
    return v


def receipt_to_trace(receipt: TransferReceipt) -> dict[str, object]:
    trace = _json_ready(asdict(receipt))
    d_b = r_b = d_c = r_c = 0
    cuda_ms = 0.0
    for p in receipt.path_stats:
        n = int(p.get("bytes", 0) or 0)
        c = int(p.get("chunk_count", p.get("chunks", 0)) or 0)
        cuda_ms = max(cuda_ms, float(p.get("cuda_ms", 0.0) or 0.0))
        if str(p.get("kind", "")).lower() == "relay":
            r_b, r_c = r_b + n, r_c + c
        else:
            d_b, d_c = d_b + n, d_c + c
    split = {"direct_bytes": d_b, "relay_bytes": r_b, "direct_chunks": d_c, "relay_chunks": r_c}
    trace.update(split)
    trace["path_split"] = dict(split)
    trace["fallback_reason"] = str(receipt.metadata.get("fallback_reason", "") or "")
    trace["measured_cuda_ms"] = cuda_ms
    timing = receipt.metadata.get("timing") or {}
    for k in ("queue_ms", "execution_ms", "lease_wait_ms"):  # daemon-side waits (0 when not reported)
        trace[k] = float(timing.get(k) or 0.0)
    return trace


def receipt_trace_line(receipt: TransferReceipt, *, prefix: str = "daemon_receipt") -> str:
    t = receipt_to_trace(receipt)
    state = getattr(receipt.state, "value", receipt.state)
    fields = [prefix] + [f"{k}={t[k]}" for k in ("intent_id", "decision_id", "topology_snapshot_id", "ticket_id")]
    fields.append(f"state={state}")
    fields += [f"{k}={t[k]}" for k in ("bytes_total", "bytes_completed", "direct_bytes", "relay_bytes",
                                       "direct_chunks", "relay_chunks")]
    if t.get("fallback_reason"):
        fields.append("fallback_reason=" + str(t["fallback_reason"]).replace(" ", "_"))
    return " ".join(fields)


def benchmark_job_id(workload: str) -> str:
    return f"benchmark-{workload}-{os.getpid()}"


def _status_line(prefix: str, data: Mapping[str, object]) -> str:
    if not data:
        return ""
    fields = [f"{k}={data[k]}" for k in sorted(data) if data[k] not in (None, "")]
    return " ".join([prefix, *fields]) if fields else ""


def daemon_profile_line(profile: Mapping[str, object]) -> str:
    return _status_line("daemon_profile", profile)


def daemon_reservation_line(reservation: Mapping[str, object]) -> str:
    return _status_line("daemon_reservation", reservation)


__all__ = ["add_daemon_options", "benchmark_job_id", "collect_daemon_reservation_info", "daemon_profile_line",
           "daemon_reservation_line", "make_benchmark_transfer_intent", "receipt_to_trace", "receipt_trace_line",
           "runtime_options_kwargs", "submit_benchmark_transfer_intent"]
