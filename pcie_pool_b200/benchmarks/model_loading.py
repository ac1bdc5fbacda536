"""Daemon-first model-weight loading benchmark (intent CLI).

    python -m pcie_pool_b200.benchmarks.model_loading --daemon-socket-path S \\
        --session-id SID --source-buffer-id HOST --destination-buffer-id GPU \\
        --bucket-count 8 --bucket-bytes 33554432 --iterations 5

Each iteration submits one ``model_weights`` intent of ``bucket_count``
ranges through ``TurboBusClient`` and (with ``--wait-timeout-seconds`` > 0)
waits for its receipt; ``load_ms`` covers submit + wait.  Output JSON is
``{config, warmup_samples, samples, summary}`` and a compact
``MODEL_LOAD_SUMMARY`` text block with ``daemon_receipt``-style lines, the
shapes of turbobus benchmarks/model_loading.py:142-356.  Because the daemon
here executes intents, the receipts carry the measured per-lane stats and a
waited iteration covers the actual data movement.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
import uuid
from pathlib import Path

from ..api import TurboBusClient
from ..schema import TransferReceipt, WorkloadKind
from .daemon_support import (add_daemon_options, benchmark_job_id, make_benchmark_transfer_intent, receipt_to_trace,
                             receipt_trace_line)


def bucket_ranges(bucket_count: int, bucket_bytes: int) -> tuple[dict[str, int], ...]:
    return tuple({"src_offset": i * int(bucket_bytes), "dst_offset": i * int(bucket_bytes), "bytes": int(bucket_bytes)}
                 for i in range(int(bucket_count)))


def _wait_timeout(args) -> float | None:
    t = getattr(args, "wait_timeout_seconds", None)
    return None if t is None or float(t) <= 0 else float(t)


def sample_from_receipt(receipt: TransferReceipt, intent, elapsed_ms: float, iteration: int, phase: str,
                        prefix: str) -> dict:
    t = receipt_to_trace(receipt)
    gib = (int(t["bytes_total"]) / (1 << 30)) / (elapsed_ms / 1e3) if elapsed_ms > 0 else 0.0
    return {"iteration": int(iteration), "phase": phase, f"{prefix}_ms": elapsed_ms,
            f"{prefix}_gib_per_second": gib,
            "intent": {"intent_id": intent.intent_id, "job_id": intent.job_id, "session_id": intent.session_id,
                       "source_buffer_id": intent.source_buffer_id,
                       "destination_buffer_id": intent.destination_buffer_id,
                       "workload_kind": intent.workload_kind.value, "total_bytes": intent.total_bytes,
                       "ranges": list(intent.ranges), "policy_hints": dict(intent.policy_hints),
                       "metadata": dict(intent.metadata)},
            "receipt": t, "bytes": int(t["bytes_total"]), "bytes_completed": int(t["bytes_completed"]),
            "direct_bytes": int(t["direct_bytes"]), "relay_bytes": int(t["relay_bytes"]),
            "direct_chunks": int(t["direct_chunks"]), "relay_chunks": int(t["relay_chunks"]),
            "measured_cuda_ms": float(t.get("measured_cuda_ms", 0.0)), "decision_id": str(t["decision_id"]),
            "topology_snapshot_id": str(t["topology_snapshot_id"]), "ticket_id": str(t["ticket_id"]),
            "fallback_reason": str(t.get("fallback_reason", "") or "")}


def build_intent(args, *, iteration: int, phase: str):
    return make_benchmark_transfer_intent(
        intent_id=f"{args.intent_prefix}-{args.run_id}-{phase}-{iteration}", workload_kind=WorkloadKind.MODEL_WEIGHTS,
        job_id=args.job_id, session_id=args.session_id, source_buffer_id=args.source_buffer_id,
        destination_buffer_id=args.destination_buffer_id, direction="h2d",
        total_bytes=int(args.bucket_count) * int(args.bucket_bytes),
        ranges=bucket_ranges(args.bucket_count, args.bucket_bytes),
        metadata={"benchmark": "model-loading", "phase": phase, "iteration": int(iteration), "policy": args.policy,
                  "storage_layout": args.storage_layout, "bucket_count": int(args.bucket_count),
                  "bucket_bytes": int(args.bucket_bytes), "chunk_bytes": int(args.chunk_bytes)})


def submit_load_intent(client, args, *, iteration: int, phase: str) -> dict:
    intent = build_intent(args, iteration=iteration, phase=phase)
    t0 = time.perf_counter()
    receipt = client.submit_transfer_intent(intent)
    if _wait_timeout(args) is not None:
        receipt = client.wait_transfer_receipt(intent.intent_id, timeout_seconds=_wait_timeout(args))
    return sample_from_receipt(receipt, intent, (time.perf_counter() - t0) * 1e3, iteration, phase, "load")


def summarize(samples: list[dict], prefix: str = "load") -> dict:
    keys = ("bytes", "bytes_completed", "direct_bytes", "relay_bytes", "direct_chunks", "relay_chunks")
    if not samples:
        return {"iterations": 0, f"median_{prefix}_ms": 0.0, "median_gib_per_second": 0.0, **{k: 0 for k in keys},
                "decision_ids": [], "topology_snapshot_ids": [], "ticket_ids": [], "receipt_ids": [],
                "fallback_reasons": []}
    return {"iterations": len(samples),
            f"median_{prefix}_ms": statistics.median(s[f"{prefix}_ms"] for s in samples),
            "median_gib_per_second": statistics.median(s[f"{prefix}_gib_per_second"] for s in samples),
            "median_measured_cuda_ms": statistics.median(s.get("measured_cuda_ms", 0.0) for s in samples),
            "median_queue_ms": statistics.median(float(s["receipt"].get("queue_ms", 0.0)) for s in samples),
            "median_lease_wait_ms": statistics.median(float(s["receipt"].get("lease_wait_ms", 0.0))
                                                      for s in samples),
            **{k: int(statistics.median(s[k] for s in samples)) for k in keys},
            "decision_ids": sorted({s["decision_id"] for s in samples}),
            "topology_snapshot_ids": sorted({s["topology_snapshot_id"] for s in samples}),
            "ticket_ids": sorted({s["ticket_id"] for s in samples}),
            "receipt_ids": sorted({str(s["receipt"].get("receipt_id")) for s in samples if s["receipt"].get("receipt_id")}),
            "fallback_reasons": sorted({s["fallback_reason"] for s in samples if s["fallback_reason"]})}


def config_dict(args) -> dict:
    return {"session_id": args.session_id, "job_id": args.job_id, "source_buffer_id": args.source_buffer_id,
            "destination_buffer_id": args.destination_buffer_id, "workload_kind": WorkloadKind.MODEL_WEIGHTS.value,
            "bucket_count": int(args.bucket_count), "bucket_bytes": int(args.bucket_bytes),
            "storage_layout": args.storage_layout, "chunk_bytes": int(args.chunk_bytes), "warmup": int(args.warmup),
            "iterations": int(args.iterations), "policy": args.policy, "run_id": args.run_id,
            "daemon_socket_path": args.daemon_socket_path, "wait_timeout_seconds": args.wait_timeout_seconds}


def run_benchmark(args, *, client=None) -> dict:
    client = client or TurboBusClient(socket_path=args.daemon_socket_path)
    warm = [submit_load_intent(client, args, iteration=i, phase="warmup") for i in range(int(args.warmup))]
    samples = [submit_load_intent(client, args, iteration=i, phase="measure") for i in range(int(args.iterations))]
    return {"config": config_dict(args), "warmup_samples": warm, "samples": samples, "summary": summarize(samples)}


def receipt_from_trace(t: dict) -> TransferReceipt:
    return TransferReceipt(receipt_id=t["receipt_id"], ticket_id=t["ticket_id"], intent_id=t["intent_id"],
                           decision_id=t["decision_id"], topology_snapshot_id=t["topology_snapshot_id"],
                           job_id=t["job_id"], session_id=t["session_id"], state=t["state"],
                           bytes_total=t["bytes_total"], bytes_completed=t["bytes_completed"],
                           started_at=t.get("started_at", 0.0), completed_at=t.get("completed_at"),
                           path_stats=tuple(t.get("path_stats", ())), error=t.get("error"),
                           metadata=t.get("metadata", {}))


def compact_summary(result: dict) -> str:
    c, s = result["config"], result["summary"]
    lines = ["MODEL_LOAD_SUMMARY_BEGIN",
             f"model_load_config session_id={c['session_id']} job_id={c['job_id']} "
             f"source_buffer_id={c['source_buffer_id']} destination_buffer_id={c['destination_buffer_id']} "
             f"bucket_count={c['bucket_count']} bucket_bytes={c['bucket_bytes']} storage_layout={c['storage_layout']} "
             f"chunk_bytes={c['chunk_bytes']} iterations={c['iterations']} policy={c['policy']} "
             f"daemon_socket_path={c['daemon_socket_path']}",
             f"model_load_summary median_load_ms={s['median_load_ms']:.3f} "
             f"median_gib_s={s['median_gib_per_second']:.3f} bytes={s['bytes']} bytes_completed={s['bytes_completed']} "
             f"direct_bytes={s['direct_bytes']} relay_bytes={s['relay_bytes']} direct_chunks={s['direct_chunks']} "
             f"relay_chunks={s['relay_chunks']}"]
    for x in result["samples"]:
        lines.append(f"model_load_sample iteration={x['iteration']} load_ms={x['load_ms']:.3f} "
                     f"gib_s={x['load_gib_per_second']:.3f} decision_id={x['decision_id']} "
                     f"topology_snapshot_id={x['topology_snapshot_id']} ticket_id={x['ticket_id']}")
        lines.append(receipt_trace_line(receipt_from_trace(x["receipt"]), prefix="model_load_receipt"))
    lines.append("MODEL_LOAD_SUMMARY_END")
    return "\n".join(lines)


def write_outputs(args, result: dict, summary_text: str) -> None:
    if args.json_output:
        p = Path(args.json_output)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(json.dumps(result, indent=2) + "\n", encoding="utf-8")
    if args.summary_output:
        p = Path(args.summary_output)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(summary_text + "\n", encoding="utf-8")
    if not args.no_copy_summary:
        sys.stdout.write(summary_text + "\n")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Submit model weight loading intents through the public client")
    p.add_argument("--session-id", required=True)
    p.add_argument("--job-id", default=benchmark_job_id("model-loading"))
    p.add_argument("--source-buffer-id", required=True)
    p.add_argument("--destination-buffer-id", required=True)
    p.add_argument("--bucket-count", type=int, default=8)
    p.add_argument("--bucket-bytes", type=int, default=32 << 20)
    p.add_argument("--storage-layout", choices=["packed", "separate"], default="packed")
    p.add_argument("--chunk-bytes", type=int, default=4 << 20)
    p.add_argument("--warmup", type=int, default=0)
    p.add_argument("--iterations", type=int, default=5)
    p.add_argument("--policy", default="daemon-default")
    p.add_argument("--run-id", default=str(uuid.uuid4()))
    p.add_argument("--intent-prefix", default="model-load")
    p.add_argument("--wait-timeout-seconds", type=float, default=0.0)
    p.add_argument("--json-output")
    p.add_argument("--summary-output")
    p.add_argument("--no-copy-summary", action="store_true")
    add_daemon_options(p)
    return p


def validate_args(args) -> None:
    for name in ("bucket_count", "bucket_bytes", "chunk_bytes", "iterations"):
        if int(getattr(args, name)) <= 0:
            raise SystemExit(f"--{name.replace('_', '-')} must be positive")
    if int(args.warmup) < 0:
        raise SystemExit("--warmup must be non-negative")
    if not args.daemon_socket_path:
        raise SystemExit("--daemon-socket-path is required")


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    validate_args(args)
    result = run_benchmark(args)
    write_outputs(args, result, compact_summary(result))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
