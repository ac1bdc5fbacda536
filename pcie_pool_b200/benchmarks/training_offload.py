"""Daemon-first training-offload benchmark (intent CLI).

    python -m pcie_pool_b200.benchmarks.training_offload --daemon-socket-path S \\
        --session-id SID --cpu-buffer-id HOST --gpu-buffer-id GPU \\
        --bucket-count 8 --active-buckets 4 --bucket-bytes 33554432 --iterations 5

Per iteration: a ``prefetch`` intent (H2D of the active buckets) -> an
optional compute delay -> an ``offload`` intent (D2H of the same buckets);
the active window rotates through the buckets each iteration.  Output JSON
``{config, warmup_samples, samples, summary}`` plus a compact
``TRAINING_OFFLOAD_SUMMARY`` block, as turbobus
benchmarks/training_offload.py:25-356.
"""

from __future__ import annotations

import argparse
import statistics
import time
import uuid

from ..api import TurboBusClient
from ..schema import WorkloadKind
from .daemon_support import (add_daemon_options, benchmark_job_id, make_benchmark_transfer_intent,
                             receipt_trace_line)
from .model_loading import _wait_timeout, receipt_from_trace, sample_from_receipt, write_outputs


def bucket_indices(bucket_count: int, active_buckets: int, iteration: int) -> tuple[int, ...]:
    start = (int(iteration) * int(active_buckets)) % int(bucket_count)
    return tuple((start + k) % int(bucket_count) for k in range(int(active_buckets)))


def bucket_ranges(bucket_count: int, active_buckets: int, bucket_bytes: int, iteration: int):
    return tuple({"src_offset": i * int(bucket_bytes), "dst_offset": i * int(bucket_bytes), "bytes": int(bucket_bytes)}
                 for i in bucket_indices(bucket_count, active_buckets, iteration))


def active_bucket_count(args) -> int:
    return int(args.bucket_count if args.active_buckets is None else args.active_buckets)


def build_training_intent(args, *, iteration: int, phase: str, operation: str):
    h2d = operation == "prefetch"
    rs = bucket_ranges(args.bucket_count, active_bucket_count(args), args.bucket_bytes, iteration)
    return make_benchmark_transfer_intent(
        intent_id=f"{args.intent_prefix}-{args.run_id}-{phase}-{iteration}-{operation}",
        workload_kind=WorkloadKind(args.workload_kind), job_id=args.job_id, session_id=args.session_id,
        source_buffer_id=args.cpu_buffer_id if h2d else args.gpu_buffer_id,
        destination_buffer_id=args.gpu_buffer_id if h2d else args.cpu_buffer_id,
        direction="h2d" if h2d else "d2h", total_bytes=sum(r["bytes"] for r in rs), ranges=rs,
        metadata={"benchmark": "training-offload", "phase": phase, "iteration": int(iteration),
                  "operation": operation, "policy": args.policy, "storage_layout": args.storage_layout,
                  "bucket_count": int(args.bucket_count), "active_buckets": active_bucket_count(args),
                  "bucket_bytes": int(args.bucket_bytes), "chunk_bytes": int(args.chunk_bytes)})


def submit_training_intent(client, args, *, iteration: int, phase: str, operation: str) -> dict:
    intent = build_training_intent(args, iteration=iteration, phase=phase, operation=operation)
    t0 = time.perf_counter()
    receipt = client.submit_transfer_intent(intent)
    if _wait_timeout(args) is not None:
        receipt = client.wait_transfer_receipt(intent.intent_id, timeout_seconds=_wait_timeout(args))
    s = sample_from_receipt(receipt, intent, (time.perf_counter() - t0) * 1e3, iteration, phase, "transfer")
    s["operation"] = operation
    return s


def run_compute_delay(delay_ms: float) -> float:
    if float(delay_ms) <= 0:
        return 0.0
    t0 = time.perf_counter()
    time.sleep(float(delay_ms) / 1e3)
    return (time.perf_counter() - t0) * 1e3


def run_iteration(client, args, *, iteration: int, phase: str) -> dict:
    t0 = time.perf_counter()
    pre = submit_training_intent(client, args, iteration=iteration, phase=phase, operation="prefetch")
    comp = run_compute_delay(args.compute_delay_ms)
    off = submit_training_intent(client, args, iteration=iteration, phase=phase, operation="offload")
    return {"iteration": int(iteration), "phase": phase, "active_buckets": active_bucket_count(args),
            "iteration_ms": (time.perf_counter() - t0) * 1e3, "transfer_ms": pre["transfer_ms"] + off["transfer_ms"],
            "compute_ms": comp, "prefetch": pre, "offload": off}


def _side(samples: list[dict], op: str) -> dict:
    keys = ("bytes", "bytes_completed", "direct_bytes", "relay_bytes", "direct_chunks", "relay_chunks")
    if not samples:
        return {"median_transfer_ms": 0.0, **{k: 0 for k in keys}, "decision_ids": [], "topology_snapshot_ids": [],
                "ticket_ids": [], "receipt_ids": [], "fallback_reasons": []}
    xs = [s[op] for s in samples]
    return {"median_transfer_ms": statistics.median(x["transfer_ms"] for x in xs),
            "median_measured_cuda_ms": statistics.median(x.get("measured_cuda_ms", 0.0) for x in xs),
            **{k: int(statistics.median(x[k] for x in xs)) for k in keys},
            "decision_ids": sorted({x["decision_id"] for x in xs}),
            "topology_snapshot_ids": sorted({x["topology_snapshot_id"] for x in xs}),
            "ticket_ids": sorted({x["ticket_id"] for x in xs}),
            "receipt_ids": sorted({str(x["receipt"].get("receipt_id")) for x in xs if x["receipt"].get("receipt_id")}),
            "fallback_reasons": sorted({x["fallback_reason"] for x in xs if x["fallback_reason"]})}


def summarize_training(samples: list[dict]) -> dict:
    if not samples:
        return {"iterations": 0, "median_iteration_ms": 0.0, "median_transfer_ms": 0.0, "median_compute_ms": 0.0,
                "median_gib_per_second": 0.0, "prefetch": _side([], "prefetch"), "offload": _side([], "offload")}
    tb = [s["prefetch"]["bytes"] + s["offload"]["bytes"] for s in samples]
    tm = [s["transfer_ms"] for s in samples]
    return {"iterations": len(samples), "median_iteration_ms": statistics.median(s["iteration_ms"] for s in samples),
            "median_transfer_ms": statistics.median(tm),
            "median_compute_ms": statistics.median(s["compute_ms"] for s in samples),
            "median_gib_per_second": statistics.median((b / (1 << 30)) / (m / 1e3) if m > 0 else 0.0
                                                       for b, m in zip(tb, tm)),
            "prefetch": _side(samples, "prefetch"), "offload": _side(samples, "offload")}


def config_dict(args) -> dict:
    return {"session_id": args.session_id, "job_id": args.job_id, "cpu_buffer_id": args.cpu_buffer_id,
            "gpu_buffer_id": args.gpu_buffer_id, "workload_kind": args.workload_kind,
            "bucket_count": int(args.bucket_count), "active_buckets": active_bucket_count(args),
            "bucket_bytes": int(args.bucket_bytes), "storage_layout": args.storage_layout,
            "chunk_bytes": int(args.chunk_bytes), "warmup": int(args.warmup), "iterations": int(args.iterations),
            "compute_delay_ms": float(args.compute_delay_ms), "policy": args.policy, "run_id": args.run_id,
            "daemon_socket_path": args.daemon_socket_path, "wait_timeout_seconds": args.wait_timeout_seconds}


def run_benchmark(args, *, client=None) -> dict:
    client = client or TurboBusClient(socket_path=args.daemon_socket_path)
    warm = [run_iteration(client, args, iteration=i, phase="warmup") for i in range(int(args.warmup))]
    samples = [run_iteration(client, args, iteration=i, phase="measure") for i in range(int(args.iterations))]
    return {"config": config_dict(args), "warmup_samples": warm, "samples": samples,
            "summary": summarize_training(samples)}


def compact_summary(result: dict) -> str:
    c, s = result["config"], result["summary"]
    lines = ["TRAINING_OFFLOAD_SUMMARY_BEGIN",
             f"training_offload_config session_id={c['session_id']} job_id={c['job_id']} "
             f"cpu_buffer_id={c['cpu_buffer_id']} gpu_buffer_id={c['gpu_buffer_id']} "
             f"workload_kind={c['workload_kind']} bucket_count={c['bucket_count']} "
             f"active_buckets={c['active_buckets']} bucket_bytes={c['bucket_bytes']} chunk_bytes={c['chunk_bytes']} "
             f"iterations={c['iterations']} compute_delay_ms={c['compute_delay_ms']} policy={c['policy']} "
             f"daemon_socket_path={c['daemon_socket_path']}",
             f"training_offload_summary median_iteration_ms={s['median_iteration_ms']:.3f} "
             f"median_transfer_ms={s['median_transfer_ms']:.3f} median_compute_ms={s['median_compute_ms']:.3f} "
             f"median_gib_s={s['median_gib_per_second']:.3f}"]
    for side in ("prefetch", "offload"):
        x = s[side]
        lines.append(f"training_offload_{side} median_transfer_ms={x['median_transfer_ms']:.3f} bytes={x['bytes']} "
                     f"direct_bytes={x['direct_bytes']} relay_bytes={x['relay_bytes']} "
                     f"direct_chunks={x['direct_chunks']} relay_chunks={x['relay_chunks']}")
    for smp in result["samples"]:
        lines.append(f"training_offload_sample iteration={smp['iteration']} iteration_ms={smp['iteration_ms']:.3f} "
                     f"transfer_ms={smp['transfer_ms']:.3f} compute_ms={smp['compute_ms']:.3f}")
        for side in ("prefetch", "offload"):
            lines.append(receipt_trace_line(receipt_from_trace(smp[side]["receipt"]),
                                            prefix=f"training_offload_{side}_receipt"))
    lines.append("TRAINING_OFFLOAD_SUMMARY_END")
    return "\n".join(lines)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Submit training offload intents through the public client")
    p.add_argument("--session-id", required=True)
    p.add_argument("--job-id", default=benchmark_job_id("training-offload"))
    p.add_argument("--cpu-buffer-id", required=True)
    p.add_argument("--gpu-buffer-id", required=True)
    p.add_argument("--workload-kind", choices=[WorkloadKind.TRAINING_STATE.value, WorkloadKind.OPTIMIZER_STATE.value],
                   default=WorkloadKind.TRAINING_STATE.value)
    p.add_argument("--bucket-count", type=int, default=8)
    p.add_argument("--active-buckets", type=int)
    p.add_argument("--bucket-bytes", type=int, default=32 << 20)
    p.add_argument("--storage-layout", choices=["packed", "separate"], default="packed")
    p.add_argument("--chunk-bytes", type=int, default=4 << 20)
    p.add_argument("--warmup", type=int, default=0)
    p.add_argument("--iterations", type=int, default=5)
    p.add_argument("--compute-delay-ms", type=float, default=0.0)
    p.add_argument("--policy", default="daemon-default")
    p.add_argument("--run-id", default=str(uuid.uuid4()))
    p.add_argument("--intent-prefix", default="training-offload")
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
    if args.active_buckets is not None and not 0 < int(args.active_buckets) <= int(args.bucket_count):
        raise SystemExit("--active-buckets must be in 1..bucket-count")
    if int(args.warmup) < 0 or float(args.compute_delay_ms) < 0:
        raise SystemExit("--warmup and --compute-delay-ms must be non-negative")
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
