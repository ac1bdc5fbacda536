"""Paper-validation orchestrator: runs the daemon-first workloads as
subprocesses against one daemon, collects their results into unified
``paper_metric`` records, validates the trace fields and writes a JSON report
plus a ``PAPER_VALIDATION_SUMMARY`` text block (the record fields and line
format of turbobus benchmarks/paper_validation.py:466-994).

    python -m pcie_pool_b200.benchmarks.paper_validation --daemon-socket-path S \\
        --session-id SID --cpu-buffer-id HOST --gpu-buffer-id GPU \\
        --workloads model-loading,training-offload,optimizer-offload,vllm-kv

Workloads: ``model-loading`` and ``training-offload`` / ``optimizer-offload``
(this package's intent CLIs) and ``vllm-kv`` (the KV connector example; its
``turbobus_kv_connector_event`` lines are parsed into save/restore metrics).
``--jobs N`` runs N concurrent copies of the vLLM workload (multi-tenant).
"""

from __future__ import annotations

import argparse
import json
import subprocess
import sys
from pathlib import Path

REPORT_SCHEMA = "pcie_pool_b200.paper_metric.v1"
WORKLOADS = ("model-loading", "training-offload", "optimizer-offload", "vllm-kv")
KIND = {"model-loading": "model_weights", "training-offload": "training_state",
        "optimizer-offload": "optimizer_state", "vllm-kv": "kv_cache"}
REQUIRED_UNIFIED_METRIC_FIELDS = ("workload", "report_schema", "policy", "job_id", "session_id", "workload_kind",
                                  "transfer_ms", "performance_ms", "transfer_bytes", "bytes_completed",
                                  "direct_bytes", "relay_bytes", "correctness_status")
METRIC_ORDER = ("workload", "report_schema", "policy", "job_index", "job_id", "session_id", "workload_kind",
                "source_buffer_id", "destination_buffer_id", "cpu_buffer_id", "gpu_buffer_id", "iterations",
                "ttft_proxy_ms", "iteration_ms", "transfer_ms", "performance_ms", "compute_ms", "measured_cuda_ms",
                "throughput_gib_s", "transfer_bytes", "bytes_completed", "direct_bytes", "relay_bytes",
                "direct_chunks", "relay_chunks", "receipt_ids", "decision_ids", "topology_snapshot_ids", "ticket_ids",
                "prefetch_decision_ids", "prefetch_receipt_ids", "offload_decision_ids", "offload_receipt_ids",
                "save_ms", "restore_ms", "save_layer_count", "save_layer_ranges", "fallback_reason",
                "correctness_status", "log_path")


def parse_csv(value: str) -> list[str]:
    return [x.strip() for x in str(value).split(",") if x.strip()]


def selected_workloads(value: str) -> list[str]:
    ws = list(WORKLOADS) if value in ("", "all") else parse_csv(value)
    bad = [w for w in ws if w not in WORKLOADS]
    if bad:
        raise SystemExit(f"unknown workloads: {','.join(bad)}")
    return ws


def output_paths(out: Path, workload: str) -> dict[str, Path]:
    return {"json": out / f"{workload}.json", "summary": out / f"{workload}.summary.txt",
            "log": out / f"{workload}.log"}


def _common(args) -> list[str]:
    return ["--daemon-socket-path", args.daemon_socket_path, "--session-id", args.session_id,
            "--chunk-bytes", str(args.chunk_bytes), "--warmup", str(args.warmup), "--iterations", str(args.iterations),
            "--policy", args.policy, "--wait-timeout-seconds", str(args.wait_timeout_seconds), "--no-copy-summary"]


def build_workload_commands(args, workload: str, paths: dict[str, Path]) -> list[list[str]]:
    py = [sys.executable, "-m"]
    outs = ["--json-output", str(paths["json"]), "--summary-output", str(paths["summary"])]
    if workload == "model-loading":
        return [py + ["pcie_pool_b200.benchmarks.model_loading", *_common(args), "--job-id", f"{args.job_id}-model",
                      "--source-buffer-id", args.cpu_buffer_id, "--destination-buffer-id", args.gpu_buffer_id,
                      "--bucket-count", str(args.bucket_count), "--bucket-bytes", str(args.bucket_bytes),
                      "--storage-layout", args.storage_layout, "--run-id", args.run_id, *outs]]
    if workload in ("training-offload", "optimizer-offload"):
        cmd = py + ["pcie_pool_b200.benchmarks.training_offload", *_common(args), "--job-id",
                    f"{args.job_id}-{workload.split('-')[0]}", "--cpu-buffer-id", args.cpu_buffer_id,
                    "--gpu-buffer-id", args.gpu_buffer_id, "--workload-kind", KIND[workload],
                    "--bucket-count", str(args.bucket_count), "--bucket-bytes", str(args.bucket_bytes),
                    "--compute-delay-ms", str(args.compute_delay_ms), "--storage-layout", args.storage_layout,
                    "--run-id", args.run_id, *outs]
        if args.active_buckets:
            cmd += ["--active-buckets", str(args.active_buckets)]
        return [cmd]
    cmds = []
    for j in range(max(1, int(args.jobs))):
        cmd = py + ["pcie_pool_b200.examples.vllm_kv_connector", "--json-output",
                    str(paths["json"].with_suffix(f".job{j}.json")), "--session-id", f"{args.session_id}-kv{j}",
                    "--job-id", f"{args.job_id}-kv{j}", "--prompt-tokens", str(args.vllm_prompt_tokens),
                    "--prefix-key", f"{args.vllm_prefix_key}-{j}", "--prompt-repeat", str(args.vllm_prompt_repeat),
                    "--second-prompt-suffix", args.vllm_second_prompt_suffix,
                    "--restore-blocks", str(args.vllm_restore_blocks),
                    "--matched-tokens", str(args.vllm_matched_tokens), "--chunk-bytes", str(args.chunk_bytes)]
        if args.vllm_model:
            cmd += ["--model", args.vllm_model]
        if args.vllm_prompt:
            cmd += ["--prompt", args.vllm_prompt]
        if args.vllm_wait_timeout_seconds is not None:
            cmd += ["--wait-timeout-seconds", str(args.vllm_wait_timeout_seconds)]
        if args.vllm_enable_multiproc_executor:
            cmd.append("--enable-multiproc-executor")
        if args.daemon_socket_path:
            cmd += ["--daemon-socket-path", args.daemon_socket_path]
        cmds.append(cmd)
    return cmds


def run_commands(cmds: list[list[str]], log: Path) -> int:
    log.parent.mkdir(parents=True, exist_ok=True)
    procs = []
    with open(log, "w", encoding="utf-8") as fh:
        for c in cmds:
            fh.write("$ " + " ".join(c) + "\n")
            fh.flush()
            procs.append(subprocess.Popen(c, stdout=fh, stderr=subprocess.STDOUT))
        rcs = [p.wait() for p in procs]
    return max(rcs) if rcs else 0


def _join(v) -> str:
    if v in (None, ""):
        return ""
    return ",".join(str(x) for x in v) if isinstance(v, (list, tuple)) else str(v)


def correctness_status(transfer_bytes: int, bytes_completed: int) -> str:
    if transfer_bytes <= 0:
        return "missing"
    return "complete" if bytes_completed == transfer_bytes else "incomplete"


def collect_model_metrics(result: dict, policy: str) -> list[dict]:
    s, c = result.get("summary") or {}, result.get("config") or {}
    if not s:
        return []
    ms = float(s.get("median_load_ms", 0.0))
    return [{"report_schema": REPORT_SCHEMA, "workload": "model-loading", "policy": policy,
             "job_id": c.get("job_id", ""), "session_id": c.get("session_id", ""),
             "source_buffer_id": c.get("source_buffer_id", ""), "destination_buffer_id": c.get("destination_buffer_id", ""),
             "cpu_buffer_id": c.get("source_buffer_id", ""), "gpu_buffer_id": c.get("destination_buffer_id", ""),
             "workload_kind": c.get("workload_kind", "model_weights"), "iterations": int(s.get("iterations", 0)),
             "ttft_proxy_ms": ms, "transfer_ms": ms, "performance_ms": ms,
             "measured_cuda_ms": float(s.get("median_measured_cuda_ms", 0.0)),
             "throughput_gib_s": float(s.get("median_gib_per_second", 0.0)),
             "transfer_bytes": int(s.get("bytes", 0)), "bytes_completed": int(s.get("bytes_completed", 0)),
             "direct_bytes": int(s.get("direct_bytes", 0)), "relay_bytes": int(s.get("relay_bytes", 0)),
             "direct_chunks": int(s.get("direct_chunks", 0)), "relay_chunks": int(s.get("relay_chunks", 0)),
             "receipt_ids": _join(s.get("receipt_ids")), "decision_ids": _join(s.get("decision_ids")),
             "topology_snapshot_ids": _join(s.get("topology_snapshot_ids")), "ticket_ids": _join(s.get("ticket_ids")),
             "fallback_reason": _join(s.get("fallback_reasons")),
             "correctness_status": correctness_status(int(s.get("bytes", 0)), int(s.get("bytes_completed", 0)))}]


def collect_training_metrics(result: dict, workload: str, policy: str) -> list[dict]:
    s, c = result.get("summary") or {}, result.get("config") or {}
    if not s:
        return []
    pre, off = s.get("prefetch") or {}, s.get("offload") or {}
    tb = int(pre.get("bytes", 0)) + int(off.get("bytes", 0))
    done = int(pre.get("bytes_completed", 0)) + int(off.get("bytes_completed", 0))
    return [{"report_schema": REPORT_SCHEMA, "workload": workload, "policy": policy, "job_id": c.get("job_id", ""),
             "session_id": c.get("session_id", ""), "cpu_buffer_id": c.get("cpu_buffer_id", ""),
             "gpu_buffer_id": c.get("gpu_buffer_id", ""), "workload_kind": c.get("workload_kind", KIND[workload]),
             "iterations": int(s.get("iterations", 0)), "iteration_ms": float(s.get("median_iteration_ms", 0.0)),
             "transfer_ms": float(s.get("median_transfer_ms", 0.0)),
             "performance_ms": float(s.get("median_iteration_ms", 0.0)),
             "compute_ms": float(s.get("median_compute_ms", 0.0)),
             "throughput_gib_s": float(s.get("median_gib_per_second", 0.0)), "transfer_bytes": tb,
             "bytes_completed": done, "direct_bytes": int(pre.get("direct_bytes", 0)) + int(off.get("direct_bytes", 0)),
             "relay_bytes": int(pre.get("relay_bytes", 0)) + int(off.get("relay_bytes", 0)),
             "direct_chunks": int(pre.get("direct_chunks", 0)) + int(off.get("direct_chunks", 0)),
             "relay_chunks": int(pre.get("relay_chunks", 0)) + int(off.get("relay_chunks", 0)),
             "prefetch_decision_ids": _join(pre.get("decision_ids")), "prefetch_receipt_ids": _join(pre.get("receipt_ids")),
             "offload_decision_ids": _join(off.get("decision_ids")), "offload_receipt_ids": _join(off.get("receipt_ids")),
             "fallback_reason": _join(sorted(set(pre.get("fallback_reasons", [])) | set(off.get("fallback_reasons", [])))),
             "correctness_status": correctness_status(tb, done)}]


def collect_vllm_kv_metrics(result: dict, policy: str, job_index: int | None = None) -> list[dict]:
    s = result.get("summary") or {}
    if not s:
        return []
    n = int(s.get("bytes", 0))
    m = {"report_schema": REPORT_SCHEMA, "workload": "vllm-kv", "policy": policy, "job_id": s.get("job_id", ""),
         "session_id": s.get("session_id", ""), "workload_kind": "kv_cache", "iterations": 1,
         "ttft_proxy_ms": float(s.get("restore_ms", 0.0)), "transfer_ms": float(s.get("save_ms", 0.0)) +
         float(s.get("restore_ms", 0.0)), "performance_ms": float(s.get("restore_ms", 0.0)),
         "save_ms": float(s.get("save_ms", 0.0)), "restore_ms": float(s.get("restore_ms", 0.0)),
         "transfer_bytes": n, "bytes_completed": int(s.get("bytes_completed", 0)),
         "direct_bytes": int(s.get("direct_bytes", 0)), "relay_bytes": int(s.get("relay_bytes", 0)),
         "save_layer_count": int(s.get("save_layer_count", 0)), "save_layer_ranges": int(s.get("save_layer_ranges", 0)),
         "correctness_status": "complete" if s.get("restore_verified") else "incomplete"}
    if job_index is not None:
        m["job_index"] = job_index
    return [m]


def metric_errors(m: dict) -> list[str]:
    return [f"missing_{k}" for k in REQUIRED_UNIFIED_METRIC_FIELDS if m.get(k) in (None, "")] + (
        [] if m.get("correctness_status") == "complete" else [f"correctness_{m.get('correctness_status')}"])


def metric_line(m: dict) -> str:
    fields = ["paper_metric"]
    for k in METRIC_ORDER:
        v = m.get(k)
        if v in (None, ""):
            continue
        fields.append(f"{k}={v:.3f}" if isinstance(v, float) else f"{k}={v}")
    return " ".join(fields)


def compact_summary(result: dict) -> str:
    c = result["config"]
    lines = ["PAPER_VALIDATION_SUMMARY_BEGIN",
             f"paper_validation_config session_id={c['session_id']} job_id={c['job_id']} "
             f"cpu_buffer_id={c['cpu_buffer_id']} gpu_buffer_id={c['gpu_buffer_id']} "
             f"workloads={','.join(c['workloads'])} policy={c['policy']} dry_run={c.get('dry_run', False)} "
             f"output_dir={c['output_dir']}"]
    for w in result["workloads"]:
        lines.append(f"paper_workload workload={w['workload']} status={w['status']} returncode={w['returncode']} "
                     f"summary={w['summary_path']} json={w['data_path']} "
                     f"validation_errors={','.join(w.get('validation_errors', []))}")
        lines += [metric_line(m) for m in w["metrics"]]
    lines.append("PAPER_VALIDATION_SUMMARY_END")
    return "\n".join(lines)


def _read(path: Path):
    try:
        return json.loads(path.read_text(encoding="utf-8"))
    except (OSError, ValueError):
        return None


def run_validation(args) -> dict:
    out = Path(args.output_dir)
    workloads = selected_workloads(args.workloads)
    report = {"config": {"session_id": args.session_id, "job_id": args.job_id, "cpu_buffer_id": args.cpu_buffer_id,
                         "gpu_buffer_id": args.gpu_buffer_id, "workloads": workloads, "policy": args.policy,
                         "dry_run": bool(args.dry_run), "output_dir": str(out), "jobs": int(args.jobs)},
              "workloads": []}
    for w in workloads:
        paths = output_paths(out, w)
        cmds = build_workload_commands(args, w, paths)
        rc = 0 if args.dry_run else run_commands(cmds, paths["log"])
        metrics, errors = [], []
        if not args.dry_run:
            if w == "vllm-kv":
                for j in range(max(1, int(args.jobs))):
                    data = _read(paths["json"].with_suffix(f".job{j}.json")) or {}
                    metrics += collect_vllm_kv_metrics(data, args.policy, j if args.jobs > 1 else None)
            else:
                data = _read(paths["json"]) or {}
                metrics = (collect_model_metrics(data, args.policy) if w == "model-loading"
                           else collect_training_metrics(data, w, args.policy))
            if not metrics:
                errors.append("missing_paper_metrics")
            for m in metrics:
                errors += metric_errors(m)
                m["log_path"] = str(paths["log"])
        status = "dry_run" if args.dry_run else ("passed" if rc == 0 and not errors else "failed")
        report["workloads"].append({"workload": w, "status": status, "returncode": rc,
                                    "commands": [" ".join(c) for c in cmds], "summary_path": str(paths["summary"]),
                                    "data_path": str(paths["json"]), "validation_errors": sorted(set(errors)),
                                    "metrics": metrics})
        if status == "failed" and not args.keep_going:
            break
    return report


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--workloads", default="all")
    p.add_argument("--daemon-socket-path", default="")
    p.add_argument("--session-id", required=True)
    p.add_argument("--job-id", default="paper-validation")
    p.add_argument("--cpu-buffer-id", required=True)
    p.add_argument("--gpu-buffer-id", required=True)
    p.add_argument("--policy", default="daemon-default")
    p.add_argument("--run-id", default="paper-validation")
    p.add_argument("--chunk-bytes", type=int, default=4 << 20)
    p.add_argument("--warmup", type=int, default=0)
    p.add_argument("--iterations", type=int, default=3)
    p.add_argument("--bucket-count", type=int, default=8)
    p.add_argument("--active-buckets", type=int)
    p.add_argument("--bucket-bytes", type=int, default=32 << 20)
    p.add_argument("--compute-delay-ms", type=float, default=0.0)
    p.add_argument("--wait-timeout-seconds", type=float, default=600.0)
    p.add_argument("--jobs", "--vllm-job-count", dest="jobs", type=int, default=1, help="concurrent vLLM KV jobs")
    p.add_argument("--storage-layout", choices=["packed", "separate"], default="packed",
                   help="host layout of the model-loading / training buckets")
    p.add_argument("--vllm-prompt-tokens", type=int, default=4096, help="random-token prefix length")
    p.add_argument("--vllm-model", default="", help="local checkpoint (default: random-init demo model)")
    p.add_argument("--vllm-prompt", default="", help="text prompt (default: random token ids)")
    p.add_argument("--vllm-prompt-repeat", type=int, default=64)
    p.add_argument("--vllm-second-prompt-suffix", default=" Italy")
    p.add_argument("--vllm-prefix-key", default="paper-validation-vllm-kv")
    p.add_argument("--vllm-restore-blocks", type=int, default=0, help="restore cap in blocks (0 = all)")
    p.add_argument("--vllm-matched-tokens", type=int, default=0, help="tokens to restore (0 = whole prefix)")
    p.add_argument("--vllm-wait-timeout-seconds", type=float, default=None)
    p.add_argument("--vllm-enforce-eager", action="store_true", help="accepted; the demo runs eager by default")
    p.add_argument("--vllm-enable-multiproc-executor", action="store_true")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--keep-going", action="store_true")
    p.add_argument("--output-dir", default="results/paper_validation")
    p.add_argument("--json-output")
    p.add_argument("--summary-output")
    p.add_argument("--no-copy-summary", action="store_true")
    return p


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    report = run_validation(args)
    text = compact_summary(report)
    if args.json_output:
        Path(args.json_output).parent.mkdir(parents=True, exist_ok=True)
        Path(args.json_output).write_text(json.dumps(report, indent=2) + "\n", encoding="utf-8")
    if args.summary_output:
        Path(args.summary_output).write_text(text + "\n", encoding="utf-8")
    if not args.no_copy_summary:
        print(text)
    return 0 if all(w["status"] in ("passed", "dry_run") for w in report["workloads"]) else 1


if __name__ == "__main__":
    raise SystemExit(main())
