"""Evaluation pipeline over paper-validation reports: baseline-vs-pooled
comparison, result checks, daemon evidence, the per-server-class bundle gate,
the acceptance inventory and artifact ingestion, and the run planner.

Sub-commands (``python -m pcie_pool_b200.benchmarks.phase7 <cmd> ...``, or the
``phase7_<cmd>`` modules):

* ``server-run``  plan (and run) the baseline and pooled paper-validation
  chains for a server class (2/4/8 GPU) and the follow-up steps;
* ``compare``     p50/p99 latency and throughput ratios per workload;
* ``check``       schema and trace-field checks of one report;
* ``evidence``    join a report with the daemon's describe/PROFILE dump
  (audit records, fallback reasons, relay quotas);
* ``gate``        accept/reject a server-class bundle;
* ``inventory``   accepted / blocked / missing server classes of a manifest;
* ``ingest``      record a gated bundle into the manifest.

Record shapes follow turbobus benchmarks/phase7_*.py (report fields, status
words, the 2gpu/4gpu/8gpu classes); the implementation is independent.
"""

from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import sys
from pathlib import Path

from .paper_validation import REQUIRED_UNIFIED_METRIC_FIELDS, WORKLOADS

BASELINE_POLICY = "paper-baseline"
POOLED_POLICY = "turbobus-daemon"
SERVER_CLASSES = ("2gpu", "4gpu", "8gpu")
STATUSES = ("accepted", "blocked", "missing")
EXPECTED_KIND = {"model-loading": "model_weights", "training-offload": "training_state",
                 "optimizer-offload": "optimizer_state", "vllm-kv": "kv_cache"}
TRACE_FIELDS = ("receipt_ids", "decision_ids", "topology_snapshot_ids", "ticket_ids", "prefetch_receipt_ids",
                "prefetch_decision_ids", "offload_receipt_ids", "offload_decision_ids")


def read_json(path) -> dict:
    data = json.loads(Path(path).read_text(encoding="utf-8"))
    if not isinstance(data, dict):
        raise ValueError(f"{path}: JSON object expected")
    return data


def write_json(path, payload: dict) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n", encoding="utf-8")


def _split(v) -> list[str]:
    if v in (None, ""):
        return []
    return [str(x) for x in v] if isinstance(v, (list, tuple)) else [x for x in str(v).split(",") if x]


def percentile(values: list[float], pct: float) -> float:
    xs = sorted(float(v) for v in values)
    if not xs:
        return 0.0
    k = (len(xs) - 1) * pct / 100.0
    lo, hi = int(k), min(int(k) + 1, len(xs) - 1)
    return xs[lo] + (xs[hi] - xs[lo]) * (k - lo)


def metrics_of(report: dict) -> list[dict]:
    out = []
    for w in report.get("workloads", []) or []:
        for m in w.get("metrics", []) or []:
            out.append(m)
    return out


def metric_key(m: dict) -> str:
    j = m.get("job_index")
    return f"{m.get('workload')}" + ("" if j in (None, "") else f"#job{j}")


# ---- compare -------------------------------------------------------------------------------------

def _side_values(report: dict, key: str) -> dict:
    ms = [m for m in metrics_of(report) if metric_key(m) == key]
    perf = [float(m.get("performance_ms", 0.0)) for m in ms]
    thr = [float(m.get("throughput_gib_s", 0.0)) for m in ms]
    samples = []
    for w in report.get("workloads", []) or []:
        path = w.get("data_path")
        if path and Path(path).exists() and w.get("workload") == key.split("#")[0]:
            try:
                data = read_json(path)
                for s in data.get("samples", []) or []:
                    v = s.get("load_ms", s.get("iteration_ms"))
                    if v is not None:
                        samples.append(float(v))
            except (OSError, ValueError):
                pass
    vals = samples or perf
    return {"metrics": len(ms), "p50_ms": percentile(vals, 50), "p99_ms": percentile(vals, 99),
            "throughput_gib_s": statistics.median(thr) if thr else 0.0,
            "relay_bytes": sum(int(m.get("relay_bytes", 0)) for m in ms),
            "correct": all(m.get("correctness_status") == "complete" for m in ms) and bool(ms)}


def compare_reports(baseline: dict, pooled: dict, baseline_label: str = BASELINE_POLICY,
                    pooled_label: str = POOLED_POLICY) -> dict:
    keys = sorted({metric_key(m) for m in metrics_of(baseline)} | {metric_key(m) for m in metrics_of(pooled)})
    rows, missing = [], []
    for k in keys:
        b, t = _side_values(baseline, k), _side_values(pooled, k)
        if not b["metrics"] or not t["metrics"]:
            missing.append(k)
        rows.append({"workload": k, baseline_label: b, pooled_label: t,
                     "p50_speedup": b["p50_ms"] / t["p50_ms"] if t["p50_ms"] > 0 else None,
                     "p99_speedup": b["p99_ms"] / t["p99_ms"] if t["p99_ms"] > 0 else None,
                     "throughput_ratio": (t["throughput_gib_s"] / b["throughput_gib_s"]
                                          if b["throughput_gib_s"] > 0 else None)})
    return {"baseline_label": baseline_label, "pooled_label": pooled_label, "workloads": rows,
            "missing_workloads": missing}


# ---- check ---------------------------------------------------------------------------------------

def check_report(report: dict) -> dict:
    errors = []
    for w in report.get("workloads", []) or []:
        name = w.get("workload")
        if w.get("status") not in ("passed", "dry_run"):
            errors.append(f"{name}:status_{w.get('status')}")
        ms = w.get("metrics", []) or []
        if not ms and w.get("status") != "dry_run":
            errors.append(f"{name}:missing_paper_metrics")
        for m in ms:
            for f in REQUIRED_UNIFIED_METRIC_FIELDS:
                if m.get(f) in (None, ""):
                    errors.append(f"{name}:missing_{f}")
            kind = EXPECTED_KIND.get(str(name))
            if kind and m.get("workload_kind") != kind:
                errors.append(f"{name}:workload_kind_{m.get('workload_kind')}")
            if int(m.get("bytes_completed", 0)) != int(m.get("transfer_bytes", -1)):
                errors.append(f"{name}:bytes_incomplete")
            if name != "vllm-kv" and not any(_split(m.get(f)) for f in TRACE_FIELDS):
                errors.append(f"{name}:missing_trace_ids")
        if name == "vllm-kv" and len({m.get("job_id") for m in ms}) != len(ms):
            errors.append("vllm-kv:duplicate_job_identity")
    return {"ok": not errors, "errors": sorted(set(errors)), "workloads": [w.get("workload") for w in
                                                                          report.get("workloads", []) or []]}


# ---- evidence ------------------------------------------------------------------------------------

def profile_from_daemon(socket_path: str) -> dict:
    from ..daemon.client import TurboBusDaemonClient

    r = TurboBusDaemonClient(socket_path).describe()
    if not r.ok:
        raise RuntimeError(r.error or "daemon describe failed")
    return dict(r.payload)


def evidence_report(report: dict, profile: dict, comparison: dict | None = None) -> dict:
    audit = profile.get("audit_records", []) or []
    quotas = profile.get("relay_quotas", {}) or {}
    rows = []
    for m in metrics_of(report):
        ids = set()
        for f in TRACE_FIELDS:
            ids |= set(_split(m.get(f)))
        recs = [a for a in audit if a.get("decision_id") in ids or a.get("ticket_id") in ids
                or (a.get("job_id") and a.get("job_id") == m.get("job_id"))]
        rows.append({"workload": metric_key(m), "job_id": m.get("job_id"), "audit_records": len(recs),
                     "event_types": sorted({a.get("event_type") for a in recs}),
                     "failures": sorted({a.get("failure_reason") for a in recs if a.get("failure_reason")}),
                     "fallback_reason": m.get("fallback_reason", ""), "relay_bytes": int(m.get("relay_bytes", 0))})
    leaked = {k: q.get("active_chunks", 0) for k, q in quotas.items() if int(q.get("active_chunks", 0) or 0)}
    return {"metrics": rows, "relay_quotas": quotas, "leaked_quota_chunks": leaked,
            "open_reservations": len(profile.get("reservations", {}) or {}),
            "comparison": None if comparison is None else {"missing_workloads": comparison.get("missing_workloads")},
            "ok": not leaked and not profile.get("reservations")}


# ---- gate ----------------------------------------------------------------------------------------

def gate_bundle(server_class: str, baseline: dict, pooled: dict, comparison: dict, evidence: list[dict],
                required=WORKLOADS) -> dict:
    reasons = []
    for side, rep in (("baseline", baseline), ("pooled", pooled)):
        chk = check_report(rep)
        if not chk["ok"]:
            reasons += [f"{side}:{e}" for e in chk["errors"]]
        have = {w.get("workload") for w in rep.get("workloads", []) or []}
        reasons += [f"{side}:missing_workload_{w}" for w in required if w not in have]
    reasons += [f"comparison:missing_{w}" for w in comparison.get("missing_workloads", [])]
    for ev in evidence:
        if not ev.get("ok", False):
            reasons.append("evidence:leaked_resources")
    return {"server_class": server_class, "status": "accepted" if not reasons else "blocked",
            "reasons": sorted(set(reasons)), "workloads": sorted({w.get("workload") for w in
                                                                  pooled.get("workloads", []) or []})}


# ---- inventory / ingest --------------------------------------------------------------------------

def inventory(manifest: dict, classes=SERVER_CLASSES) -> dict:
    entries = {e.get("server_class"): e for e in manifest.get("server_classes", []) or []}
    rows = []
    for c in classes:
        e = entries.get(c)
        st = "missing" if e is None else e.get("status", "missing")
        if st not in STATUSES:
            st = "blocked"
        rows.append({"server_class": c, "status": st, "bundle": None if e is None else e.get("bundle"),
                     "reasons": [] if e is None else list(e.get("reasons", []))})
    return {"server_classes": rows, "accepted": [r["server_class"] for r in rows if r["status"] == "accepted"],
            "complete": all(r["status"] == "accepted" for r in rows)}


def ingest(manifest_path, gate_path) -> dict:
    mp = Path(manifest_path)
    manifest = read_json(mp) if mp.exists() else {"server_classes": []}
    gate = read_json(gate_path)
    rest = [e for e in manifest.get("server_classes", []) if e.get("server_class") != gate["server_class"]]
    rest.append({"server_class": gate["server_class"], "status": gate["status"], "bundle": str(gate_path),
                 "reasons": gate.get("reasons", [])})
    manifest["server_classes"] = sorted(rest, key=lambda e: e["server_class"])
    write_json(mp, manifest)
    return manifest


# ---- server run plan -----------------------------------------------------------------------------

def server_run_plan(a) -> dict:
    root = Path(a.output_root) / a.server_class
    steps = []
    for policy in (BASELINE_POLICY, POOLED_POLICY):
        tag = "baseline" if policy == BASELINE_POLICY else "pooled"
        steps.append({"name": f"paper-validation-{tag}", "command": [
            sys.executable, "-m", "pcie_pool_b200.benchmarks.paper_validation", "--daemon-socket-path",
            a.daemon_socket_path, "--session-id", a.session_id, "--cpu-buffer-id", a.cpu_buffer_id,
            "--gpu-buffer-id", a.gpu_buffer_id, "--policy", policy, "--workloads", a.workloads,
            "--bucket-count", str(a.bucket_count), "--bucket-bytes", str(a.bucket_bytes),
            "--chunk-bytes", str(a.chunk_bytes), "--warmup", str(a.warmup), "--iterations", str(a.iterations),
            "--output-dir", str(root / tag), "--json-output", str(root / f"{tag}.json"), "--keep-going",
            "--no-copy-summary"]})
    mod = [sys.executable, "-m", "pcie_pool_b200.benchmarks.phase7"]
    steps += [{"name": "check-baseline", "command": mod + ["check", str(root / "baseline.json"), "--json-output",
                                                            str(root / "baseline.check.json")]},
              {"name": "check-pooled", "command": mod + ["check", str(root / "pooled.json"), "--json-output",
                                                          str(root / "pooled.check.json")]},
              {"name": "compare", "command": mod + ["compare", "--baseline", str(root / "baseline.json"),
                                                    "--turbobus", str(root / "pooled.json"), "--json-output",
                                                    str(root / "comparison.json")]},
              {"name": "evidence", "command": mod + ["evidence", "--result", str(root / "pooled.json"),
                                                     "--daemon-socket-path", a.daemon_socket_path, "--json-output",
                                                     str(root / "evidence.json")]},
              {"name": "gate", "command": mod + ["gate", "--server-class", a.server_class, "--baseline-result",
                                                 str(root / "baseline.json"), "--turbobus-result",
                                                 str(root / "pooled.json"), "--comparison",
                                                 str(root / "comparison.json"), "--evidence",
                                                 str(root / "evidence.json"), "--json-output",
                                                 str(root / "gate.json")]}]
    return {"server_class": a.server_class, "output_root": str(root), "steps": steps}


def execute_plan(plan: dict) -> dict:
    results = []
    for st in plan["steps"]:
        rc = subprocess.call(st["command"])
        results.append({"name": st["name"], "returncode": rc})
    return {**plan, "results": results}


# ---- CLI -----------------------------------------------------------------------------------------

def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("compare")
    s.add_argument("--baseline", required=True)
    s.add_argument("--turbobus", required=True)
    s.add_argument("--baseline-label", default=BASELINE_POLICY)
    s.add_argument("--turbobus-label", default=POOLED_POLICY)
    s.add_argument("--json-output")
    s = sub.add_parser("check")
    s.add_argument("result")
    s.add_argument("--json-output")
    s = sub.add_parser("evidence")
    s.add_argument("--result", required=True)
    s.add_argument("--profile")
    s.add_argument("--daemon-socket-path")
    s.add_argument("--comparison")
    s.add_argument("--json-output")
    s = sub.add_parser("gate")
    s.add_argument("--server-class", default="unknown")
    s.add_argument("--baseline-result", required=True)
    s.add_argument("--turbobus-result", required=True)
    s.add_argument("--comparison", required=True)
    s.add_argument("--evidence", action="append", default=[])
    s.add_argument("--required-workloads", default=",".join(WORKLOADS))
    s.add_argument("--json-output")
    s = sub.add_parser("inventory")
    s.add_argument("--manifest", required=True)
    s.add_argument("--json-output")
    s = sub.add_parser("ingest")
    s.add_argument("--manifest", required=True)
    s.add_argument("--gate", required=True)
    s = sub.add_parser("server-run")
    s.add_argument("--server-class", required=True, choices=SERVER_CLASSES)
    s.add_argument("--output-root", default="results/phase7")
    s.add_argument("--daemon-socket-path", default="/tmp/pcie_pool.sock")
    s.add_argument("--session-id", default="phase7")
    s.add_argument("--cpu-buffer-id", default="phase7-cpu")
    s.add_argument("--gpu-buffer-id", default="phase7-gpu")
    s.add_argument("--workloads", default="all")
    s.add_argument("--bucket-count", type=int, default=8)
    s.add_argument("--bucket-bytes", type=int, default=32 << 20)
    s.add_argument("--chunk-bytes", type=int, default=4 << 20)
    s.add_argument("--warmup", type=int, default=1)
    s.add_argument("--iterations", type=int, default=5)
    s.add_argument("--dry-run", action="store_true")
    s.add_argument("--plan-output")
    return p


def main(argv=None) -> int:
    a = build_parser().parse_args(argv)
    out = None
    if a.cmd == "compare":
        out = compare_reports(read_json(a.baseline), read_json(a.turbobus), a.baseline_label, a.turbobus_label)
    elif a.cmd == "check":
        out = check_report(read_json(a.result))
    elif a.cmd == "evidence":
        prof = read_json(a.profile) if a.profile else profile_from_daemon(a.daemon_socket_path)
        prof = prof.get("payload", prof)
        out = evidence_report(read_json(a.result), prof, read_json(a.comparison) if a.comparison else None)
    elif a.cmd == "gate":
        from .paper_validation import parse_csv

        out = gate_bundle(a.server_class, read_json(a.baseline_result), read_json(a.turbobus_result),
                          read_json(a.comparison), [read_json(e) for e in a.evidence],
                          tuple(parse_csv(a.required_workloads)))
    elif a.cmd == "inventory":
        out = inventory(read_json(a.manifest))
    elif a.cmd == "ingest":
        out = ingest(a.manifest, a.gate)
    else:
        plan = server_run_plan(a)
        out = plan if a.dry_run else execute_plan(plan)
        if a.plan_output:
            write_json(a.plan_output, plan)
    if getattr(a, "json_output", None):
        write_json(a.json_output, out)
    print(json.dumps(out, indent=2, sort_keys=True))
    ok = out.get("ok", True) and out.get("status", "accepted") != "blocked"
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
