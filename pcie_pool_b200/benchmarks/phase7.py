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
    """Join a report's metrics with the daemon's state dump: per workload the
    audit records and transfer records its trace ids (or job) match, failures
    and fallback reasons; relay quotas and reservations that were left open."""
    audit = profile.get("audit_records", []) or []
    transfers = profile.get("transfers", profile.get("statuses", {})) or {}
    transfer_jobs = {str((t or {}).get("job_id")) for t in (transfers.values() if isinstance(transfers, dict)
                                                             else transfers) if isinstance(t, dict)}
    quotas = profile.get("relay_quotas", {}) or {}
    rows, errors = [], []
    for m in metrics_of(report):
        ids = set()
        for f in TRACE_FIELDS:
            ids |= set(_split(m.get(f)))
        recs = [a for a in audit if a.get("decision_id") in ids or a.get("ticket_id") in ids
                or (a.get("job_id") and a.get("job_id") == m.get("job_id"))]
        flags = {"has_audit_record": bool(recs), "has_transfer_record": str(m.get("job_id")) in transfer_jobs,
                 "has_trace_ids": bool(ids)}
        rows.append({"workload": metric_key(m), "key": metric_key(m), "job_id": m.get("job_id"),
                     "audit_records": len(recs), "event_types": sorted({a.get("event_type") for a in recs}),
                     "failures": sorted({a.get("failure_reason") for a in recs if a.get("failure_reason")}),
                     "fallback_reason": m.get("fallback_reason", ""), "relay_bytes": int(m.get("relay_bytes", 0)),
                     "flags": flags})
    leaked = {k: q.get("active_chunks", 0) for k, q in quotas.items() if int(q.get("active_chunks", 0) or 0)}
    if leaked:
        errors.append("relay_quota_chunks_leaked")
    if profile.get("reservations"):
        errors.append("reservations_left_open")
    return {"ok": not errors, "errors": errors, "metrics": rows, "workloads": rows, "relay_quotas": quotas,
            "leaked_quota_chunks": leaked, "open_reservations": len(profile.get("reservations", {}) or {}),
            "profile_summary": {"audit_records": len(audit), "relay_quotas": len(quotas),
                                "transfers": len(transfers)},
            "comparison": None if comparison is None else {"missing_workloads": comparison.get("missing_workloads")}}


# ---- gate ----------------------------------------------------------------------------------------

def _base_workload(name) -> str:
    return str(name).split("#", 1)[0].split("[", 1)[0]


def correctness_state(data) -> tuple[bool | None, list[str]]:
    """Pass / fail / unknown of one correctness artifact: an ``ok`` flag, a
    ``returncode``, a list of ``commands`` (all must pass) or a ``status`` word."""
    if isinstance(data, list):
        states = [correctness_state(x) for x in data]
        known = [ok for ok, _ in states if ok is not None]
        errs = [e for _, es in states for e in es]
        return (all(known), errs) if known else (None, errs or ["correctness_status_unknown"])
    if not isinstance(data, dict):
        return None, ["correctness_status_unknown"]
    if "ok" in data:
        return bool(data["ok"]), [str(e) for e in data.get("errors", []) or []]
    if "returncode" in data:
        return int(data.get("returncode") or 0) == 0, []
    if "commands" in data:
        return correctness_state(data["commands"])
    st = str(data.get("status", "")).lower()
    if st in ("ok", "pass", "passed", "complete", "success"):
        return True, []
    if st in ("failed", "fail", "error"):
        return False, [str(data.get("error", "correctness_failed"))]
    return None, ["correctness_status_unknown"]


def gate_bundle(server_class: str, baseline: dict, pooled: dict, comparison: dict, evidence: list[dict],
                required=WORKLOADS, *, baseline_check: dict | None = None, turbobus_check: dict | None = None,
                correctness: list | None = None, baseline_label: str = BASELINE_POLICY,
                turbobus_label: str = POOLED_POLICY) -> dict:
    """Accept or block one server class's bundle from existing artifacts only.

    Each side must carry its policy label and every required workload and
    pass the result check (recomputed here; a provided check must pass too);
    the comparison must cover the required workloads; every evidence report
    must be clean and tie each workload to daemon records; correctness
    artifacts, when given, must pass.  When ``vllm-kv`` is required the pooled
    side must include it (the real-framework workload).  Record shape of
    turbobus benchmarks/phase7_bundle_gate.py (ok / errors / warnings and the
    per-section summaries), plus ``status`` / ``reasons``."""
    errors: list[str] = []
    warnings: list[str] = []
    sides = {}
    for side, rep, label, provided in (("baseline", baseline, baseline_label, baseline_check),
                                       ("turbobus", pooled, turbobus_label, turbobus_check)):
        policy = str((rep.get("config") or {}).get("policy", "") or "")
        if policy != label:
            errors.append(f"{side}:policy_mismatch:{policy or 'missing'}")
        have = {w.get("workload") for w in rep.get("workloads", []) or []}
        missing = [w for w in required if w not in have]
        errors += [f"{side}:missing_workload:{w}" for w in missing]
        chk = check_report(rep)
        if not chk["ok"]:
            errors.append(f"{side}:computed_check_failed")
            errors += [f"{side}:{e}" for e in chk["errors"]]
        if provided is not None and not provided.get("ok"):
            errors.append(f"{side}:provided_check_failed")
        sides[side] = {"policy": policy, "workloads": sorted(w for w in have if w), "missing_workloads": missing,
                       "check": {"ok": chk["ok"] and (provided is None or bool(provided.get("ok"))),
                                 "computed": chk, "provided": provided or {},
                                 "source": "provided_and_computed" if provided is not None else "computed"}}
    rows = comparison.get("workloads", comparison.get("comparisons", [])) or []
    cmp_workloads = {_base_workload(r.get("workload", r.get("key", ""))) for r in rows if isinstance(r, dict)}
    cmp_ok = bool(comparison.get("ok", not comparison.get("missing_workloads")))
    if not cmp_ok:
        errors.append("comparison:not_ok")
    errors += [f"comparison:missing_workload:{w}" for w in required if w not in cmp_workloads]
    ev_workloads: set[str] = set()
    ev_reports = []
    if not evidence:
        errors.append("evidence:missing")
    for i, ev in enumerate(evidence):
        if not ev.get("ok", False):
            errors.append(f"evidence:{i}:not_ok")
        items = [x for x in ev.get("workloads", ev.get("metrics", [])) or [] if isinstance(x, dict)]
        names = {_base_workload(x.get("workload", x.get("key", ""))) for x in items}
        ev_workloads |= names
        untraced = [x.get("key", x.get("workload")) for x in items
                    if not ((x.get("flags") or {}).get("has_transfer_record")
                            or (x.get("flags") or {}).get("has_audit_record") or x.get("audit_records"))]
        if untraced:
            errors.append(f"evidence:{i}:missing_daemon_trace")
        if not ev.get("comparison"):
            warnings.append(f"evidence:{i}:comparison_not_attached")
        ev_reports.append({"ok": bool(ev.get("ok")), "errors": list(ev.get("errors", []) or []),
                           "workloads": sorted(names), "missing_trace": untraced})
    errors += [f"evidence:missing_workload:{w}" for w in required if w not in ev_workloads]
    corr_reports = []
    if not correctness:
        warnings.append("correctness:not_provided")
    for i, c in enumerate(correctness or []):
        ok, errs = correctness_state(c)
        if ok is False:
            errors.append(f"correctness:{i}:failed")
        elif ok is None:
            warnings.append(f"correctness:{i}:unknown")
        corr_reports.append({"ok": ok, "errors": errs})
    if "vllm-kv" in required and "vllm-kv" not in sides["turbobus"]["workloads"]:
        errors.append("real_workload:vllm_kv_missing")
    errors = list(dict.fromkeys(errors))
    warnings = list(dict.fromkeys(warnings))
    return {"ok": not errors, "errors": errors, "warnings": warnings, "server_class": server_class,
            "status": "accepted" if not errors else "blocked", "reasons": errors,
            "required_workloads": list(required), "baseline_label": baseline_label,
            "turbobus_label": turbobus_label, "baseline": sides["baseline"], "turbobus": sides["turbobus"],
            "workloads": sides["turbobus"]["workloads"],
            "comparison": {"ok": cmp_ok, "workloads": sorted(cmp_workloads), "comparison_count": len(rows)},
            "evidence": {"ok": all(r["ok"] for r in ev_reports) and bool(ev_reports), "workloads": sorted(ev_workloads),
                         "reports": ev_reports},
            "correctness": {"provided": bool(correctness), "ok": (all(r["ok"] is True for r in corr_reports)
                                                                  if corr_reports else None),
                            "reports": corr_reports}}


def gate_files(a) -> dict:
    """The ``gate`` sub-command over artifact paths (``artifacts`` lists them)."""
    from .paper_validation import parse_csv

    out = gate_bundle(a.server_class, read_json(a.baseline_result), read_json(a.turbobus_result),
                      read_json(a.comparison), [read_json(e) for e in a.evidence],
                      tuple(parse_csv(a.required_workloads)),
                      baseline_check=read_json(a.baseline_check) if a.baseline_check else None,
                      turbobus_check=read_json(a.turbobus_check) if a.turbobus_check else None,
                      correctness=[json.loads(Path(c).read_text(encoding="utf-8")) for c in a.correctness],
                      baseline_label=a.baseline_label, turbobus_label=a.turbobus_label)
    out["artifacts"] = {"baseline_result": a.baseline_result, "turbobus_result": a.turbobus_result,
                        "baseline_check": a.baseline_check, "turbobus_check": a.turbobus_check,
                        "comparison": a.comparison, "evidence": list(a.evidence),
                        "correctness": list(a.correctness)}
    return out


# ---- inventory / ingest --------------------------------------------------------------------------

REAL_WORKLOAD = "vllm-kv"


def _as_list(v) -> list[str]:
    if v in (None, ""):
        return []
    return [str(x) for x in v if x not in (None, "")] if isinstance(v, (list, tuple, set)) else [str(v)]


def manifest_entries(manifest: dict) -> tuple[list[dict], list[str]]:
    """Entries of an acceptance manifest: ``server_classes`` (or ``servers``)
    as a list of objects or an object keyed by server class."""
    raw = manifest.get("server_classes", manifest.get("servers", []))
    if isinstance(raw, dict):
        out, errs = [], []
        for k, e in raw.items():
            if isinstance(e, dict):
                out.append({**e, "server_class": e.get("server_class", k)})
            else:
                errs.append(f"{k}:entry_not_object")
        return out, errs
    if isinstance(raw, list):
        return ([dict(e) for e in raw if isinstance(e, dict)],
                [f"entry_{i}:not_object" for i, e in enumerate(raw) if not isinstance(e, dict)])
    return [], ["manifest:server_classes_not_list_or_object"]


def _entry_bundle(entry: dict, base_dir: Path | None) -> tuple[dict, list[str]]:
    path = entry.get("bundle_gate", entry.get("bundle_gate_path", entry.get("bundle")))
    if path in (None, ""):
        return {"provided": False}, []
    bp = Path(str(path))
    if not bp.is_absolute() and base_dir is not None and not bp.exists():
        bp = base_dir / bp
    if not bp.exists():
        return {"provided": True, "path": str(bp), "exists": False, "ok": False, "workloads": [],
                "has_real_workload": False}, [f"bundle_gate_missing:{bp}"]
    b = read_json(bp)
    ok = bool(b.get("ok", b.get("status") == "accepted"))
    wl = set(_as_list(b.get("workloads")))
    for sec in ("turbobus", "baseline", "comparison", "evidence"):
        v = b.get(sec) or {}
        if isinstance(v, dict):
            wl |= {_base_workload(w) for w in _as_list(v.get("workloads"))}
    return ({"provided": True, "path": str(bp), "exists": True, "ok": ok, "server_class": b.get("server_class", ""),
             "errors": list(b.get("errors", b.get("reasons", [])) or []), "workloads": sorted(wl),
             "has_real_workload": REAL_WORKLOAD in wl}, [] if ok else ["bundle_gate_not_ok"])


def _entry_status(entry: dict) -> str:
    st = str(entry.get("status", "") or "").strip().lower()
    if st:
        return st
    return "accepted" if entry.get("bundle_gate") or entry.get("bundle_gate_path") else "missing"


def summarize_entry(entry: dict, base_dir: Path | None = None) -> tuple[dict, list[str], list[str]]:
    """One server class: an accepted class needs an ok bundle gate from real
    server artifacts that includes the real-framework workload; a blocked or
    missing class needs its environment gap and the commands to run next."""
    cls = str(entry.get("server_class", "") or "") or "unknown"
    errors, warnings = ([] if entry.get("server_class") else ["server_class_missing"]), []
    st = _entry_status(entry)
    if st not in STATUSES:
        errors.append(f"{cls}:invalid_status:{st or 'missing'}")
    bundle, berrs = _entry_bundle(entry, base_dir)
    real = bool(entry["real_artifacts"]) if "real_artifacts" in entry else \
        str(entry.get("artifact_source", "")).lower() in ("server", "real-server")
    gaps = _as_list(entry.get("environment_gaps")) + _as_list(entry.get("environment_gap"))
    block = str(entry.get("block_reason") or entry.get("missing_reason") or entry.get("environment_gap") or "")
    nexts = _as_list(entry.get("next_commands", entry.get("commands")))
    if st == "accepted":
        if not bundle.get("provided"):
            errors.append(f"{cls}:accepted_missing_bundle_gate")
        errors += [f"{cls}:{e}" for e in berrs]
        if not real:
            errors.append(f"{cls}:accepted_requires_real_artifacts")
        if not bundle.get("has_real_workload"):
            errors.append(f"{cls}:accepted_missing_vllm_kv_bundle")
    elif st in ("blocked", "missing"):
        if not block and not gaps:
            errors.append(f"{cls}:{st}_missing_environment_gap")
        if not nexts:
            errors.append(f"{cls}:{st}_missing_next_commands")
        if bundle.get("provided") and not bundle.get("ok"):
            warnings += [f"{cls}:{e}" for e in berrs]
    row = {"server_class": cls, "status": st, "ok": not errors, "real_artifacts": real, "bundle_gate": bundle,
           "bundle": bundle.get("path"), "reasons": list(entry.get("reasons", []) or []),
           "real_workload": {"name": REAL_WORKLOAD, "accepted": st == "accepted" and real and bool(bundle.get("ok"))
                             and bool(bundle.get("has_real_workload"))},
           "block_reason": block, "environment_gaps": list(dict.fromkeys(gaps)),
           "remaining_risks": _as_list(entry.get("remaining_risks", entry.get("risks"))), "next_commands": nexts,
           "notes": _as_list(entry.get("notes"))}
    return row, errors, warnings


def inventory(manifest: dict, classes=SERVER_CLASSES, base_dir: Path | None = None) -> dict:
    """Acceptance inventory of a manifest over the required server classes
    (record shape of turbobus benchmarks/phase7_acceptance_inventory.py)."""
    entries, errors = manifest_entries(manifest)
    warnings: list[str] = []
    by: dict[str, dict] = {}
    for e in entries:
        c = str(e.get("server_class", "") or "")
        if not c:
            errors.append("manifest:entry_missing_server_class")
        elif c in by:
            errors.append(f"{c}:duplicate_entry")
        else:
            by[c] = e
    rows = []
    for c in list(classes) + sorted(x for x in by if x not in classes):
        if c not in by:
            errors.append(f"{c}:missing_manifest_entry")
            rows.append({"server_class": c, "status": "missing", "ok": False, "real_artifacts": False,
                         "bundle_gate": {"provided": False}, "bundle": None, "reasons": [],
                         "real_workload": {"name": REAL_WORKLOAD, "accepted": False}, "block_reason": "",
                         "environment_gaps": [], "remaining_risks": [], "next_commands": [], "notes": []})
            continue
        row, errs, warns = summarize_entry(by[c], base_dir)
        rows.append(row)
        errors += errs
        warnings += warns
    real_ok = any(r["real_workload"]["accepted"] for r in rows)
    if not real_ok:
        errors.append("phase7:no_accepted_real_llm_framework_bundle")
    risks = [{"server_class": r["server_class"], "risk": x} for r in rows
             for x in r["remaining_risks"] + r["environment_gaps"]]
    return {"ok": not errors, "errors": list(dict.fromkeys(errors)), "warnings": list(dict.fromkeys(warnings)),
            "schema": "phase7_acceptance_inventory_v1", "server_classes": rows,
            "accepted": [r["server_class"] for r in rows if r["status"] == "accepted" and r["ok"]],
            "accepted_count": sum(r["status"] == "accepted" and r["ok"] for r in rows),
            "blocked_count": sum(r["status"] == "blocked" for r in rows),
            "missing_count": sum(r["status"] == "missing" for r in rows),
            "complete": all(r["status"] == "accepted" and r["ok"] for r in rows),
            "real_workload_accepted": real_ok,
            "next_commands": [{"server_class": r["server_class"], "commands": r["next_commands"]}
                              for r in rows if r["next_commands"]],
            "remaining_server_only_risks": risks}


def ingest_entry(manifest_path, entry: dict, classes=SERVER_CLASSES, inventory_output=None,
                 allow_incomplete_inventory: bool = False) -> dict:
    """Validate one manifest entry, upsert it (ordered by server class), write
    the manifest and rebuild the inventory (turbobus
    benchmarks/phase7_ingest_artifacts.py)."""
    mp = Path(manifest_path)
    cls, st = str(entry.get("server_class", "")), str(entry.get("status", ""))
    errors = []
    if cls not in classes:
        errors.append(f"{cls or 'missing'}:unknown_server_class")
    row, row_errors, _w = summarize_entry(entry, mp.parent)
    if st == "accepted":
        errors += [e for e in row_errors if e.endswith(("accepted_missing_bundle_gate",
                                                        "accepted_requires_real_artifacts", "bundle_gate_not_ok"))
                   or ":bundle_gate_missing:" in e]
    elif st in ("blocked", "missing"):
        errors += [e for e in row_errors if e.endswith(("_missing_environment_gap", "_missing_next_commands"))]
    else:
        errors.append(f"{cls}:invalid_status:{st or 'missing'}")
    if errors:
        return {"ok": False, "errors": errors, "manifest_path": str(mp), "updated_entry": entry, "written": False}
    manifest = read_json(mp) if mp.exists() else {"server_classes": []}
    entries, merr = manifest_entries(manifest)
    if merr:
        raise ValueError(";".join(merr))
    rest = [e for e in entries if str(e.get("server_class", "")) != cls] + [dict(entry)]
    order = {c: i for i, c in enumerate(SERVER_CLASSES)}
    rest.sort(key=lambda e: (order.get(str(e.get("server_class", "")), 99), str(e.get("server_class", ""))))
    write_json(mp, {"server_classes": rest})
    inv = inventory({"server_classes": rest}, classes, mp.parent)
    if inventory_output:
        write_json(inventory_output, inv)
    ok = inv["ok"] or allow_incomplete_inventory
    return {"ok": ok, "errors": [] if ok else inv["errors"], "manifest_path": str(mp),
            "inventory_output_path": None if inventory_output is None else str(inventory_output),
            "updated_entry": entry, "written": True, "inventory_ok": inv["ok"], "inventory": inv}


def build_entry(server_class: str, status: str, manifest_path, bundle_gate=None, real_artifacts: bool = False,
                block_reason: str = "", environment_gaps=(), next_commands=(), remaining_risks=(),
                notes=()) -> dict:
    e: dict = {"server_class": server_class, "status": status}
    if bundle_gate:
        bp, mp = Path(bundle_gate), Path(manifest_path)
        try:
            e["bundle_gate"] = bp.resolve().relative_to(mp.parent.resolve()).as_posix()
        except ValueError:
            e["bundle_gate"] = bp.as_posix()
    if real_artifacts:
        e["real_artifacts"] = True
    for key, val in (("block_reason", block_reason), ("environment_gaps", list(environment_gaps)),
                     ("next_commands", list(next_commands)), ("remaining_risks", list(remaining_risks)),
                     ("notes", list(notes))):
        if val:
            e[key] = val
    return e


def ingest(manifest_path, gate_path) -> dict:
    """Record a gate JSON as its server class's entry (status from the gate;
    the gate must come from real server artifacts).  Returns the manifest."""
    gate = read_json(gate_path)
    st = "accepted" if gate.get("ok", gate.get("status") == "accepted") else "blocked"
    entry = build_entry(gate["server_class"], st, manifest_path, bundle_gate=str(gate_path),
                        real_artifacts=st == "accepted",
                        block_reason=";".join(gate.get("errors", gate.get("reasons", [])) or [])[:500],
                        next_commands=[] if st == "accepted" else
                        [f"python -m pcie_pool_b200.benchmarks.phase7 server-run --server-class {gate['server_class']}"])
    res = ingest_entry(manifest_path, entry, allow_incomplete_inventory=True)
    if not res["written"]:
        raise ValueError(";".join(res["errors"]))
    return read_json(manifest_path)


# ---- server run plan -----------------------------------------------------------------------------

def _validation_command(a, policy: str, out_dir: Path) -> list[str]:
    rid = f"phase7-{a.server_class}-{'baseline' if policy == BASELINE_POLICY else 'turbobus'}"
    cmd = [sys.executable, "-m", "pcie_pool_b200.benchmarks.paper_validation", "--daemon-socket-path",
           a.daemon_socket_path, "--session-id", a.session_id or rid, "--job-id", rid,
           "--cpu-buffer-id", a.cpu_buffer_id or f"{rid}-cpu", "--gpu-buffer-id", a.gpu_buffer_id or f"{rid}-gpu",
           "--policy", policy, "--run-id", rid, "--workloads", a.workloads,
           "--bucket-count", str(a.bucket_count), "--bucket-bytes", str(a.bucket_bytes),
           "--chunk-bytes", str(a.chunk_bytes), "--warmup", str(a.warmup), "--iterations", str(a.iterations),
           "--vllm-job-count", str(a.vllm_job_count), "--vllm-restore-blocks", str(a.vllm_restore_blocks),
           "--vllm-matched-tokens", str(a.vllm_matched_tokens), "--vllm-prompt-repeat", str(a.vllm_prompt_repeat),
           "--output-dir", str(out_dir), "--json-output", str(out_dir.with_suffix(".json")),
           "--summary-output", str(out_dir.with_suffix(".summary.txt")), "--keep-going", "--no-copy-summary"]
    if a.vllm_model:
        cmd += ["--vllm-model", a.vllm_model]
    if a.vllm_enforce_eager:
        cmd.append("--vllm-enforce-eager")
    return cmd


def server_run_plan(a) -> dict:
    """Every step of one server class's evaluation: the baseline and pooled
    paper-validation runs, their result checks, the comparison, daemon
    evidence (a saved ``--profile`` or the live daemon), the bundle gate
    (with the checks and optional ``--correctness``) and the ingest into the
    acceptance manifest at the output root."""
    out_root = Path(a.output_root)
    root = out_root / a.server_class
    mod = [sys.executable, "-m", "pcie_pool_b200.benchmarks.phase7"]
    steps = [{"name": f"paper-validation-{tag}", "command": _validation_command(a, policy, root / tag)}
             for tag, policy in (("baseline", BASELINE_POLICY), ("pooled", POOLED_POLICY))]
    evidence = mod + ["evidence", "--result", str(root / "pooled.json"), "--comparison", str(root / "comparison.json"),
                      "--json-output", str(root / "evidence.json")]
    evidence += ["--profile", a.profile] if a.profile else ["--daemon-socket-path", a.daemon_socket_path]
    gate = mod + ["gate", "--server-class", a.server_class, "--baseline-result", str(root / "baseline.json"),
                  "--turbobus-result", str(root / "pooled.json"), "--baseline-check",
                  str(root / "baseline.check.json"), "--turbobus-check", str(root / "pooled.check.json"),
                  "--comparison", str(root / "comparison.json"), "--evidence", str(root / "evidence.json"),
                  "--json-output", str(root / "gate.json")]
    if a.correctness:
        gate += ["--correctness", a.correctness]
    ingest_cmd = mod + ["ingest", "--manifest", str(out_root / "acceptance-manifest.json"), "--server-class",
                        a.server_class, "--status", "accepted", "--bundle-gate", str(root / "gate.json"),
                        "--real-artifacts", "--inventory-output", str(out_root / "acceptance-inventory.json")]
    if a.allow_incomplete_inventory:
        ingest_cmd.append("--allow-incomplete-inventory")
    steps += [{"name": "check-baseline", "command": mod + ["check", str(root / "baseline.json"), "--json-output",
                                                            str(root / "baseline.check.json")]},
              {"name": "check-pooled", "command": mod + ["check", str(root / "pooled.json"), "--json-output",
                                                          str(root / "pooled.check.json")]},
              {"name": "compare", "command": mod + ["compare", "--baseline", str(root / "baseline.json"),
                                                    "--turbobus", str(root / "pooled.json"), "--json-output",
                                                    str(root / "comparison.json")]},
              {"name": "evidence", "command": evidence},
              {"name": "gate", "command": gate},
              {"name": "ingest", "command": ingest_cmd}]
    return {"ok": True, "server_class": a.server_class, "output_root": str(root), "steps": steps}


def execute_plan(plan: dict) -> dict:
    """Run the steps in order; stop at the first that fails."""
    done = []
    for st in plan["steps"]:
        rc = subprocess.call(st["command"])
        done.append({"name": st["name"], "returncode": rc, "command": st["command"]})
        if rc != 0:
            return {**plan, "ok": False, "failed_step": st["name"], "results": done}
    return {**plan, "ok": True, "results": done}


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
    s.add_argument("--profile", help="saved daemon describe/PROFILE JSON (default: ask --daemon-socket-path)")
    s.add_argument("--daemon-socket-path")
    s.add_argument("--comparison")
    s.add_argument("--json-output")
    s = sub.add_parser("gate")
    s.add_argument("--server-class", default="unknown")
    s.add_argument("--baseline-result", required=True)
    s.add_argument("--turbobus-result", required=True)
    s.add_argument("--baseline-check", help="result-check JSON of the baseline side (must pass)")
    s.add_argument("--turbobus-check", help="result-check JSON of the pooled side (must pass)")
    s.add_argument("--comparison", required=True)
    s.add_argument("--evidence", action="append", default=[])
    s.add_argument("--correctness", action="append", default=[], help="correctness artifact JSON (repeatable)")
    s.add_argument("--required-workloads", default=",".join(WORKLOADS))
    s.add_argument("--baseline-label", default=BASELINE_POLICY)
    s.add_argument("--turbobus-label", default=POOLED_POLICY)
    s.add_argument("--json-output")
    s = sub.add_parser("inventory")
    s.add_argument("--manifest", required=True)
    s.add_argument("--server-classes", default=",".join(SERVER_CLASSES))
    s.add_argument("--json-output")
    s = sub.add_parser("ingest")
    s.add_argument("--manifest", required=True)
    s.add_argument("--gate", help="gate JSON: records its server class with the gate's verdict")
    s.add_argument("--server-class")
    s.add_argument("--status", choices=STATUSES)
    s.add_argument("--bundle-gate", help="bundle-gate JSON path of an accepted server class")
    s.add_argument("--real-artifacts", action="store_true", help="the artifacts come from a real server run")
    s.add_argument("--block-reason", default="")
    s.add_argument("--environment-gap", action="append", default=[])
    s.add_argument("--next-command", action="append", default=[])
    s.add_argument("--remaining-risk", action="append", default=[])
    s.add_argument("--note", action="append", default=[])
    s.add_argument("--server-classes", default=",".join(SERVER_CLASSES))
    s.add_argument("--inventory-output")
    s.add_argument("--allow-incomplete-inventory", action="store_true",
                   help="write the entry even while other server classes are still missing")
    s = sub.add_parser("server-run")
    s.add_argument("--server-class", required=True, choices=SERVER_CLASSES)
    s.add_argument("--output-root", default="results/phase7")
    s.add_argument("--daemon-socket-path", default="/tmp/pcie_pool.sock")
    s.add_argument("--profile", help="saved daemon PROFILE JSON for the evidence step")
    s.add_argument("--correctness", help="correctness artifact JSON for the gate")
    s.add_argument("--session-id", default="")
    s.add_argument("--cpu-buffer-id", default="")
    s.add_argument("--gpu-buffer-id", default="")
    s.add_argument("--workloads", default="all")
    s.add_argument("--bucket-count", type=int, default=8)
    s.add_argument("--bucket-bytes", type=int, default=32 << 20)
    s.add_argument("--chunk-bytes", type=int, default=4 << 20)
    s.add_argument("--warmup", type=int, default=1)
    s.add_argument("--iterations", type=int, default=5)
    s.add_argument("--vllm-model", default="")
    s.add_argument("--vllm-job-count", type=int, default=1)
    s.add_argument("--vllm-restore-blocks", type=int, default=0)
    s.add_argument("--vllm-matched-tokens", type=int, default=0)
    s.add_argument("--vllm-prompt-repeat", type=int, default=64)
    s.add_argument("--vllm-enforce-eager", action="store_true")
    s.add_argument("--allow-incomplete-inventory", action="store_true")
    s.add_argument("--dry-run", action="store_true")
    s.add_argument("--plan-output")
    return p


def main(argv=None) -> int:
    from .paper_validation import parse_csv

    a = build_parser().parse_args(argv)
    out = None
    if a.cmd == "compare":
        out = compare_reports(read_json(a.baseline), read_json(a.turbobus), a.baseline_label, a.turbobus_label)
    elif a.cmd == "check":
        out = check_report(read_json(a.result))
    elif a.cmd == "evidence":
        if not a.profile and not a.daemon_socket_path:
            raise SystemExit("evidence needs --profile or --daemon-socket-path")
        prof = read_json(a.profile) if a.profile else profile_from_daemon(a.daemon_socket_path)
        prof = prof.get("payload", prof)
        out = evidence_report(read_json(a.result), prof, read_json(a.comparison) if a.comparison else None)
    elif a.cmd == "gate":
        out = gate_files(a)
    elif a.cmd == "inventory":
        out = inventory(read_json(a.manifest), tuple(parse_csv(a.server_classes)), Path(a.manifest).parent)
        out["manifest_path"] = str(a.manifest)
    elif a.cmd == "ingest":
        if a.gate and not a.status:
            out = inventory(ingest(a.manifest, a.gate), tuple(parse_csv(a.server_classes)), Path(a.manifest).parent)
            out["ok"] = True
        else:
            if not a.server_class or not a.status:
                raise SystemExit("ingest needs --gate, or --server-class and --status")
            entry = build_entry(a.server_class, a.status, a.manifest, bundle_gate=a.bundle_gate or a.gate,
                                real_artifacts=a.real_artifacts, block_reason=a.block_reason,
                                environment_gaps=a.environment_gap, next_commands=a.next_command,
                                remaining_risks=a.remaining_risk, notes=a.note)
            out = ingest_entry(a.manifest, entry, tuple(parse_csv(a.server_classes)), a.inventory_output,
                               a.allow_incomplete_inventory)
    else:
        plan = server_run_plan(a)
        out = plan if a.dry_run else execute_plan(plan)
        if a.plan_output:
            write_json(a.plan_output, plan)
    if getattr(a, "json_output", None):
        write_json(a.json_output, out)
    print(json.dumps(out, indent=2, sort_keys=True, default=str))
    ok = out.get("ok", True) and out.get("status", "accepted") != "blocked"
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
