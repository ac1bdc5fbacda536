"""Paper validation and the phase-7 evaluation tools end to end on the CPU:
the workload subprocesses are replaced by a fake that writes each workload's
result JSON, so the orchestrator collects real-shaped results into unified
metrics; the reports then go through ``check``, ``compare``, ``evidence``,
``gate``, ``ingest`` and ``inventory`` via their command lines.  Further
tests pin each rule: failed and missing workloads, ``--keep-going``, vLLM job
identities, result checks, comparisons from per-sample data, leaked quotas,
what blocks a bundle, correctness artifact shapes, manifest shapes, the
server-run plan and the per-command module entry points.  Behaviours follow
e2e/test_paper_validation.py and e2e/test_phase7_*.py of the reference with
independent fixtures."""

from __future__ import annotations

import json
import runpy
import sys
from pathlib import Path

import pytest

from pcie_pool_b200.benchmarks import paper_validation as pv
from pcie_pool_b200.benchmarks import phase7
from pcie_pool_b200.benchmarks.summarize_result import compact_summary_for_result

MiB = 1 << 20


def _arg(cmd, flag):
    return cmd[cmd.index(flag) + 1]


class FakeRuns:
    """Stands in for the workload subprocesses: writes the result JSON each
    command would write.  ``fail`` names workloads whose command exits 1;
    ``skip`` names workloads that exit 0 without writing a result."""

    def __init__(self, ms: float = 10.0, fail=(), skip=()):
        self.ms, self.fail, self.skip, self.calls = ms, set(fail), set(skip), []

    def __call__(self, cmds, log):
        log.parent.mkdir(parents=True, exist_ok=True)
        log.write_text("\n".join(" ".join(c) for c in cmds) + "\n")
        rc = 0
        for c in cmds:
            mod = c[c.index("-m") + 1]
            out = Path(_arg(c, "--json-output"))
            if mod.endswith("model_loading"):
                w, data = "model-loading", self._model(c)
            elif mod.endswith("training_offload"):
                kind = _arg(c, "--workload-kind")
                w = "training-offload" if kind == "training_state" else "optimizer-offload"
                data = self._training(c, kind)
            else:
                w, data = "vllm-kv", self._kv(c)
            self.calls.append(w)
            if w in self.fail:
                rc = 1
                continue
            if w not in self.skip:
                out.write_text(json.dumps(data))
        return rc

    def _model(self, c):
        n = 8 * 32 * MiB
        return {"config": {"job_id": _arg(c, "--job-id"), "session_id": _arg(c, "--session-id"),
                           "source_buffer_id": _arg(c, "--source-buffer-id"),
                           "destination_buffer_id": _arg(c, "--destination-buffer-id"),
                           "workload_kind": "model_weights"},
                "summary": {"iterations": 5, "median_load_ms": self.ms, "median_gib_per_second": 25.0 / self.ms,
                            "bytes": n, "bytes_completed": n, "direct_bytes": n // 4, "relay_bytes": 3 * n // 4,
                            "decision_ids": ["d-model"], "receipt_ids": ["r-model"], "fallback_reasons": []}}

    def _training(self, c, kind):
        half = {"bytes": 64 * MiB, "bytes_completed": 64 * MiB, "direct_bytes": 16 * MiB, "relay_bytes": 48 * MiB,
                "decision_ids": ["d-" + kind], "receipt_ids": ["r-" + kind], "fallback_reasons": []}
        return {"config": {"job_id": _arg(c, "--job-id"), "session_id": _arg(c, "--session-id"),
                           "cpu_buffer_id": _arg(c, "--cpu-buffer-id"), "gpu_buffer_id": _arg(c, "--gpu-buffer-id"),
                           "workload_kind": kind},
                "summary": {"iterations": 5, "median_iteration_ms": 2 * self.ms, "median_transfer_ms": self.ms,
                            "median_compute_ms": self.ms, "median_gib_per_second": 12.5 / self.ms,
                            "prefetch": dict(half), "offload": dict(half)}}

    def _kv(self, c):
        return {"summary": {"job_id": _arg(c, "--job-id"), "session_id": _arg(c, "--session-id"), "bytes": 4 * MiB,
                            "bytes_completed": 4 * MiB, "direct_bytes": MiB, "relay_bytes": 3 * MiB,
                            "save_ms": self.ms / 2, "restore_ms": self.ms / 2, "save_layer_count": 32,
                            "save_layer_ranges": 64, "restore_verified": True}}


def validate(monkeypatch, tmp_path, policy, fake, *extra):
    monkeypatch.setattr(pv, "run_commands", fake)
    tag = "baseline" if policy == phase7.BASELINE_POLICY else "pooled"
    out = tmp_path / tag
    rc = pv.main(["--daemon-socket-path", "/tmp/none.sock", "--session-id", "s", "--job-id", f"run-{tag}",
                  "--cpu-buffer-id", "cpu", "--gpu-buffer-id", "gpu", "--policy", policy, "--output-dir", str(out),
                  "--json-output", str(out.with_suffix(".json")), "--summary-output",
                  str(out.with_suffix(".summary.txt")), "--no-copy-summary", *extra])
    return rc, json.loads(out.with_suffix(".json").read_text()), out.with_suffix(".json")


def daemon_dump(report):
    jobs = sorted({m["job_id"] for m in phase7.metrics_of(report)})
    return {"payload": {"audit_records": [{"job_id": j, "event_type": "worker_completion"} for j in jobs],
                        "relay_quotas": {"1": {"active_chunks": 0}}, "reservations": {}}}


# ---- paper validation -------------------------------------------------------------------------------

def test_paper_validation_collects_every_workload(monkeypatch, tmp_path):
    rc, rep, path = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, FakeRuns())
    assert rc == 0 and [w["status"] for w in rep["workloads"]] == ["passed"] * 4
    kinds = {m["workload"]: m["workload_kind"] for m in phase7.metrics_of(rep)}
    assert kinds == dict(pv.KIND)
    model = rep["workloads"][0]["metrics"][0]
    assert model["decision_ids"] == "d-model" and model["correctness_status"] == "complete"
    assert model["relay_bytes"] == 3 * model["transfer_bytes"] // 4
    train = rep["workloads"][1]["metrics"][0]
    assert train["transfer_bytes"] == 128 * MiB and train["prefetch_decision_ids"] == "d-training_state"
    assert all(m["log_path"].endswith(".log") for m in phase7.metrics_of(rep))
    out = path.with_suffix(".summary.txt").read_text()
    assert out.startswith("PAPER_VALIDATION_SUMMARY_BEGIN") and out.count("paper_metric ") == 4
    assert phase7.check_report(rep)["ok"]


def test_a_failed_workload_stops_the_run_unless_keep_going(monkeypatch, tmp_path):
    rc, rep, _ = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, FakeRuns(fail={"model-loading"}))
    assert rc != 0 and [w["status"] for w in rep["workloads"]] == ["failed"]
    rc, rep, _ = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, FakeRuns(fail={"model-loading"}),
                          "--keep-going")
    assert rc != 0 and [w["status"] for w in rep["workloads"]] == ["failed", "passed", "passed", "passed"]
    assert "model-loading:status_failed" in phase7.check_report(rep)["errors"]


def test_a_workload_without_a_result_is_missing_its_metrics(monkeypatch, tmp_path):
    rc, rep, _ = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, FakeRuns(skip={"training-offload"}),
                          "--keep-going")
    w = rep["workloads"][1]
    assert rc != 0 and w["status"] == "failed" and w["validation_errors"] == ["missing_paper_metrics"]
    assert {"training-offload:missing_paper_metrics", "training-offload:status_failed"} <= set(
        phase7.check_report(rep)["errors"])


def test_concurrent_vllm_jobs_keep_distinct_identities(monkeypatch, tmp_path):
    fake = FakeRuns()
    rc, rep, _ = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, fake, "--workloads", "vllm-kv",
                          "--vllm-job-count", "3")
    ms = rep["workloads"][0]["metrics"]
    assert rc == 0 and [m["job_index"] for m in ms] == [0, 1, 2] and fake.calls == ["vllm-kv"] * 3
    assert len({m["job_id"] for m in ms}) == 3 and phase7.check_report(rep)["ok"]
    assert [phase7.metric_key(m) for m in ms] == ["vllm-kv#job0", "vllm-kv#job1", "vllm-kv#job2"]
    ms[1]["job_id"] = ms[0]["job_id"]
    assert "vllm-kv:duplicate_job_identity" in phase7.check_report(rep)["errors"]


def test_unknown_workloads_are_refused():
    with pytest.raises(SystemExit):
        pv.selected_workloads("model-loading,teleport")
    assert pv.selected_workloads("all") == list(pv.WORKLOADS)
    assert pv.correctness_status(0, 0) == "missing" and pv.correctness_status(8, 4) == "incomplete"


# ---- the whole evaluation chain through the command lines ------------------------------------------

def test_evaluation_chain_accepts_a_complete_server_class(monkeypatch, tmp_path, capsys):
    _, base, bpath = validate(monkeypatch, tmp_path, phase7.BASELINE_POLICY, FakeRuns(ms=20.0))
    _, pooled, ppath = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, FakeRuns(ms=10.0))
    d = tmp_path / "2gpu"
    prof = tmp_path / "daemon.json"
    prof.write_text(json.dumps(daemon_dump(pooled)))
    steps = [["check", str(bpath), "--json-output", str(d / "baseline.check.json")],
             ["check", str(ppath), "--json-output", str(d / "pooled.check.json")],
             ["compare", "--baseline", str(bpath), "--turbobus", str(ppath), "--json-output", str(d / "cmp.json")],
             ["evidence", "--result", str(ppath), "--profile", str(prof), "--comparison", str(d / "cmp.json"),
              "--json-output", str(d / "evidence.json")],
             ["gate", "--server-class", "2gpu", "--baseline-result", str(bpath), "--turbobus-result", str(ppath),
              "--baseline-check", str(d / "baseline.check.json"), "--turbobus-check", str(d / "pooled.check.json"),
              "--comparison", str(d / "cmp.json"), "--evidence", str(d / "evidence.json"),
              "--json-output", str(d / "gate.json")],
             ["ingest", "--manifest", str(tmp_path / "manifest.json"), "--server-class", "2gpu", "--status",
              "accepted", "--bundle-gate", str(d / "gate.json"), "--real-artifacts", "--inventory-output",
              str(tmp_path / "inventory.json"), "--allow-incomplete-inventory"]]
    for s in steps:
        assert phase7.main(s) == 0, (s[0], capsys.readouterr().out[-2000:])
    cmp_ = json.loads((d / "cmp.json").read_text())
    rows = {r["workload"]: r for r in cmp_["workloads"]}
    assert rows["model-loading"]["p50_speedup"] == pytest.approx(2.0) and not cmp_["missing_workloads"]
    gate = json.loads((d / "gate.json").read_text())
    assert gate["status"] == "accepted" and gate["turbobus"]["check"]["source"] == "provided_and_computed"
    assert gate["artifacts"]["evidence"] == [str(d / "evidence.json")]
    inv = json.loads((tmp_path / "inventory.json").read_text())
    assert inv["accepted"] == ["2gpu"] and inv["real_workload_accepted"] and not inv["complete"]
    # the inventory command over the manifest agrees, and fails while classes are missing
    assert phase7.main(["inventory", "--manifest", str(tmp_path / "manifest.json")]) == 1
    assert phase7.main(["inventory", "--manifest", str(tmp_path / "manifest.json"), "--server-classes", "2gpu"]) == 0


# ---- individual rules -------------------------------------------------------------------------------

def _metric(workload="model-loading", kind="model_weights", **kw):
    m = {"workload": workload, "report_schema": pv.REPORT_SCHEMA, "policy": "p", "job_id": "j", "session_id": "s",
         "workload_kind": kind, "transfer_ms": 1.0, "performance_ms": 1.0, "transfer_bytes": 8, "bytes_completed": 8,
         "direct_bytes": 8, "relay_bytes": 0, "correctness_status": "complete", "decision_ids": "d"}
    m.update(kw)
    return m


def _rep(*metrics, status="passed", data_path=""):
    by: dict[str, list] = {}
    for m in metrics:
        by.setdefault(m["workload"], []).append(m)
    return {"config": {"policy": "p"}, "workloads": [{"workload": w, "status": status, "data_path": data_path,
                                                      "metrics": ms} for w, ms in by.items()]}


def test_result_check_rules():
    assert phase7.check_report(_rep(_metric()))["ok"]
    errs = phase7.check_report(_rep(_metric(workload_kind="kv_cache", decision_ids="", session_id="")))["errors"]
    assert errs == ["model-loading:missing_session_id", "model-loading:missing_trace_ids",
                    "model-loading:workload_kind_kv_cache"]
    assert phase7.check_report(_rep(_metric(), status="dry_run"))["ok"]
    assert phase7.check_report({"workloads": [{"workload": "x", "status": "dry_run", "metrics": []}]})["ok"]
    assert "x:missing_paper_metrics" in phase7.check_report(
        {"workloads": [{"workload": "x", "status": "passed", "metrics": []}]})["errors"]


def test_comparison_uses_per_sample_data_and_reports_missing_workloads(tmp_path):
    samples = tmp_path / "samples.json"
    samples.write_text(json.dumps({"samples": [{"load_ms": v} for v in (10.0, 20.0, 30.0, 40.0, 100.0)]}))
    base = _rep(_metric(performance_ms=99.0), _metric("vllm-kv", "kv_cache"), data_path=str(samples))
    pooled = _rep(_metric(performance_ms=10.0, throughput_gib_s=5.0))
    c = phase7.compare_reports(base, pooled)
    row = next(r for r in c["workloads"] if r["workload"] == "model-loading")
    assert row["paper-baseline"]["p50_ms"] == pytest.approx(30.0)
    assert row["paper-baseline"]["p99_ms"] == pytest.approx(phase7.percentile([10, 20, 30, 40, 100], 99))
    assert row["p50_speedup"] == pytest.approx(3.0) and row["throughput_ratio"] is None
    assert c["missing_workloads"] == ["vllm-kv"]
    assert phase7.percentile([], 50) == 0.0 and phase7.percentile([4.0], 99) == 4.0


def test_evidence_flags_untraced_metrics_leaked_quota_and_open_reservations():
    rep = _rep(_metric(job_id="a", decision_ids="d1"), _metric("vllm-kv", "kv_cache", job_id="b", decision_ids=""))
    ev = phase7.evidence_report(rep, {"audit_records": [{"decision_id": "d1", "event_type": "relay_completion",
                                                         "failure_reason": "lane 2 timed out"}],
                                      "relay_quotas": {"1": {"active_chunks": 3}, "2": {"active_chunks": 0}},
                                      "reservations": {"r": {}}})
    assert ev["errors"] == ["relay_quota_chunks_leaked", "reservations_left_open"]
    assert ev["leaked_quota_chunks"] == {"1": 3} and ev["open_reservations"] == 1
    a, b = ev["metrics"]
    assert a["audit_records"] == 1 and a["failures"] == ["lane 2 timed out"] and a["flags"]["has_trace_ids"]
    assert b["audit_records"] == 0 and not b["flags"]["has_audit_record"]


def test_each_missing_piece_blocks_the_bundle():
    req = ("model-loading",)
    base = {**_rep(_metric()), "config": {"policy": phase7.BASELINE_POLICY}}
    pooled = {**_rep(_metric()), "config": {"policy": phase7.POOLED_POLICY}}
    cmp_ = phase7.compare_reports(base, pooled)
    ev = phase7.evidence_report(pooled, {"audit_records": [{"job_id": "j"}]}, cmp_)
    assert phase7.gate_bundle("4gpu", base, pooled, cmp_, [ev], required=req)["ok"]
    assert "evidence:missing" in phase7.gate_bundle("4gpu", base, pooled, cmp_, [], required=req)["errors"]
    untraced = phase7.evidence_report(pooled, {}, cmp_)
    assert "evidence:0:missing_daemon_trace" in phase7.gate_bundle("4gpu", base, pooled, cmp_, [untraced],
                                                                   required=req)["errors"]
    g = phase7.gate_bundle("4gpu", base, pooled, {"workloads": []}, [ev], required=req + ("vllm-kv",))
    assert {"comparison:missing_workload:vllm-kv", "turbobus:missing_workload:vllm-kv",
            "real_workload:vllm_kv_missing", "evidence:missing_workload:vllm-kv"} <= set(g["errors"])
    assert g["status"] == "blocked" and g["reasons"] == g["errors"]
    lost = {**pooled, "config": {}}
    assert "turbobus:policy_mismatch:missing" in phase7.gate_bundle("4gpu", base, lost, cmp_, [ev],
                                                                    required=req)["errors"]
    no_ev_cmp = phase7.evidence_report(pooled, {"audit_records": [{"job_id": "j"}]})
    assert "evidence:0:comparison_not_attached" in phase7.gate_bundle("4gpu", base, pooled, cmp_, [no_ev_cmp],
                                                                      required=req)["warnings"]


@pytest.mark.parametrize("artifact,state", [
    ({"ok": True}, True), ({"ok": False, "errors": ["x"]}, False), ({"returncode": 0}, True),
    ({"returncode": 2}, False), ({"commands": [{"returncode": 0}, {"status": "passed"}]}, True),
    ({"commands": [{"returncode": 0}, {"returncode": 1}]}, False), ({"status": "complete"}, True),
    ({"status": "error", "error": "mismatch at 4096"}, False), ({"status": "pending"}, None), ("text", None),
    ([{"ok": True}, {"status": "???"}], True), ([], None),
])
def test_correctness_artifact_shapes(artifact, state):
    assert phase7.correctness_state(artifact)[0] is state


def test_manifest_shapes_and_entry_rules(tmp_path):
    gate = tmp_path / "gate.json"
    gate.write_text(json.dumps({"ok": True, "server_class": "8gpu", "workloads": ["model-loading", "vllm-kv"]}))
    keyed = {"server_classes": {
        "2gpu": {"status": "blocked", "block_reason": "one GPU host", "next_commands": ["run it"]},
        "4gpu": {"status": "accepted", "bundle_gate": "gate.json"},
        "8gpu": {"status": "accepted", "bundle_gate": "gate.json", "real_artifacts": True}}}
    inv = phase7.inventory(keyed, base_dir=tmp_path)
    assert inv["accepted"] == ["8gpu"] and inv["blocked_count"] == 1 and inv["real_workload_accepted"]
    assert "4gpu:accepted_requires_real_artifacts" in inv["errors"]
    assert inv["next_commands"] == [{"server_class": "2gpu", "commands": ["run it"]}]
    dup = phase7.inventory({"server_classes": [{"server_class": "2gpu", "status": "missing"},
                                               {"server_class": "2gpu", "status": "missing"}, 5]})
    assert {"2gpu:duplicate_entry", "entry_2:not_object", "2gpu:missing_missing_environment_gap",
            "phase7:no_accepted_real_llm_framework_bundle"} <= set(dup["errors"])
    bad = phase7.inventory({"server_classes": [{"server_class": "2gpu", "status": "maybe"},
                                               {"server_class": "4gpu", "status": "accepted",
                                                "bundle_gate": "nowhere.json", "real_artifacts": True}]},
                           base_dir=tmp_path)
    assert "2gpu:invalid_status:maybe" in bad["errors"]
    assert any(e.startswith("4gpu:bundle_gate_missing:") for e in bad["errors"])
    assert phase7.inventory({"server_classes": 3})["errors"][0] == "manifest:server_classes_not_list_or_object"
    res = phase7.ingest_entry(tmp_path / "m.json", {"server_class": "16gpu", "status": "accepted"})
    assert not res["written"] and "16gpu:unknown_server_class" in res["errors"]


def test_server_run_dry_run_and_execution_stop_at_the_first_failure(monkeypatch, tmp_path, capsys):
    plan_path = tmp_path / "plan.json"
    rc = phase7.main(["server-run", "--server-class", "4gpu", "--output-root", str(tmp_path), "--dry-run",
                      "--plan-output", str(plan_path), "--workloads", "model-loading,vllm-kv"])
    plan = json.loads(plan_path.read_text())
    assert rc == 0 and len(plan["steps"]) == 8 and plan["output_root"] == str(tmp_path / "4gpu")
    pooled = plan["steps"][1]["command"]
    assert _arg(pooled, "--policy") == phase7.POOLED_POLICY and _arg(pooled, "--workloads") == "model-loading,vllm-kv"
    assert "--daemon-socket-path" in plan["steps"][5]["command"], "no saved profile: ask the live daemon"
    calls = []
    monkeypatch.setattr(phase7.subprocess, "call", lambda cmd: calls.append(cmd) or (3 if len(calls) == 2 else 0))
    res = phase7.execute_plan(plan)
    assert not res["ok"] and res["failed_step"] == "paper-validation-pooled" and len(calls) == 2
    assert [r["returncode"] for r in res["results"]] == [0, 3]
    capsys.readouterr()


@pytest.mark.parametrize("module,cmd", [("phase7_compare", "compare"), ("phase7_result_check", "check"),
                                        ("phase7_evidence", "evidence"), ("phase7_bundle_gate", "gate"),
                                        ("phase7_acceptance_inventory", "inventory"),
                                        ("phase7_ingest_artifacts", "ingest"), ("phase7_server_run", "server-run")])
def test_per_command_modules_forward_to_the_sub_command(monkeypatch, module, cmd):
    seen = []
    monkeypatch.setattr(phase7, "main", lambda argv: seen.append(argv) or 0)
    monkeypatch.setattr(sys, "argv", [module, "--flag", "x"])
    with pytest.raises(SystemExit) as e:
        runpy.run_module(f"pcie_pool_b200.benchmarks.{module}", run_name="__main__")
    assert e.value.code == 0 and seen == [[cmd, "--flag", "x"]]


def test_summarize_result_prints_the_paper_validation_block(monkeypatch, tmp_path):
    _, rep, path = validate(monkeypatch, tmp_path, phase7.POOLED_POLICY, FakeRuns(), "--workloads", "model-loading")
    text = compact_summary_for_result(rep)
    assert text.splitlines()[0] == "PAPER_VALIDATION_SUMMARY_BEGIN" and "paper_metric workload=model-loading" in text
    with pytest.raises(ValueError):
        compact_summary_for_result([1])
