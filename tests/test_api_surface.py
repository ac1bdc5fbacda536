"""Public surface on the CPU: package boundaries, runtime-engine
marshalling, the backend's IPC-handle checks, the offload-store state
machine, phase-7 and paper-validation tooling on synthetic reports, and the
examples' import-level entry points.  Mirrors test_package_boundaries,
test_runtime_engine, test_backend_cuda, test_offload_store,
test_phase7_* and test_paper_validation of the reference."""

import json
import subprocess
import sys

import numpy as np
import pytest


def test_control_plane_imports_without_vllm():
    code = ("import sys, pcie_pool_b200, pcie_pool_b200.daemon, pcie_pool_b200.worker, pcie_pool_b200.scheduler; "
            "print(','.join(m for m in ('vllm', 'pcie_pool_b200.adapters') if m in sys.modules))")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True).stdout.strip()
    assert out == ""


def test_daemon_requires_a_topology_provider():
    from pcie_pool_b200.daemon import TurboBusDaemon

    d = TurboBusDaemon(relay_gpus=[1])
    inv, disc = d.get_inventory(), d.discover_relays(target_gpu=0, requested_relays=[1])
    assert not inv.ok and not disc.ok
    assert "topology provider is required" in inv.error and "topology provider is required" in disc.error


def test_runtime_options_from_json(tmp_path):
    from pcie_pool_b200.runtime_engine import RuntimeOptions

    (tmp_path / "t.json").write_text(json.dumps({"best": {"chunk_bytes": 8 << 20, "staging_slots": 4}}))
    o = RuntimeOptions.from_tuning_json(tmp_path / "t.json")
    assert (o.chunk_bytes, o.staging_slots) == (8 << 20, 4)
    (tmp_path / "p.json").write_text(json.dumps({"config": {"chunk_bytes": 4 << 20, "profile_bytes": 1 << 20}}))
    o = RuntimeOptions.from_profile_json(tmp_path / "p.json")
    assert (o.chunk_bytes, o.profile_bytes) == (4 << 20, 1 << 20)
    (tmp_path / "bad.json").write_text(json.dumps({"best": 3}))
    with pytest.raises(ValueError):
        RuntimeOptions.from_tuning_json(tmp_path / "bad.json")
    assert o.planner_options().min_chunks_for_relay == 2


def test_plan_to_lanes_validation():
    from pcie_pool_b200.runtime_engine import plan_to_lanes

    plan = {"total_bytes": 3 << 20, "chunk_bytes": 1 << 20, "assignments": [
        {"path": {"kind": "direct", "enabled": True}, "chunks": [{"src_offset": 0, "dst_offset": 0, "bytes": 1 << 20}]},
        {"path": {"kind": "relay", "relay_device": 2, "enabled": True},
         "chunks": [{"src_offset": 1 << 20, "dst_offset": 1 << 20, "bytes": 2 << 20}]}]}
    lanes = plan_to_lanes(plan, 0, source_bytes=3 << 20, destination_bytes=3 << 20)
    assert [l.device for l in lanes] == [0, 2] and lanes[1].total_bytes == 2 << 20
    with pytest.raises(ValueError, match="past"):
        plan_to_lanes(plan, 0, source_bytes=2 << 20)
    bad = json.loads(json.dumps(plan))
    bad["assignments"][1]["path"]["enabled"] = False
    with pytest.raises(ValueError, match="disabled"):
        plan_to_lanes(bad, 0)
    bad = dict(plan, total_bytes=5)
    with pytest.raises(ValueError, match="total_bytes"):
        plan_to_lanes(bad, 0)


def test_profile_daemon_roundtrip():
    from pcie_pool_b200.runtime_engine import profile_from_daemon_entry, profile_to_daemon_dict

    d = {"target_device": 0, "direct_h2d_bw_gbps": 50.0, "direct_d2h_bw_gbps": 52.0,
         "relays": [{"relay_device": 3, "target_device": 0, "h2d_bw_gbps": 40.0, "d2h_bw_gbps": 41.0,
                     "p2p_bw_gbps": 700.0, "effective_bw_gbps": 40.0, "effective_d2h_bw_gbps": 41.0,
                     "p2p_enabled": True}]}
    p = profile_from_daemon_entry({"profile": d}, 0)
    assert p.relays[0].relay_device == 3 and p.direct_d2h_bw_gbps == 52.0
    assert profile_to_daemon_dict(p) == d
    with pytest.raises(ValueError):
        profile_from_daemon_entry({"profile": {"direct_h2d_bw_gbps": 0}}, 0)


def test_backend_ipc_handle_checks():
    from pcie_pool_b200.backends.cuda import coerce_ipc_handle

    h = bytes(range(64))
    assert coerce_ipc_handle(h) == h and coerce_ipc_handle(h.hex()) == h
    with pytest.raises(ValueError):
        coerce_ipc_handle(b"short")


def test_offload_store_state_machine():
    from pcie_pool_b200.offload_store import AdapterTransferContext, BlockState, OffloadStore
    from pcie_pool_b200.schema import TransferReceipt, TransferStatusState

    class Client:
        def __init__(self):
            self.intents = []

        def submit_transfer_intent(self, intent):
            self.intents.append(intent)
            return self._receipt(intent, TransferStatusState.RUNNING)

        def wait_transfer_receipt(self, intent_id, timeout_seconds=None):
            it = next(i for i in self.intents if i.intent_id == intent_id)
            return self._receipt(it, TransferStatusState.COMPLETE)

        @staticmethod
        def _receipt(it, state):
            return TransferReceipt(receipt_id="r-" + it.intent_id, ticket_id="t", intent_id=it.intent_id,
                                   decision_id="d", topology_snapshot_id="s", job_id=it.job_id,
                                   session_id=it.session_id, state=state, bytes_total=it.total_bytes,
                                   bytes_completed=it.total_bytes if state is TransferStatusState.COMPLETE else 0,
                                   started_at=0.0, path_stats=({"kind": "direct", "bytes": it.total_bytes,
                                                                "chunk_count": 1},))

    class T:
        def __init__(self, n):
            self.n = n

        def numel(self):
            return self.n

        def element_size(self):
            return 1

    c = Client()
    store = OffloadStore(c, AdapterTransferContext("j", "s", "cpu", "gpu", intent_prefix="st"))
    cpu, gpu = T(4096), T(4096)
    for i in range(4):
        store.add(f"b{i}", cpu, gpu, cpu_offset=i * 1024, gpu_offset=i * 1024, byte_count=1024)
    with pytest.raises(ValueError):
        store.add("b0", cpu, gpu)
    store.prefetch_many(["b0", "b1", "b2"])
    assert len(c.intents) == 1 and len(c.intents[0].ranges) == 3  # one batched multi-range intent
    assert c.intents[0].intent_id == "st-prefetch-1"
    assert store.block("b0").state is BlockState.PREFETCHING
    store.wait_many(["b0", "b1", "b2"])
    assert store.block("b1").state is BlockState.GPU and store.block("b3").state is BlockState.CPU
    store.evict("b1")
    store.wait("b1")
    assert store.block("b1").state is BlockState.CPU
    assert store.transfer_stats_many(["b0"]).bytes == 3072


def _report(policy, ms):
    def metric(workload, kind, job):
        return {"workload": workload, "report_schema": "x", "policy": policy, "job_id": job, "session_id": "s",
                "workload_kind": kind, "transfer_ms": ms, "performance_ms": ms, "throughput_gib_s": 1000 / ms,
                "transfer_bytes": 10, "bytes_completed": 10, "direct_bytes": 10, "relay_bytes": 0,
                "correctness_status": "complete", "decision_ids": "d1"}

    return {"config": {"policy": policy}, "workloads": [
        {"workload": "model-loading", "status": "passed", "returncode": 0, "data_path": "",
         "metrics": [metric("model-loading", "model_weights", "j")]},
        {"workload": "vllm-kv", "status": "passed", "returncode": 0, "data_path": "",
         "metrics": [metric("vllm-kv", "kv_cache", "kv0")]}]}


def test_phase7_compare_check_gate_inventory(tmp_path):
    from pcie_pool_b200.benchmarks import phase7

    base, pooled = _report("paper-baseline", 20.0), _report("turbobus-daemon", 10.0)
    cmp_ = phase7.compare_reports(base, pooled)
    row = cmp_["workloads"][0]
    assert row["p50_speedup"] == pytest.approx(2.0) and row["throughput_ratio"] == pytest.approx(2.0)
    assert phase7.check_report(pooled)["ok"]
    broken = json.loads(json.dumps(pooled))
    broken["workloads"][0]["metrics"][0]["bytes_completed"] = 3
    assert "model-loading:bytes_incomplete" in phase7.check_report(broken)["errors"]
    ev = phase7.evidence_report(pooled, {"audit_records": [{"job_id": "j", "event_type": "worker_completion"},
                                                           {"job_id": "kv0", "event_type": "worker_completion"}],
                                         "relay_quotas": {"1": {"active_chunks": 0}}, "reservations": {}},
                                cmp_)
    assert ev["ok"] and ev["metrics"][0]["audit_records"] == 1 and ev["workloads"][0]["flags"]["has_audit_record"]
    req = ("model-loading", "vllm-kv")
    gate = phase7.gate_bundle("8gpu", base, pooled, cmp_, [ev], required=req)
    assert gate["ok"] and gate["status"] == "accepted", gate["errors"]
    assert gate["warnings"] == ["correctness:not_provided"]
    # labels, provided checks and correctness artifacts can each block the bundle
    assert "baseline:policy_mismatch:paper-baseline" in phase7.gate_bundle(
        "8gpu", base, pooled, cmp_, [ev], required=req, baseline_label="other")["errors"]
    assert "turbobus:provided_check_failed" in phase7.gate_bundle(
        "8gpu", base, pooled, cmp_, [ev], required=req, turbobus_check={"ok": False})["errors"]
    assert "correctness:0:failed" in phase7.gate_bundle(
        "8gpu", base, pooled, cmp_, [ev], required=req, correctness=[{"commands": [{"returncode": 1}]}])["errors"]
    assert phase7.correctness_state({"status": "passed"}) == (True, [])
    gp = tmp_path / "gate.json"
    gp.write_text(json.dumps(gate))
    manifest = phase7.ingest(tmp_path / "manifest.json", gp)
    inv = phase7.inventory(manifest, base_dir=tmp_path)
    assert inv["accepted"] == ["8gpu"] and not inv["complete"] and inv["real_workload_accepted"]
    assert "2gpu:missing_manifest_entry" in inv["errors"]
    # a blocked class needs its environment gap and next commands
    res = phase7.ingest_entry(tmp_path / "manifest.json", phase7.build_entry("2gpu", "blocked", tmp_path / "m"))
    assert not res["written"] and "2gpu:blocked_missing_environment_gap" in res["errors"]
    res = phase7.ingest_entry(tmp_path / "manifest.json",
                              phase7.build_entry("2gpu", "blocked", tmp_path / "m", block_reason="no 2-GPU host",
                                                 next_commands=["phase7 server-run --server-class 2gpu"]),
                              allow_incomplete_inventory=True)
    assert res["written"] and res["ok"] and not res["inventory_ok"]
    assert [e["server_class"] for e in json.loads((tmp_path / "manifest.json").read_text())["server_classes"]] == \
        ["2gpu", "8gpu"]
    plan = phase7.server_run_plan(phase7.build_parser().parse_args(
        ["server-run", "--server-class", "2gpu", "--output-root", str(tmp_path), "--profile", "p.json",
         "--correctness", "c.json", "--vllm-model", "/m", "--allow-incomplete-inventory"]))
    names = [s["name"] for s in plan["steps"]]
    assert names[:2] == ["paper-validation-baseline", "paper-validation-pooled"] and names[-1] == "ingest"
    steps = {s["name"]: s["command"] for s in plan["steps"]}
    assert "--profile" in steps["evidence"] and "--correctness" in steps["gate"]
    assert "--baseline-check" in steps["gate"] and "--allow-incomplete-inventory" in steps["ingest"]
    assert steps["paper-validation-pooled"][steps["paper-validation-pooled"].index("--vllm-model") + 1] == "/m"


def test_paper_validation_dry_run_and_metric_line(tmp_path):
    from pcie_pool_b200.benchmarks import paper_validation as pv

    args = pv.build_parser().parse_args(["--session-id", "s", "--cpu-buffer-id", "c", "--gpu-buffer-id", "g",
                                         "--dry-run", "--output-dir", str(tmp_path)])
    rep = pv.run_validation(args)
    assert [w["status"] for w in rep["workloads"]] == ["dry_run"] * 4
    assert "PAPER_VALIDATION_SUMMARY_BEGIN" in pv.compact_summary(rep)
    m = pv.collect_model_metrics({"config": {"job_id": "j", "session_id": "s", "source_buffer_id": "c",
                                             "destination_buffer_id": "g", "workload_kind": "model_weights"},
                                  "summary": {"iterations": 2, "median_load_ms": 5.0, "median_gib_per_second": 2.0,
                                              "bytes": 100, "bytes_completed": 100, "decision_ids": ["d"]}},
                                 "turbobus-daemon")[0]
    assert not pv.metric_errors(m)
    assert pv.metric_line(m).startswith("paper_metric workload=model-loading report_schema=")
    # reference flags reach the workload commands
    args = pv.build_parser().parse_args(["--session-id", "s", "--cpu-buffer-id", "c", "--gpu-buffer-id", "g",
                                         "--storage-layout", "separate", "--vllm-job-count", "2",
                                         "--vllm-prompt", "hello", "--vllm-matched-tokens", "64",
                                         "--vllm-enable-multiproc-executor"])
    paths = {"json": tmp_path / "w.json", "summary": tmp_path / "w.txt"}
    ml = pv.build_workload_commands(args, "model-loading", paths)[0]
    assert ml[ml.index("--storage-layout") + 1] == "separate"
    kv = pv.build_workload_commands(args, "vllm-kv", paths)
    assert len(kv) == 2 and kv[1][kv[1].index("--prompt") + 1] == "hello"
    assert kv[0][kv[0].index("--matched-tokens") + 1] == "64" and "--enable-multiproc-executor" in kv[0]
    from pcie_pool_b200.examples.vllm_kv_connector import parse_args as kv_args

    parsed = kv_args(kv[0][kv[0].index("pcie_pool_b200.examples.vllm_kv_connector") + 1:])
    assert parsed.prompt == "hello" and parsed.disable_multiproc_executor is False


def test_examples_entry_points():
    from pcie_pool_b200.examples.framework_kv_slot_adapter import make_contiguous_slots
    from pcie_pool_b200.examples.torch_tensor_fetch import build_intent, main
    from pcie_pool_b200.examples.vllm_kv_connector import SHAPES, write_model_dir

    assert len(make_contiguous_slots("x", 3, 4096)) == 3
    cfg = json.loads(open(write_model_dir("tiny", 2048) + "/config.json").read())
    assert cfg["num_hidden_layers"] == SHAPES["tiny"]["num_hidden_layers"] and cfg["head_dim"] == 128
    args = type("A", (), dict(intent_id="i", job_id="j", session_id="s", source_buffer_id="a",
                              destination_buffer_id="b", direction="h2d", bytes=16, src_offset=0, dst_offset=0,
                              policy="p"))()
    assert build_intent(args).total_bytes == 16
    with pytest.raises(SystemExit):
        main(["--bytes", "16"])  # needs a daemon socket unless --self-contained


def test_checksum_rebase_matches_whole_buffer():
    from pcie_pool_b200.parallel.engine import Lane
    from pcie_pool_b200.utils.checksum import checksum_bytes, combine, rebase_chunk_sums

    data = np.random.default_rng(1).integers(0, 256, 4096 + 12, dtype=np.uint8)
    offs = [0, 1024, 2048, 3072, 4096]
    sizes = [1024, 1024, 1024, 1024, 12]
    lanes = [Lane(0, np.array(offs[:3], np.uint64), np.zeros(3, np.uint64), np.array(sizes[:3], np.uint64)),
             Lane(1, np.array(offs[3:], np.uint64), np.zeros(2, np.uint64), np.array(sizes[3:], np.uint64))]
    sums = [checksum_bytes(data[o:o + n]) for o, n in zip(offs, sizes)]
    assert combine(rebase_chunk_sums(sums, lanes)) == checksum_bytes(data)


def test_device_trace_events_from_stamps():
    from types import SimpleNamespace

    from pcie_pool_b200.parallel.engine import Lane
    from pcie_pool_b200.plan_trace import device_trace_events

    lanes = [Lane(0, np.array([0, 10], np.uint64), np.zeros(2, np.uint64), np.array([10, 10], np.uint64)),
             Lane(3, np.array([20], np.uint64), np.zeros(1, np.uint64), np.array([10], np.uint64))]
    tr = np.array([[1000, 1500, 4000, 4], [4000, 4000, 6000, 4], [1200, 3000, 5000, 4]], np.uint64)
    ev = device_trace_events(SimpleNamespace(trace=tr), lanes, name="x")
    assert [(e["name"], e["tid"], e["ts"], e["dur"]) for e in ev][:2] == [("x:wait", 0, 0.0, 0.5),
                                                                          ("x:move", 0, 0.5, 2.5)]
    assert {e["tid"] for e in ev} == {0, 3} and len(ev) == 6
    assert device_trace_events(SimpleNamespace(trace=None), lanes) == []


def test_native_options_backend_binding_and_prefix_release():
    """RuntimeOptions.to_native fills the engine options; bind_runtime swaps
    the native core under the CUDA backend; a saved prefix's CPU backings go
    back to the connector's pool."""
    from pcie_pool_b200.adapters.vllm_kv_connector import TurboBusCPUBackingPool, TurboBusSavedPrefix
    from pcie_pool_b200.backends.cuda import CudaNativeBackend
    from pcie_pool_b200.runtime_engine import RuntimeOptions

    o = RuntimeOptions(chunk_bytes=8 << 20, staging_slots=4, ctas_per_lane=6, timeout_s=3.0).to_native()
    assert (o.slot_bytes, o.slots, o.ctas_per_lane, o.timeout_s) == (8 << 20, 4, 6, 3.0)

    class FakeNative:
        def __init__(self):
            self.devices = []

        def set_device(self, d):
            self.devices.append(d)

    fake = FakeNative()
    be = CudaNativeBackend()
    be.bind_runtime(fake, None)
    be.set_device(3)
    assert fake.devices == [3]

    import dataclasses

    pool = TurboBusCPUBackingPool()
    fields = {f.name for f in dataclasses.fields(TurboBusSavedPrefix)}
    backing = ["layer0-backing"]
    kw = {name: None for name in fields}
    kw.update(cpu_backings=backing, block_count=2)
    prefix = TurboBusSavedPrefix(**kw)
    kv = []
    pool.release_prefix(prefix, kv)
    got, reused = pool.acquire(2, kv)
    assert reused and got is backing


def test_vllm_example_prompts_and_summary_lines():
    """The vLLM example's prompt builder (random ids, byte-level text, second
    save) and its COPY_SUMMARY lines, without an engine."""
    from pcie_pool_b200.examples.vllm_kv_connector import (build_prompts, byte_token_ids, parse_args,
                                                            prompt_text, summary_lines)

    a = parse_args(["--prompt-tokens", "100", "--suffix-tokens", "5"])
    p = build_prompts(a, 32000)
    assert len(p["first"]) == 96 and p["restore"][:96] == p["first"] and len(p["restore"]) == 101
    assert a.data_path == "engine" and a.restore_enabled and a.save_enabled

    a = parse_args(["--prompt", "ab", "--prompt-repeat", "3", "--second-prompt-suffix", "!",
                    "--second-save-prefix-key", "k2", "--second-save-prompt", "cd",
                    "--daemon-socket-path", "/tmp/x.sock", "--no-restore"])
    assert prompt_text("ab", 3) == "ab ab ab" and byte_token_ids("a", 32000) == [256 + 97]
    p = build_prompts(a, 32000)
    assert p["first"] == byte_token_ids("ab ab ab", 32000)
    assert p["restore"] == byte_token_ids("cd cd cd", 32000) + byte_token_ids("!", 32000)
    assert a.data_path == "intent" and not a.restore_enabled

    summary = {"restore_prefix_key": "k2", "matched_tokens": 0, "prompt_tokens": 8, "restore_verified": None,
               "restored_tokens": [5, 6]}
    lines = summary_lines(a, summary, {"request_id": "r1", "block_count": 1, "bytes": 10}, {})
    assert lines[0] == "COPY_SUMMARY_BEGIN" and lines[-1] == "COPY_SUMMARY_END"
    assert any(l.startswith("vllm_kv_connector_save source_request=r1") for l in lines)
    assert "generated_tokens=5,6" in lines[-2]


def test_vllm_sweep_rows_commands_and_outputs(tmp_path):
    import json

    from pcie_pool_b200.examples import vllm_kv_connector_sweep as S

    a = S.parse_args(["--restore-blocks-list", "0,4", "--case-ids", "engine,daemon",
                      "--summary-output", str(tmp_path / "s.txt"), "--cases-json-output", str(tmp_path / "c.json"),
                      "--cases-csv-output", str(tmp_path / "c.csv")])
    cmd = S.case_command(a, "daemon", 1024, 4, tmp_path / "x.log")
    assert cmd[cmd.index("--data-path") + 1] == "intent" and cmd[cmd.index("--matched-tokens") + 1] == "64"
    assert "--log-output" in cmd
    summary = {"data_path": "engine", "job_id": "j", "session_id": "s", "save_ms": 2.0, "save_cuda_ms": 1.0,
               "restore_ms": 1.0, "restore_cuda_ms": 0.5, "bytes_completed": 1 << 30, "save_blocks": 64,
               "restore_blocks": 64, "restore_verified": True, "prompt_tokens": 1024}
    row = S.case_row("engine", 1024, 0, 16, 0, "noise\nVLLM_KV_SUMMARY " + json.dumps(summary), None)
    assert row["restore_gib_s"] == "1000.000" and row["restore_verified"] is True
    bad = S.case_row("engine", 1024, 0, 16, 1, "", None)
    assert bad["save_ms"] == "NA" and bad["returncode"] == 1
    lines = S.summary_lines(a, [row, bad])
    assert lines[0] == "SWEEP_SUMMARY_BEGIN" and lines[-1] == "SWEEP_SUMMARY_END" and len(lines) == 5
    S.write_outputs(a, [row, bad], lines)
    assert json.loads((tmp_path / "c.json").read_text())[0]["case_id"] == "engine"
    assert (tmp_path / "c.csv").read_text().splitlines()[0].startswith("case_id,prompt_tokens")


def test_vllm_probe_describers_and_observer_wrapping():
    """The probe's text forms and its wrapper install/remove, on stand-in
    classes (no engine)."""
    import types

    from pcie_pool_b200.examples import vllm_probe as P

    class Blocks:
        def get_block_ids(self, allow_none=False):
            return ([3, 4],)

    assert P.describe_blocks(Blocks()) == "([3, 4],)" and P.describe_blocks(None) == "None"
    assert P.describe_value({"a": [1, 2]}) == "dict{a:list[int,int]}"
    cfg = types.SimpleNamespace(num_blocks=7, kv_cache_tensors=[1, 2], kv_cache_groups=[
        types.SimpleNamespace(layer_names=["l0", "l1"], kv_cache_spec=types.SimpleNamespace(block_size=16))])
    assert P.describe_cache_config(cfg).startswith("num_blocks=7 tensor_count=2 group_count=1 groups=[g0:layers=2")
    a = P.parse_args(["--model", "/m", "--max-tokens", "3"])
    assert a.model == "/m" and a.max_tokens == 3 and not a.run


def test_vllm_probe_observers_wrap_and_restore_vllm_methods():
    pytest.importorskip("vllm")
    from vllm.v1.core import kv_cache_manager as km
    from vllm.v1.worker import gpu_model_runner as gm

    from pcie_pool_b200.examples import vllm_probe as P

    before = (gm.GPUModelRunner.initialize_kv_cache, km.KVCacheManager.allocate_slots,
              km.KVCacheManager.get_computed_blocks)
    saved = P.install_observers(emit=lambda line: None)
    try:
        assert len(saved) == 3 and km.KVCacheManager.allocate_slots is not before[1]
        assert km.KVCacheManager.allocate_slots.__wrapped__ is before[1]
    finally:
        P.remove_observers(saved)
    assert (gm.GPUModelRunner.initialize_kv_cache, km.KVCacheManager.allocate_slots,
            km.KVCacheManager.get_computed_blocks) == before


def test_checksum_at_offsets_compose_and_unit_addresses():
    import numpy as np
    import torch

    from pcie_pool_b200.ops import unit_addresses
    from pcie_pool_b200.utils.checksum import checksum_at, checksum_bytes, combine

    data = np.random.default_rng(4).integers(0, 256, 4096 + 12, dtype=np.uint8)
    whole = checksum_bytes(data)
    parts = [checksum_at(data[a:b], a) for a, b in ((0, 1024), (1024, 3000), (3000, data.size))]
    assert combine(np.array(parts, dtype=np.uint64)) == whole
    with pytest.raises(ValueError, match="multiple of 4"):
        checksum_at(data[:8], 2)
    base = torch.zeros(64, dtype=torch.uint8)
    addrs = unit_addresses(base, 16, [3, 0, 2])
    assert addrs.tolist() == [base.data_ptr() + 48, base.data_ptr(), base.data_ptr() + 32]


def test_public_intent_example_builds_a_path_free_intent_and_reports_trace_ids():
    from pcie_pool_b200.examples import torch_tensor_fetch as ex
    from pcie_pool_b200.schema import TransferReceipt, TransferStatusState

    a = ex.build_parser().parse_args(["--daemon-socket-path", "/tmp/d.sock", "--session-id", "s1", "--job-id", "j1",
                                      "--intent-id", "i1", "--source-buffer-id", "cpu", "--destination-buffer-id",
                                      "gpu", "--bytes", "4096"])
    it = ex.build_intent(a)
    assert (it.workload_kind.value, it.direction, it.total_bytes, it.policy_hints) == ("generic", "h2d", 4096, {})
    for key in ("mode", "target_gpu", "relay_gpus", "path"):
        assert key not in it.policy_hints and key not in it.metadata
    r = TransferReceipt(receipt_id="r1", ticket_id="t1", intent_id="i1", decision_id="d1", topology_snapshot_id="x1",
                        job_id="j1", session_id="s1", state=TransferStatusState.COMPLETE, bytes_total=96,
                        bytes_completed=96, path_stats=({"kind": "direct", "bytes": 64}, {"kind": "relay", "bytes": 32}))
    line = ex.receipt_line(r)
    for want in ("decision_id=d1", "topology_snapshot_id=x1", "ticket_id=t1", "direct_bytes=64", "relay_bytes=32",
                 "state=complete"):
        assert want in line
    with pytest.raises(SystemExit):
        ex.main(["--bytes", "16"])  # a daemon socket, session and buffers are required without --self-contained
