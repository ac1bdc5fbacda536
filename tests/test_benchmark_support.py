"""Benchmark support utilities: daemon CLI options, intent construction and
submission, receipt traces and their key=value lines, reservation info,
status lines and the summary dispatcher over every result shape.
Behaviours follow e2e/test_benchmark_daemon_support.py and
test_summarize_result.py of the reference with independent fakes."""

from __future__ import annotations

import argparse
import json

import pytest

from pcie_pool_b200.benchmarks import daemon_support as ds
from pcie_pool_b200.benchmarks.summarize_result import compact_summary_for_result, main as summarize_main
from pcie_pool_b200.schema import TransferReceipt, TransferStatusState, WorkloadKind


def receipt(state=TransferStatusState.COMPLETE, fallback=None):
    md = {"lease_ids": ["l1", "l2"]}
    if fallback:
        md["fallback_reason"] = fallback
    return TransferReceipt(receipt_id="r", ticket_id="tk", intent_id="i", decision_id="d", topology_snapshot_id="s",
                           job_id="j", session_id="x", state=state, bytes_total=100,
                           bytes_completed=100 if state is TransferStatusState.COMPLETE else 0,
                           error=None if state is TransferStatusState.COMPLETE else "boom",
                           path_stats=({"kind": "direct", "bytes": 60, "chunk_count": 3, "cuda_ms": 2.0},
                                       {"kind": "relay", "bytes": 40, "chunk_count": 2, "relay_device": 3,
                                        "cuda_ms": 2.5}), metadata=md)


def test_daemon_options_and_runtime_kwargs():
    p = argparse.ArgumentParser()
    ds.add_daemon_options(p)
    a = p.parse_args(["--daemon-socket-path", "/tmp/d.sock", "--daemon-max-inflight-chunks", "16"])
    kw = ds.runtime_options_kwargs(a)
    assert kw == {"daemon_socket_path": "/tmp/d.sock", "daemon_max_inflight_chunks": 16,
                  "daemon_profile_max_age_seconds": 3600.0}
    assert "daemon_socket_path" not in ds.runtime_options_kwargs(p.parse_args([]))


def test_intent_construction_and_submission():
    it = ds.make_benchmark_transfer_intent(intent_id="i", workload_kind="model_weights", job_id="j", session_id="s",
                                           source_buffer_id="a", destination_buffer_id="b", direction="h2d",
                                           total_bytes=16, ranges=[{"src_offset": 0, "dst_offset": 0, "bytes": 16}],
                                           metadata={"chunk_bytes": 8}, priority=2)
    assert it.workload_kind is WorkloadKind.MODEL_WEIGHTS and it.priority == 2 and it.metadata["chunk_bytes"] == 8

    class C:
        def __init__(self):
            self.calls = []

        def submit_transfer_intent(self, i):
            self.calls.append("submit")
            return "live"

        def wait_transfer_receipt(self, iid, timeout_seconds=None):
            self.calls.append(("wait", timeout_seconds))
            return "done"

    c = C()
    assert ds.submit_benchmark_transfer_intent(c, it) == "live" and c.calls == ["submit"]
    assert ds.submit_benchmark_transfer_intent(c, it, 5.0) == "done" and c.calls[-1] == ("wait", 5.0)


def test_receipt_trace_and_line():
    t = ds.receipt_to_trace(receipt(fallback="fairness fallback"))
    assert (t["direct_bytes"], t["relay_bytes"], t["direct_chunks"], t["relay_chunks"]) == (60, 40, 3, 2)
    assert t["measured_cuda_ms"] == 2.5 and t["state"] == "complete" and t["fallback_reason"] == "fairness fallback"
    assert t["queue_ms"] == 0.0 and t["lease_wait_ms"] == 0.0
    json.dumps(t)  # JSON ready
    line = ds.receipt_trace_line(receipt(fallback="fairness fallback"))
    assert line.startswith("daemon_receipt intent_id=i decision_id=d topology_snapshot_id=s ticket_id=tk state=")
    assert "relay_bytes=40" in line and line.endswith("fallback_reason=fairness_fallback")
    assert ds.receipt_trace_line(receipt(), prefix="x").startswith("x ")


def test_reservation_info_and_status_lines():
    class H:
        def __init__(self, r):
            self.receipt = r

    info = ds.collect_daemon_reservation_info([H(receipt()), H(receipt())])
    assert info["reservation_count"] == 4 and info["relay_gpus"] == "3"
    assert ds.daemon_profile_line({"b": 2, "a": 1, "z": None}) == "daemon_profile a=1 b=2"
    assert ds.daemon_reservation_line({}) == ""
    assert ds.benchmark_job_id("kv").startswith("benchmark-kv-")


def test_summary_dispatch_over_result_shapes(tmp_path, capsys):
    one_line = {"metric": "pooled GB/s", "value": 217.9, "unit": "GB/s", "n_gpus": 8, "impl": "ours"}
    assert compact_summary_for_result(one_line) == "metric=pooled GB/s value=217.9 unit=GB/s n_gpus=8 impl=ours"
    with pytest.raises(ValueError, match="unsupported"):
        compact_summary_for_result({"config": {}, "summary": {}})
    with pytest.raises(ValueError, match="object"):
        compact_summary_for_result([1])
    with pytest.raises(ValueError, match="invalid"):
        compact_summary_for_result({"config": [1], "summary": {}})
    p = tmp_path / "r.json"
    p.write_text(json.dumps(one_line))
    assert summarize_main([str(p)]) == 0
    assert "value=217.9" in capsys.readouterr().out


def test_relay_interference_scenarios_and_args():
    from pcie_pool_b200.benchmarks import relay_interference as ri

    a = ri.parse_args(["--scenarios", "idle,relays_busy", "--bytes", "1G", "--load-bytes", "256M"])
    assert a.scenario_list == ["idle", "relays_busy"] and ri.parse_size(a.bytes) == 1 << 30
    assert ri.loaded_devices("relays_busy", 0, [1, 2]) == [1, 2]
    assert ri.loaded_devices("target_busy", 0, [1, 2]) == [0]
    assert ri.loaded_devices("all_busy", 0, [1]) == [0, 1]
    assert ri.loaded_devices("target_link_busy", 0, [1]) == [] and ri.loaded_devices("idle", 0, [1]) == []
    with pytest.raises(SystemExit):
        ri.parse_args(["--scenarios", "idle,volcano"])


def test_op_kernel_benchmark_traffic_model_and_args():
    from pcie_pool_b200.benchmarks import op_kernels as ok

    assert ok.traffic_bytes("gather", 1 << 20) == 2 << 20
    assert ok.traffic_bytes("checksum", 1 << 20) == 1 << 20
    assert ok.traffic_bytes("adamw", 4 * 1000) == 1000 * 28, "fp32 master/m/v and bf16 grad in, all four out"
    n = 2 * 128 * 128 * 4  # 4 blocks of bf16
    assert ok.traffic_bytes("fp8", n) == n + n // 2 + 4 * 4
    assert ok.parse_args(["--kernels", "adamw,fp8"]).kernel_list == ["adamw", "fp8"]
    with pytest.raises(SystemExit):
        ok.parse_args(["--kernels", "warp-drive"])


def test_control_plane_benchmark_runs_on_cpu(capsys):
    from pcie_pool_b200.benchmarks import control_plane as cp

    assert cp.main(["--lanes", "3", "--bytes", "64M", "--chunk", "4M", "--intents", "10", "--history", "15"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["chunks"] == 16 and out["ms_per_intent"] > 0 and out["retained_transfers"] >= 35


@pytest.mark.parametrize("impl", ["ours", "reference"])
def test_daemon_protocol_benchmark_runs_on_cpu(impl, capsys):
    import os

    from pcie_pool_b200.benchmarks import control_plane

    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref", "turbobus")
    if impl == "reference" and not os.path.isdir(ref):
        pytest.skip("reference not installed under baseline/_ref")
    assert control_plane.main(["--protocol", "daemon", "--impl", impl, "--lanes", "4", "--bytes", "256M",
                               "--chunk", "16M", "--intents", "10", "--history", "5"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["impl"] == impl and out["chunks"] == 16 and out["relay_leases_per_intent"] == 3
    assert out["ms_per_intent"] > 0
