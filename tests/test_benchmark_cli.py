"""Intent benchmark CLIs against an in-process daemon whose executor moves
bytes through the mock lanes (CPU)."""

import json

import numpy as np
import pytest

from pcie_pool_b200 import TurboBusClient
from pcie_pool_b200.benchmarks import model_loading, summarize_result, training_offload
from pcie_pool_b200.benchmarks.daemon_support import receipt_trace_line
from pcie_pool_b200.daemon import InProcessDaemonClient, IntentExecutor, TurboBusDaemon
from pcie_pool_b200.mock import MockDataPlane, MockWorld
from pcie_pool_b200.topology import StaticTopologyProvider

MiB = 1 << 20


@pytest.fixture
def node():
    world = MockWorld(gpu_count=4)
    d = TurboBusDaemon(relay_gpus=[1, 2, 3], max_inflight_chunks_per_relay=4096,
                       topology_provider=StaticTopologyProvider(gpu_count=4),
                       executor=IntentExecutor(MockDataPlane(world)))
    d.put_profile(0, [1, 2, 3], world.profile(0))
    dc = InProcessDaemonClient(d)
    sid = dc.register_session(0, [1, 2, 3], max_inflight_chunks=4096).payload["session"]["session_id"]
    host = np.random.default_rng(0).integers(0, 256, 16 * MiB, dtype=np.uint8)
    gpu = world.alloc(0, 16 * MiB)
    return dc, sid, host, gpu


def _register(dc, job, sid, host, gpu):
    assert dc.register_job(job, session_id=sid).ok
    assert dc.register_buffer("host", job, "cpu_pinned", host.nbytes, address=host.ctypes.data, pinned=True).ok
    assert dc.register_buffer("gpu", job, "gpu", gpu.nbytes, device_index=0, address=gpu.ctypes.data).ok


def test_model_loading_cli(node, tmp_path, capsys):
    dc, sid, host, gpu = node
    _register(dc, "ml", sid, host, gpu)
    args = model_loading.build_parser().parse_args([
        "--session-id", sid, "--job-id", "ml", "--source-buffer-id", "host", "--destination-buffer-id", "gpu",
        "--bucket-count", "4", "--bucket-bytes", str(4 * MiB), "--chunk-bytes", str(MiB), "--iterations", "2",
        "--warmup", "1", "--wait-timeout-seconds", "60", "--daemon-socket-path", "unused",
        "--json-output", str(tmp_path / "ml.json")])
    res = model_loading.run_benchmark(args, client=TurboBusClient(daemon=dc))
    assert np.array_equal(gpu, host)
    s = res["summary"]
    assert s["iterations"] == 2 and s["bytes_completed"] == 16 * MiB and s["relay_bytes"] > 0
    text = model_loading.compact_summary(res)
    assert text.startswith("MODEL_LOAD_SUMMARY_BEGIN") and "model_load_receipt" in text
    model_loading.write_outputs(args, res, text)
    assert summarize_result.compact_summary_for_result(json.loads((tmp_path / "ml.json").read_text())) == text


def test_training_offload_cli_rotates_buckets(node):
    dc, sid, host, gpu = node
    _register(dc, "tr", sid, host, gpu)
    args = training_offload.build_parser().parse_args([
        "--session-id", sid, "--job-id", "tr", "--cpu-buffer-id", "host", "--gpu-buffer-id", "gpu",
        "--bucket-count", "4", "--active-buckets", "2", "--bucket-bytes", str(4 * MiB), "--chunk-bytes", str(MiB),
        "--iterations", "2", "--wait-timeout-seconds", "60", "--daemon-socket-path", "unused"])
    assert training_offload.bucket_indices(4, 2, 0) == (0, 1)
    assert training_offload.bucket_indices(4, 2, 1) == (2, 3)
    res = training_offload.run_benchmark(args, client=TurboBusClient(daemon=dc))
    assert np.array_equal(gpu, host), "prefetch of iterations 0 and 1 covered every bucket"
    s = res["summary"]
    assert s["prefetch"]["bytes"] == 8 * MiB and s["offload"]["bytes"] == 8 * MiB
    text = training_offload.compact_summary(res)
    assert "training_offload_prefetch_receipt" in text and text.endswith("TRAINING_OFFLOAD_SUMMARY_END")


def test_receipt_trace_line_format(node):
    dc, sid, host, gpu = node
    _register(dc, "tl", sid, host, gpu)
    args = model_loading.build_parser().parse_args([
        "--session-id", sid, "--job-id", "tl", "--source-buffer-id", "host", "--destination-buffer-id", "gpu",
        "--bucket-count", "1", "--bucket-bytes", str(MiB), "--iterations", "1", "--wait-timeout-seconds", "30",
        "--daemon-socket-path", "unused"])
    res = model_loading.run_benchmark(args, client=TurboBusClient(daemon=dc))
    line = receipt_trace_line(model_loading.receipt_from_trace(res["samples"][0]["receipt"]))
    assert line.startswith("daemon_receipt intent_id=") and "state=complete" in line


def test_multi_tenant_setup_and_concurrent_steps_on_mock_world():
    """The config-5 benchmark's daemon layout (one job per GPU shard, tenant
    weight split between its shards) with concurrent grads-D2H / params-H2D
    intents of two tenants on the mock world: all complete, bytes exact,
    nothing leaks."""
    from concurrent.futures import ThreadPoolExecutor

    from pcie_pool_b200 import TransferIntent
    from pcie_pool_b200.benchmarks.multi_tenant_offload import setup_tenants, shard_job

    world = MockWorld(gpu_count=4)
    d = TurboBusDaemon(relay_gpus=[0, 1, 2, 3], max_sessions_per_relay=4, max_inflight_chunks_per_relay=1 << 16,
                       topology_provider=StaticTopologyProvider(gpu_count=4),
                       executor=IntentExecutor(MockDataPlane(world), max_workers=8))
    dc = InProcessDaemonClient(d)
    n = 2 * MiB
    gpus, job_of = [0, 1, 2, 3], {0: 0, 1: 0, 2: 1, 3: 1}
    rng = np.random.default_rng(5)
    bufs = {g: (rng.integers(0, 256, n, dtype=np.uint8), np.zeros(n, np.uint8), world.alloc(g, n),
                rng.integers(0, 256, n, dtype=np.uint8)) for g in gpus}
    sessions = setup_tenants(d, dc, gpus, job_of, 2, n, {g: tuple(b.ctypes.data for b in bufs[g]) for g in gpus})
    client = TurboBusClient(daemon=dc)
    rr = ({"src_offset": 0, "dst_offset": 0, "bytes": n},)

    def one(g, kind, step=0):
        job = shard_job(job_of[g], g)
        if kind == "grads":
            it = TransferIntent(f"{job}-grads-{step}", job, sessions[g], f"dg{g}", f"hg{g}", "d2h", n, rr,
                                workload_kind="training_state", metadata={"chunk_bytes": 256 << 10})
        else:
            it = TransferIntent(f"{job}-params-{step}", job, sessions[g], f"hp{g}", f"dp{g}", "h2d", n, rr,
                                workload_kind="training_state", metadata={"chunk_bytes": 256 << 10})
        return client.transfer(it, timeout_seconds=60)

    relay_bytes = []
    with ThreadPoolExecutor(8) as pool:
        for step in range(3):  # every GPU is a target each step: after the first, none is lent
            res = list(pool.map(lambda a: one(*a), [(g, k, step) for g in gpus for k in ("grads", "params")]))
            assert all(r.state.value == "complete" for r in res), [r.error for r in res]
            relay_bytes.append(sum(int(p.get("bytes", 0)) for r in res for p in r.path_stats
                                   if p.get("kind") == "relay"))
    assert relay_bytes[1:] == [0, 0], relay_bytes
    for g in gpus:
        hp, hg, dp, dg = bufs[g]
        assert np.array_equal(dp, hp) and np.array_equal(hg, dg)
    desc = d.describe().payload
    assert desc["reservations"] == {} and all(q["active_chunks"] == 0 for q in desc["relay_quotas"].values())
    assert desc["jobs"]["job0-gpu1"]["weight"] == 0.5 and desc["jobs"]["job1-gpu2"]["user_id"] == "tenant1"


def test_multi_tenant_slow_transfers_never_wait_on_the_link_hold():
    """Two single-GPU tenants whose transfers overlap in time (each takes
    tens of ms): every intent completes well inside its timeout in every
    step (a relay kept out by the link-hold window is left out of the plan,
    never parked in delayed admission), and once both GPUs are targets
    neither is lent to the other."""
    import time
    from concurrent.futures import ThreadPoolExecutor

    from pcie_pool_b200 import TransferIntent
    from pcie_pool_b200.benchmarks.multi_tenant_offload import setup_tenants, shard_job

    class SlowPlane(MockDataPlane):
        def execute(self, *a, **k):
            time.sleep(0.04)
            return super().execute(*a, **k)

    world = MockWorld(gpu_count=2)
    d = TurboBusDaemon(relay_gpus=[0, 1], max_sessions_per_relay=2, max_inflight_chunks_per_relay=1 << 16,
                       topology_provider=StaticTopologyProvider(gpu_count=2),
                       executor=IntentExecutor(SlowPlane(world), max_workers=8))
    dc = InProcessDaemonClient(d)
    n = 4 * MiB
    gpus, job_of = [0, 1], {0: 0, 1: 1}
    rng = np.random.default_rng(9)
    bufs = {g: (rng.integers(0, 256, n, dtype=np.uint8), np.zeros(n, np.uint8), world.alloc(g, n),
                rng.integers(0, 256, n, dtype=np.uint8)) for g in gpus}
    sessions = setup_tenants(d, dc, gpus, job_of, 1, n, {g: tuple(b.ctypes.data for b in bufs[g]) for g in gpus})
    client = TurboBusClient(daemon=dc)
    rr = ({"src_offset": 0, "dst_offset": 0, "bytes": n},)

    def one(g, kind, step):
        job = shard_job(job_of[g], g)
        src, dst, direction = (f"dg{g}", f"hg{g}", "d2h") if kind == "grads" else (f"hp{g}", f"dp{g}", "h2d")
        it = TransferIntent(f"{job}-{kind}-{step}", job, sessions[g], src, dst, direction, n, rr,
                            workload_kind="training_state", metadata={"chunk_bytes": 512 << 10})
        t0 = time.perf_counter()
        r = client.transfer(it, timeout_seconds=10)
        return r, time.perf_counter() - t0

    relay_bytes = []
    with ThreadPoolExecutor(4) as pool:
        for step in range(4):
            out = list(pool.map(lambda a: one(*a), [(g, k, step) for g in gpus for k in ("grads", "params")]))
            assert all(r.state.value == "complete" for r, _ in out), [r.error for r, _ in out]
            assert max(t for _, t in out) < 5.0
            relay_bytes.append(sum(int(p.get("bytes", 0)) for r, _ in out for p in r.path_stats
                                   if p.get("kind") == "relay"))
    assert relay_bytes[1:] == [0, 0, 0], relay_bytes
    for g in gpus:
        hp, hg, dp, dg = bufs[g]
        assert np.array_equal(dp, hp) and np.array_equal(hg, dg)


def test_bench_lane_set_is_chosen_once_and_shared_by_every_rank(tmp_path):
    """bench.py: local rank 0 measures and chooses the lane set before any
    process group exists; the other ranks of the launch (same launcher
    process, same port) read its choice.  Two ranks as child processes of
    this test, the non-zero rank started first."""
    import os
    import subprocess
    import sys
    import time
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = ("import json, bench\n"
            "bench._measured_lane_set = lambda n: ([0, 4, 1, 5][:n], {'rule': 'test'})\n"
            "print(json.dumps(bench.choose_lane_set(4)))\n")
    port = str(20000 + os.getpid() % 20000)
    env = {**os.environ, "WORLD_SIZE": "2", "MASTER_PORT": port, "PYTHONPATH": str(root)}
    r1 = subprocess.Popen([sys.executable, "-c", code], cwd=root, env={**env, "LOCAL_RANK": "1", "RANK": "1"},
                          stdout=subprocess.PIPE, text=True)
    time.sleep(1.0)
    r0 = subprocess.run([sys.executable, "-c", code], cwd=root, env={**env, "LOCAL_RANK": "0", "RANK": "0"},
                        stdout=subprocess.PIPE, text=True, timeout=120)
    out1, _ = r1.communicate(timeout=120)
    a, b = json.loads(r0.stdout.strip().splitlines()[-1]), json.loads(out1.strip().splitlines()[-1])
    assert a == b == [[0, 4, 1, 5], {"rule": "test"}]
    import tempfile

    (Path(tempfile.gettempdir()) / f"ppb_lane_set_{os.getpid()}_{port}.json").unlink(missing_ok=True)


def test_bench_child_runs_report_results_crashes_and_stalls(tmp_path, monkeypatch):
    """bench.py runs the reference arm's extra figures in child processes:
    a result comes back as its JSON, a crash as its exit code and last error
    line, a stall past the limit as an error after the child's process
    group is killed."""
    import os
    import sys
    import time

    pkg = tmp_path / "childmods"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("")
    (pkg / "ok.py").write_text(
        "import json, sys\npath = sys.argv[sys.argv.index('--json-out') + 1]\n"
        "open(path, 'w').write(json.dumps({'value': 1.5, 'unit': 's'}))\n")
    (pkg / "crash.py").write_text("import sys\nprint('reference exploded', file=sys.stderr)\nsys.exit(3)\n")
    (pkg / "stall.py").write_text("import time\ntime.sleep(120)\n")
    monkeypatch.setenv("PYTHONPATH", os.pathsep.join([str(tmp_path), os.environ.get("PYTHONPATH", "")]))
    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parents[1]))
    import bench

    assert bench._child_json(["childmods.ok"], 60) == {"value": 1.5, "unit": "s"}
    r = bench._child_json(["childmods.crash"], 60)
    assert "exit code 3" in r["error"] and "exploded" in r["error"]
    t0 = time.monotonic()
    r = bench._child_json(["childmods.stall"], 2)
    assert "no result within 2 s" in r["error"] and time.monotonic() - t0 < 30
