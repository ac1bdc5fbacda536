"""Every command-line entry point answers ``--help`` when started from the
repository root with no PYTHONPATH and no GPU: the benchmarks, the examples,
the daemon, the worker, the verification tool, the plan-trace tool and
``bench.py``.  A module that needs a GPU, vLLM or a daemon at import time
fails here.  One child process runs them all (``runpy``, as ``python -m``
does), so the check stays cheap.  Behaviour follows
e2e/test_benchmark_cli_entrypoints.py of the reference."""

from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MODULES = [
    *[f"pcie_pool_b200.benchmarks.{m}" for m in (
        "control_plane", "kv_offload", "land_kernel", "llama_load", "model_loading", "multi_tenant_offload",
        "op_kernels", "paper_validation", "phase7", "phase7_acceptance_inventory", "phase7_bundle_gate",
        "phase7_compare", "phase7_evidence", "phase7_ingest_artifacts", "phase7_result_check",
        "phase7_server_run", "pool_sweep", "relay_interference", "summarize_result", "training_offload")],
    *[f"pcie_pool_b200.examples.{m}" for m in (
        "torch_tensor_fetch", "vllm_kv_connector", "vllm_kv_connector_sweep", "vllm_probe")],
    "pcie_pool_b200.daemon", "pcie_pool_b200.worker", "pcie_pool_b200.verification",
]

RUNNER = r"""
import contextlib, io, json, runpy, sys
out = {}
for target in sys.argv[1:]:
    sys.argv = [target, "--help"]
    buf = io.StringIO()
    code = "no exit"
    try:
        with contextlib.redirect_stdout(buf):
            if target.endswith(".py"):
                runpy.run_path(target, run_name="__main__")
            else:
                runpy.run_module(target, run_name="__main__", alter_sys=True)
    except SystemExit as e:
        code = e.code
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        code = f"{type(e).__name__}: {e}"
    out[target] = {"code": code, "usage": "usage:" in buf.getvalue()}
print("RESULT " + json.dumps(out))
"""


def test_every_entry_point_answers_help_without_pythonpath():
    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    env["CUDA_VISIBLE_DEVICES"] = ""
    targets = MODULES + ["bench.py"]
    p = subprocess.run([sys.executable, "-c", RUNNER, *targets], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    line = next((l for l in p.stdout.splitlines() if l.startswith("RESULT ")), None)
    assert line is not None, p.stderr[-3000:]
    res = json.loads(line[len("RESULT "):])
    bad = {t: r for t, r in res.items() if r["code"] not in (0, None) or not r["usage"]}
    assert not bad, bad
    assert set(res) == set(targets)
