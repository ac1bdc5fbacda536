"""Print the compact text summary of a benchmark result JSON:
``python -m pcie_pool_b200.benchmarks.summarize_result result.json``.
Dispatches on the JSON shape like turbobus benchmarks/summarize_result.py:
a paper-validation report, an intent model-loading run, a training-offload
run, or a one-line result of this package's device-timed benchmarks."""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def compact_summary_for_result(data: dict) -> str:
    if not isinstance(data, dict):
        raise ValueError("benchmark JSON must be an object")
    config, summary = data.get("config", {}) or {}, data.get("summary", {}) or {}
    if not isinstance(config, dict) or not isinstance(summary, dict):
        raise ValueError("benchmark JSON has invalid config or summary fields")
    if isinstance(data.get("workloads"), list) and isinstance(config.get("workloads"), list):
        from .paper_validation import compact_summary

        return compact_summary(data)
    if "source_buffer_id" in config and "destination_buffer_id" in config:
        from .model_loading import compact_summary

        return compact_summary(data)
    if "cpu_buffer_id" in config and "gpu_buffer_id" in config and "prefetch" in summary and "offload" in summary:
        from .training_offload import compact_summary

        return compact_summary(data)
    if "metric" in data and "value" in data:
        keys = ("metric", "value", "unit", "n_gpus", "impl", "variant", "verified")
        return " ".join(f"{k}={data[k]}" for k in keys if k in data)
    raise ValueError("unsupported benchmark JSON shape")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Print a compact benchmark summary")
    ap.add_argument("json_path")
    a = ap.parse_args(argv)
    sys.stdout.write(compact_summary_for_result(json.loads(Path(a.json_path).read_text(encoding="utf-8"))) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
