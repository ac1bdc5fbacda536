"""Sweep the vLLM KV connector demo over prefix lengths, restore caps and
cases, one engine instance (subprocess) per point.

    python -m pcie_pool_b200.examples.vllm_kv_connector_sweep --prompt-tokens 1024,4096,16384 \\
        --restore-blocks-list 0,32 --case-ids engine,intent

Each point runs ``pcie_pool_b200.examples.vllm_kv_connector`` and reads its
``VLLM_KV_SUMMARY`` line; one JSON row per point is printed, then a
``SWEEP_SUMMARY_BEGIN`` / ``_END`` block of ``vllm_kv_connector_sweep_case``
key=value lines, and (optionally) the rows as JSON and CSV files -- the
outputs of examples/vllm_turbobus_kv_connector_sweep.py of the reference.
A case id names the data path of the point: ``engine`` (in-process pooled
engine), ``intent`` or ``daemon`` (daemon intents; ``--daemon-socket-path``
for an external daemon).  ``--matched-tokens`` of a point is its restore cap
times ``--tokens-per-block`` (0 = the whole saved prefix).
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import subprocess
import sys
from pathlib import Path

CASE_KEYS = ("case_id", "prompt_tokens", "restore_blocks", "matched_tokens", "returncode", "data_path", "job_id",
             "session_id", "save_ms", "save_cuda_ms", "restore_ms", "restore_cuda_ms", "restore_gib_s", "bytes",
             "save_blocks", "restored_blocks", "restore_verified", "log")


def csv_ints(value: str) -> list[int]:
    return [int(x) for x in str(value).split(",") if x.strip()]


def csv_strings(value: str) -> list[str]:
    return [x.strip() for x in str(value).split(",") if x.strip()]


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default=None, help="local model directory (default: random-init --shape)")
    p.add_argument("--shape", default="tiny")
    p.add_argument("--prompt", default=None, help="text prompt (default: random token ids)")
    p.add_argument("--prompt-repeat", type=int, default=64)
    p.add_argument("--second-prompt-suffix", default=" Italy")
    p.add_argument("--prompt-tokens", default="1024,4096", help="random-token mode: prefix lengths")
    p.add_argument("--restore-blocks", "--restore-blocks-list", dest="restore_blocks", default="0",
                   help="restore caps in blocks (0 = all)")
    p.add_argument("--tokens-per-block", type=int, default=16)
    p.add_argument("--case-ids", default="engine", help="comma list of engine / intent / daemon")
    p.add_argument("--job-id", default="vllm-kv-sweep-job")
    p.add_argument("--session-id", default="vllm-kv-sweep-session")
    p.add_argument("--cpu-buffer-id", default="vllm-kv-cpu-buffer")
    p.add_argument("--gpu-buffer-id", default="vllm-kv-gpu-buffer")
    p.add_argument("--prefix-key", default="sweep-prefix")
    p.add_argument("--chunk-bytes", type=int, default=4 << 20)
    p.add_argument("--relay-gpus", default="")
    p.add_argument("--daemon-socket-path", default="")
    p.add_argument("--wait-timeout-seconds", type=float, default=None)
    p.add_argument("--gpu-memory-utilization", type=float, default=0.5)
    p.add_argument("--enforce-eager", action="store_true", help="accepted; the demo runs eager by default")
    p.add_argument("--enable-multiproc-executor", action="store_true")
    p.add_argument("--log-dir", default=None, help="per-point logs (connector events + summary lines)")
    p.add_argument("--summary-output", default=None)
    p.add_argument("--cases-json-output", default=None)
    p.add_argument("--cases-csv-output", default=None)
    return p.parse_args(argv)


def case_command(a, case_id: str, n: int, rb: int, log_path: Path | None) -> list[str]:
    data_path = "engine" if case_id == "engine" else "intent"
    cmd = [sys.executable, "-m", "pcie_pool_b200.examples.vllm_kv_connector", "--shape", a.shape,
           "--prompt-tokens", str(n), "--restore-blocks", str(rb), "--relay-gpus", a.relay_gpus,
           "--gpu-memory-utilization", str(a.gpu_memory_utilization), "--data-path", data_path,
           "--job-id", a.job_id, "--session-id", f"{a.session_id}-{case_id}-blocks{rb}",
           "--cpu-buffer-id", a.cpu_buffer_id, "--gpu-buffer-id", a.gpu_buffer_id,
           "--prefix-key", f"{a.prefix_key}-{case_id}-{rb}", "--matched-tokens", str(rb * a.tokens_per_block),
           "--chunk-bytes", str(a.chunk_bytes), "--prompt-repeat", str(a.prompt_repeat),
           "--second-prompt-suffix", a.second_prompt_suffix]
    if a.model:
        cmd += ["--model", a.model]
    if a.prompt is not None:
        cmd += ["--prompt", a.prompt]
    if a.daemon_socket_path:
        cmd += ["--daemon-socket-path", a.daemon_socket_path]
    if a.wait_timeout_seconds is not None:
        cmd += ["--wait-timeout-seconds", str(a.wait_timeout_seconds)]
    if a.enable_multiproc_executor:
        cmd.append("--enable-multiproc-executor")
    if log_path is not None:
        cmd += ["--log-output", str(log_path)]
    return cmd


def case_row(case_id: str, n: int, rb: int, tokens_per_block: int, returncode: int, stdout: str,
             log_path: Path | None) -> dict:
    """One sweep row from a point's ``VLLM_KV_SUMMARY`` line ("NA" where absent)."""
    row = {k: "NA" for k in CASE_KEYS}
    row.update(case_id=case_id, prompt_tokens=n, restore_blocks=rb, matched_tokens=rb * tokens_per_block,
               returncode=returncode, log=str(log_path) if log_path else "NA")
    line = next((ln for ln in stdout.splitlines() if ln.startswith("VLLM_KV_SUMMARY ")), None)
    if line:
        s = json.loads(line[len("VLLM_KV_SUMMARY "):])
        row.update(data_path=s.get("data_path", "NA"), job_id=s.get("job_id", "NA"),
                   session_id=s.get("session_id", "NA"), save_ms=s.get("save_ms", "NA"),
                   save_cuda_ms=s.get("save_cuda_ms", "NA"), restore_ms=s.get("restore_ms", "NA"),
                   restore_cuda_ms=s.get("restore_cuda_ms", "NA"), bytes=s.get("bytes_completed", "NA"),
                   save_blocks=s.get("save_blocks", "NA"), restored_blocks=s.get("restore_blocks", "NA"),
                   restore_verified=s.get("restore_verified", "NA"), prompt_tokens=s.get("prompt_tokens", n))
        try:
            b, ms = float(row["bytes"]), float(row["restore_ms"])
            row["restore_gib_s"] = f"{b / (1 << 30) / (ms / 1e3):.3f}" if b > 0 and ms > 0 else "NA"
        except (TypeError, ValueError):
            pass
    return row


def summary_lines(a, rows: list[dict]) -> list[str]:
    cfg = ["vllm_kv_connector_sweep_config", f"cuda_visible_devices={os.environ.get('CUDA_VISIBLE_DEVICES', '')}",
           f"model={a.model or 'dummy:' + a.shape}", f"job_id={a.job_id}", f"session_id={a.session_id}",
           f"cpu_buffer_id={a.cpu_buffer_id}", f"gpu_buffer_id={a.gpu_buffer_id}", f"prompt_repeat={a.prompt_repeat}",
           f"case_ids={a.case_ids}", f"restore_blocks_list={a.restore_blocks}", f"chunk_bytes={a.chunk_bytes}",
           f"daemon_socket_path={a.daemon_socket_path}", f"wait_timeout_seconds={a.wait_timeout_seconds}"]
    out = ["SWEEP_SUMMARY_BEGIN", " ".join(cfg)]
    out += [" ".join(["vllm_kv_connector_sweep_case", *(f"{k}={r[k]}" for k in CASE_KEYS)]) for r in rows]
    out.append("SWEEP_SUMMARY_END")
    return out


def write_outputs(a, rows: list[dict], lines: list[str]) -> None:
    if a.summary_output:
        Path(a.summary_output).parent.mkdir(parents=True, exist_ok=True)
        Path(a.summary_output).write_text("\n".join(lines) + "\n", encoding="utf-8")
    if a.cases_json_output:
        Path(a.cases_json_output).parent.mkdir(parents=True, exist_ok=True)
        Path(a.cases_json_output).write_text(json.dumps(rows, indent=2) + "\n", encoding="utf-8")
    if a.cases_csv_output:
        Path(a.cases_csv_output).parent.mkdir(parents=True, exist_ok=True)
        with Path(a.cases_csv_output).open("w", encoding="utf-8", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(CASE_KEYS))
            w.writeheader()
            w.writerows(rows)


def main(argv=None) -> int:
    a = parse_args(argv)
    log_dir = Path(a.log_dir) if a.log_dir else None
    if log_dir is not None:
        log_dir.mkdir(parents=True, exist_ok=True)
    rows, failed = [], 0
    prompt_lengths = csv_ints(a.prompt_tokens) if a.prompt is None and a.model is None else [0]
    for n in prompt_lengths:
        for rb in csv_ints(a.restore_blocks):
            for case_id in csv_strings(a.case_ids):
                if case_id not in ("engine", "intent", "daemon"):
                    raise SystemExit(f"unknown case id {case_id!r} (engine, intent or daemon)")
                log_path = log_dir / f"{case_id}_tokens{n}_blocks{rb}.log" if log_dir else None
                out = subprocess.run(case_command(a, case_id, n, rb, log_path), capture_output=True, text=True)
                row = case_row(case_id, n, rb, a.tokens_per_block, out.returncode, out.stdout, log_path)
                if out.returncode != 0:
                    row["error_tail"] = (out.stderr or out.stdout)[-2000:]
                failed += out.returncode != 0
                rows.append(row)
                print(json.dumps(row), flush=True)
    lines = summary_lines(a, rows)
    print("\n".join(lines), flush=True)
    write_outputs(a, [{k: r[k] for k in CASE_KEYS} for r in rows], lines)
    print(json.dumps({"points": len(rows), "failed": failed}))
    return 1 if failed else 0


if __name__ == "__main__":
    raise SystemExit(main())
