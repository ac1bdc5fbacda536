"""Sweep the vLLM KV connector demo over prefix lengths and restore caps on
one engine instance per point; one JSON line per point plus a summary.
``python -m pcie_pool_b200.examples.vllm_kv_connector_sweep --prompt-tokens
1024,4096,16384 --restore-blocks 0,32``"""

from __future__ import annotations

import argparse
import json
import subprocess
import sys


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--shape", default="tiny")
    p.add_argument("--prompt-tokens", default="1024,4096")
    p.add_argument("--restore-blocks", default="0")
    p.add_argument("--relay-gpus", default="")
    p.add_argument("--gpu-memory-utilization", type=float, default=0.5)
    a = p.parse_args(argv)
    rows, failed = [], 0
    for n in [int(x) for x in a.prompt_tokens.split(",") if x]:
        for rb in [int(x) for x in a.restore_blocks.split(",") if x]:
            cmd = [sys.executable, "-m", "pcie_pool_b200.examples.vllm_kv_connector", "--shape", a.shape,
                   "--prompt-tokens", str(n), "--restore-blocks", str(rb), "--relay-gpus", a.relay_gpus,
                   "--gpu-memory-utilization", str(a.gpu_memory_utilization)]
            out = subprocess.run(cmd, capture_output=True, text=True)
            line = next((ln for ln in out.stdout.splitlines() if ln.startswith("VLLM_KV_SUMMARY ")), None)
            row = {"prompt_tokens": n, "restore_blocks": rb, "returncode": out.returncode}
            if line:
                s = json.loads(line[len("VLLM_KV_SUMMARY "):])
                row.update({k: s[k] for k in ("save_ms", "restore_ms", "save_cuda_ms", "restore_cuda_ms", "bytes",
                                              "restore_blocks", "restore_verified")})
            else:
                row["error_tail"] = (out.stderr or out.stdout)[-2000:]
            failed += out.returncode != 0
            rows.append(row)
            print(json.dumps(row), flush=True)
    print(json.dumps({"points": len(rows), "failed": failed}))
    return 1 if failed else 0


if __name__ == "__main__":
    raise SystemExit(main())
