"""Real vLLM run with the pooled KV connector: save a prompt's KV prefix to
host memory, then serve a second prompt that shares the prefix by restoring
the KV into freshly allocated (differently numbered) blocks.

    python -m pcie_pool_b200.examples.vllm_kv_connector --shape llama3-8b \\
        --prompt-tokens 4096 --relay-gpus 1,2,3 --json-output kv.json

No checkpoint or tokenizer is needed: the model directory holds only a
config.json of the chosen shape and vLLM initialises random weights
(``load_format="dummy"``); prompts are token ids.  vLLM's own prefix cache is
off, so the second prompt's prefix can only come from the connector.  The
second prompt is generated twice -- with restore, and with the connector's
restore disabled (full recompute) -- and the greedy tokens must agree.
Every connector step prints a ``turbobus_kv_connector_event`` line; the JSON
summary carries save / restore times and bytes (the fields the
paper-validation ``vllm-kv`` workload reads).  Mirrors
examples/vllm_turbobus_kv_connector.py of the reference (prompt 1 with
``do_save``, prompt 2 with ``do_restore``).
"""

from __future__ import annotations

import argparse
import json
import os
import tempfile
import time
from pathlib import Path

SHAPES = {
    "tiny": dict(hidden_size=1024, intermediate_size=3584, num_hidden_layers=8, num_attention_heads=8,
                 num_key_value_heads=8, vocab_size=32000),
    "llama3-8b": dict(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
                      num_key_value_heads=8, vocab_size=128256),
}


def write_model_dir(shape: str, max_len: int) -> str:
    d = tempfile.mkdtemp(prefix=f"ppb-{shape}-")
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_act": "silu",
           "max_position_embeddings": max(8192, max_len), "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
           "torch_dtype": "bfloat16", "tie_word_embeddings": False, "bos_token_id": 1, "eos_token_id": 2,
           "head_dim": 128, **SHAPES[shape]}
    Path(d, "config.json").write_text(json.dumps(cfg))
    return d


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--shape", choices=sorted(SHAPES), default="tiny")
    p.add_argument("--prompt-tokens", type=int, default=4096)
    p.add_argument("--suffix-tokens", type=int, default=64)
    p.add_argument("--max-tokens", type=int, default=8)
    p.add_argument("--relay-gpus", default="")
    p.add_argument("--data-path", choices=["engine", "intent"], default="engine")
    p.add_argument("--chunk-bytes", type=int, default=4 << 20)
    p.add_argument("--restore-blocks", type=int, default=0, help="cap on restored blocks (0 = all)")
    p.add_argument("--gpu-memory-utilization", type=float, default=0.5)
    p.add_argument("--session-id", default="vllm-kv-demo")
    p.add_argument("--job-id", default="vllm-kv-demo")
    p.add_argument("--prefix-key", default="demo-prefix")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--json-output", default="")
    return p.parse_args(argv)


def run(a) -> dict:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # connector events stay in this process
    import numpy as np
    from vllm import LLM, SamplingParams
    from vllm.config import KVTransferConfig
    from vllm.inputs import TokensPrompt

    from ..adapters.vllm_kv_connector import clear_connector_events, clear_saved_prefixes, get_connector_events

    clear_connector_events()
    clear_saved_prefixes()
    block = 16
    n = (a.prompt_tokens // block) * block
    model_dir = write_model_dir(a.shape, n + a.suffix_tokens + a.max_tokens + 64)
    extra = {"turbobus.job_id": a.job_id, "turbobus.session_id": a.session_id, "turbobus.chunk_bytes": a.chunk_bytes,
             "turbobus.restore_enabled": True, "turbobus.restore_block_limit": a.restore_blocks,
             "turbobus.data_path": a.data_path, "turbobus.relay_gpus": a.relay_gpus}
    t0 = time.perf_counter()
    llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True, seed=a.seed,
              enable_prefix_caching=False, max_model_len=n + a.suffix_tokens + a.max_tokens + 64, block_size=block,
              gpu_memory_utilization=a.gpu_memory_utilization, dtype="bfloat16",
              kv_transfer_config=KVTransferConfig(kv_connector="TurboBusConnector", kv_role="kv_both",
                                                  kv_connector_module_path="pcie_pool_b200.vllm_kv_connector",
                                                  kv_connector_extra_config=extra))
    init_s = time.perf_counter() - t0
    rng = np.random.default_rng(a.seed)
    vocab = SHAPES[a.shape]["vocab_size"]
    prefix = rng.integers(100, vocab - 100, n).tolist()
    suffix = rng.integers(100, vocab - 100, a.suffix_tokens).tolist()

    def sp(params):
        return SamplingParams(temperature=0.0, max_tokens=a.max_tokens, detokenize=False,
                              extra_args={"kv_transfer_params": params})

    llm.generate([TokensPrompt(prompt_token_ids=prefix)],
                 sp({"turbobus.do_save": True, "turbobus.prefix_key": a.prefix_key,
                     "turbobus.save_blocks": n // block}), use_tqdm=False)
    out_restore = llm.generate([TokensPrompt(prompt_token_ids=prefix + suffix)],
                               sp({"turbobus.do_restore": True, "turbobus.prefix_key": a.prefix_key}),
                               use_tqdm=False)
    out_plain = llm.generate([TokensPrompt(prompt_token_ids=prefix + suffix)], sp({}), use_tqdm=False)
    ev = get_connector_events()
    saves = [e for e in ev if e.get("event") == "save"]
    restores = [e for e in ev if e.get("event") == "restore"]
    matches = [e for e in ev if e.get("event") == "match"]
    toks_r = list(out_restore[0].outputs[0].token_ids)
    toks_p = list(out_plain[0].outputs[0].token_ids)
    s = saves[-1] if saves else {}
    r = restores[-1] if restores else {}
    summary = {"job_id": a.job_id, "session_id": a.session_id, "shape": a.shape, "prompt_tokens": n,
               "matched_tokens": int(matches[-1]["available_tokens"]) if matches else 0,
               "save_blocks": int(s.get("block_count", 0)), "restore_blocks": int(r.get("block_count", 0)),
               "bytes": int(s.get("bytes", 0)), "bytes_completed": int(r.get("bytes", 0)),
               "save_ms": float(s.get("total_ms", 0.0) or 0.0), "save_cuda_ms": float(s.get("cuda_ms", 0.0) or 0.0),
               "restore_ms": float(r.get("transfer_ms", 0.0) or 0.0),
               "restore_cuda_ms": float(r.get("cuda_ms", 0.0) or 0.0), "data_path": a.data_path,
               "relay_gpus": a.relay_gpus, "direct_bytes": 0, "relay_bytes": 0,
               "save_layer_count": SHAPES[a.shape]["num_hidden_layers"], "save_layer_ranges": 0,
               "restored_tokens": toks_r, "recomputed_tokens": toks_p, "restore_verified": toks_r == toks_p,
               "engine_init_s": round(init_s, 1), "events": len(ev)}
    return {"config": vars(a), "summary": summary}


def main(argv=None) -> int:
    a = parse_args(argv)
    res = run(a)
    line = json.dumps(res["summary"])
    print("VLLM_KV_SUMMARY " + line, flush=True)
    if a.json_output:
        Path(a.json_output).parent.mkdir(parents=True, exist_ok=True)
        Path(a.json_output).write_text(json.dumps(res, indent=2) + "\n")
    return 0 if res["summary"]["restore_verified"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
