"""Real vLLM run with the pooled KV connector: save a prompt's KV prefix to
host memory, then serve a second prompt that shares the prefix by restoring
the KV into freshly allocated (differently numbered) blocks.

    python -m pcie_pool_b200.examples.vllm_kv_connector --shape llama3-8b \\
        --prompt-tokens 4096 --relay-gpus 1,2,3 --json-output kv.json

No checkpoint or tokenizer is needed: by default the model directory holds
only a config.json of the chosen shape and vLLM initialises random weights
(``load_format="dummy"``); prompts are random token ids, or, with
``--prompt``, the repeated text as byte-level ids.  ``--model DIR`` runs a
local checkpoint with its tokenizer instead.  The reference example's flags
are accepted (``--prompt/--prompt-repeat/--second-prompt-suffix``,
``--second-save-prefix-key/--second-save-prompt``, ``--matched-tokens``,
``--restore-blocks``, ``--max-saved-prefixes``, ``--save-enabled/--no-save``,
``--restore-enabled``, buffer and session ids, ``--daemon-socket-path``,
``--wait-timeout-seconds``, ``--log-output``, engine flags); restore is on by
default here (``--no-restore`` turns it off).  vLLM's own prefix cache is
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
    # model and prompts
    p.add_argument("--model", default=None,
                   help="local model directory with weights and tokenizer (default: a random-init --shape model)")
    p.add_argument("--shape", choices=sorted(SHAPES), default="tiny")
    p.add_argument("--prompt", default=None,
                   help="text prompt (tokenised by --model's tokenizer, else byte-level); default: random token ids")
    p.add_argument("--prompt-repeat", type=int, default=64, help="the text prompt is repeated this many times")
    p.add_argument("--second-prompt-suffix", default=" Italy", help="text appended to the restored prompt")
    p.add_argument("--prompt-tokens", type=int, default=4096, help="random-token mode: prefix length")
    p.add_argument("--suffix-tokens", type=int, default=64, help="random-token mode: suffix length")
    p.add_argument("--second-save-prefix-key", default=None,
                   help="also save a second prompt under this key and restore that one")
    p.add_argument("--second-save-prompt", default="The capital of Germany is")
    p.add_argument("--max-tokens", type=int, default=8)
    # engine
    p.add_argument("--tensor-parallel-size", type=int, default=1)
    p.add_argument("--gpu-memory-utilization", type=float, default=0.5)
    p.add_argument("--enforce-eager", dest="enforce_eager", action="store_true", default=True)
    p.add_argument("--no-enforce-eager", dest="enforce_eager", action="store_false",
                   help="let vLLM capture CUDA graphs")
    p.add_argument("--enable-multiproc-executor", dest="disable_multiproc_executor", action="store_false",
                   help="run the engine core in its own process (connector events then stay there)")
    p.set_defaults(disable_multiproc_executor=True)
    p.add_argument("--seed", type=int, default=0)
    # connector
    p.add_argument("--job-id", default="vllm-kv-demo")
    p.add_argument("--session-id", default="vllm-kv-demo")
    p.add_argument("--cpu-buffer-id", default="vllm-kv-cpu-buffer")
    p.add_argument("--gpu-buffer-id", default="vllm-kv-gpu-buffer")
    p.add_argument("--prefix-key", default="demo-prefix")
    p.add_argument("--matched-tokens", type=int, default=0, help="tokens to restore (0 = the whole saved prefix)")
    p.add_argument("--restore-blocks", type=int, default=0, help="cap on saved / restored blocks (0 = all)")
    p.add_argument("--max-saved-prefixes", type=int, default=0, help="LRU bound on saved prefixes (0 = none)")
    p.add_argument("--save-enabled", dest="save_enabled", action="store_true", default=True)
    p.add_argument("--no-save", dest="save_enabled", action="store_false")
    p.add_argument("--restore-enabled", dest="restore_enabled", action="store_true", default=True)
    p.add_argument("--no-restore", dest="restore_enabled", action="store_false")
    p.add_argument("--relay-gpus", default="")
    p.add_argument("--data-path", choices=["engine", "intent"], default=None,
                   help="engine: in-process pooled engine; intent: daemon intents (default: intent when "
                        "--daemon-socket-path is given, else engine)")
    p.add_argument("--daemon-socket-path", default="")
    p.add_argument("--chunk-bytes", type=int, default=4 << 20)
    p.add_argument("--wait-timeout-seconds", type=float, default=None)
    # output
    p.add_argument("--json-output", default="")
    p.add_argument("--log-output", default=None, help="also write the summary lines and connector events here")
    a = p.parse_args(argv)
    if a.data_path is None:
        a.data_path = "intent" if a.daemon_socket_path else "engine"
    return a


def prompt_text(prompt: str, repeat: int) -> str:
    """``repeat`` copies of ``prompt`` joined by spaces."""
    return prompt if repeat <= 1 else " ".join([prompt] * repeat)


def byte_token_ids(text: str, vocab: int) -> list[int]:
    """Byte-level token ids for a model without a tokenizer: UTF-8 byte b -> 256 + b."""
    if vocab < 512:
        raise ValueError("vocabulary too small for byte-level token ids")
    return [256 + b for b in text.encode("utf-8")]


def build_prompts(a, vocab: int, encode=None) -> dict[str, list[int]]:
    """Token ids of the saved prompt(s) and the restored prompt.

    Random-token mode (no ``--prompt`` and no ``--model``): ``--prompt-tokens``
    random ids (rounded down to whole 16-token blocks) and ``--suffix-tokens``
    more.  Text mode: the repeated prompt through ``encode`` (the model's
    tokenizer) or byte-level ids; the suffix is encoded on its own and
    appended, so the restored prompt starts with exactly the saved tokens.
    """
    import numpy as np

    block = 16
    out: dict[str, list[int]] = {}
    if a.prompt is None and a.model is None:
        rng = np.random.default_rng(a.seed)
        n = (a.prompt_tokens // block) * block
        out["first"] = rng.integers(100, vocab - 100, n).tolist()
        suffix = rng.integers(100, vocab - 100, a.suffix_tokens).tolist()
        if a.second_save_prefix_key:
            out["second_save"] = np.random.default_rng(a.seed + 1).integers(100, vocab - 100, n).tolist()
    else:
        enc = encode or (lambda t: byte_token_ids(t, vocab))
        out["first"] = list(enc(prompt_text(a.prompt or "The capital of France is", a.prompt_repeat)))
        suffix = list(enc(a.second_prompt_suffix))
        if a.second_save_prefix_key:
            out["second_save"] = list(enc(prompt_text(a.second_save_prompt, a.prompt_repeat)))
    base = out["second_save"] if a.second_save_prefix_key else out["first"]
    out["restore"] = base + suffix
    return out


def summary_lines(a, summary: dict, save: dict, restore: dict) -> list[str]:
    """Key=value summary lines between COPY_SUMMARY_BEGIN / _END (the layout
    examples/vllm_turbobus_kv_connector.py of the reference prints)."""
    def kv(tag: str, **fields) -> str:
        return " ".join([tag, *(f"{k}={v}" for k, v in fields.items())])

    receipt = {k: (save or {}).get(k, 0) for k in ("direct_bytes", "relay_bytes")}
    lines = ["COPY_SUMMARY_BEGIN",
             kv("vllm_kv_connector_config", model=a.model or f"dummy:{a.shape}", job_id=a.job_id,
                session_id=a.session_id, cpu_buffer_id=a.cpu_buffer_id, gpu_buffer_id=a.gpu_buffer_id,
                daemon_socket_path=a.daemon_socket_path, wait_timeout_seconds=a.wait_timeout_seconds,
                cuda_visible_devices=os.environ.get("CUDA_VISIBLE_DEVICES", ""), prompt_repeat=a.prompt_repeat,
                prefix_key=a.prefix_key, second_save_prefix_key=a.second_save_prefix_key,
                restore_prefix_key=summary["restore_prefix_key"], matched_tokens=summary["matched_tokens"],
                restore_blocks=a.restore_blocks, save_enabled=a.save_enabled, restore_enabled=a.restore_enabled,
                max_saved_prefixes=a.max_saved_prefixes, chunk_bytes=a.chunk_bytes, data_path=a.data_path),
             kv("vllm_kv_connector_scenario", type="real_vllm_kv_transfer_connector",
                boundary="KVConnectorBase_V1", entry="start_load_kv")]
    if save:
        lines.append(kv("vllm_kv_connector_save", source_request=save.get("request_id", "unknown"),
                        blocks=save.get("block_count", 0), bytes=save.get("bytes", 0),
                        total_ms=save.get("total_ms", 0), cuda_ms=save.get("cuda_ms", 0), **receipt))
    if restore:
        lines.append(kv("vllm_kv_connector_restore", request_id=restore.get("request_id", "unknown"),
                        prefix_key=restore.get("prefix_key", summary["restore_prefix_key"]),
                        bytes=restore.get("bytes", 0), transfer_ms=restore.get("transfer_ms", 0),
                        cuda_ms=restore.get("cuda_ms", 0)))
    lines.append(kv("vllm_kv_connector_result", prompt_tokens=summary["prompt_tokens"],
                    restore_verified=summary["restore_verified"],
                    generated_tokens=",".join(str(t) for t in summary["restored_tokens"])))
    lines.append("COPY_SUMMARY_END")
    return lines


def run(a) -> dict:
    if a.disable_multiproc_executor:
        os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # connector events stay in this process
    from vllm import LLM, SamplingParams
    from vllm.config import KVTransferConfig
    from vllm.inputs import TokensPrompt

    from ..adapters.vllm_kv_connector import clear_connector_events, clear_saved_prefixes, get_connector_events

    clear_connector_events()
    clear_saved_prefixes()
    block = 16
    extra = {"turbobus.job_id": a.job_id, "turbobus.session_id": a.session_id, "turbobus.chunk_bytes": a.chunk_bytes,
             "turbobus.cpu_buffer_id": a.cpu_buffer_id, "turbobus.gpu_buffer_id": a.gpu_buffer_id,
             "turbobus.restore_enabled": a.restore_enabled, "turbobus.restore_block_limit": a.restore_blocks,
             "turbobus.max_saved_prefixes": a.max_saved_prefixes,
             "turbobus.data_path": a.data_path, "turbobus.relay_gpus": a.relay_gpus}
    if a.daemon_socket_path:
        extra["turbobus.daemon_socket_path"] = a.daemon_socket_path
    if a.wait_timeout_seconds is not None:
        extra["turbobus.wait_timeout_seconds"] = a.wait_timeout_seconds
    ktc = KVTransferConfig(kv_connector="TurboBusConnector", kv_role="kv_both",
                           kv_connector_module_path="pcie_pool_b200.vllm_kv_connector",
                           kv_connector_extra_config=extra)
    if a.model is None:
        prompts = build_prompts(a, SHAPES[a.shape]["vocab_size"])
        max_prompt = max(len(v) for v in prompts.values())
        model_dir = write_model_dir(a.shape, max_prompt + a.max_tokens + 64)
        llm_kw = dict(model=model_dir, load_format="dummy", skip_tokenizer_init=True,
                      max_model_len=max_prompt + a.max_tokens + 64, dtype="bfloat16")
    else:
        llm_kw = dict(model=a.model)
    t0 = time.perf_counter()
    llm = LLM(**llm_kw, enforce_eager=a.enforce_eager, seed=a.seed, enable_prefix_caching=False, block_size=block,
              tensor_parallel_size=a.tensor_parallel_size, gpu_memory_utilization=a.gpu_memory_utilization,
              kv_transfer_config=ktc)
    init_s = time.perf_counter() - t0
    if a.model is not None:
        tok = llm.get_tokenizer()
        prompts = build_prompts(a, int(getattr(tok, "vocab_size", 1 << 16)),
                                encode=lambda t: tok.encode(t, add_special_tokens=False))

    def sp(params):
        return SamplingParams(temperature=0.0, max_tokens=a.max_tokens, detokenize=False,
                              extra_args={"kv_transfer_params": params})

    def save_params(key: str, ids: list[int]) -> dict:
        blocks = len(ids) // block if a.restore_blocks <= 0 else min(a.restore_blocks, len(ids) // block)
        params = {"turbobus.do_save": a.save_enabled, "turbobus.prefix_key": key, "turbobus.save_blocks": blocks}
        if a.matched_tokens > 0:
            params["turbobus.matched_tokens"] = a.matched_tokens
        return params

    llm.generate([TokensPrompt(prompt_token_ids=prompts["first"])], sp(save_params(a.prefix_key, prompts["first"])),
                 use_tqdm=False)
    restore_key = a.prefix_key
    if a.second_save_prefix_key:
        llm.generate([TokensPrompt(prompt_token_ids=prompts["second_save"])],
                     sp(save_params(a.second_save_prefix_key, prompts["second_save"])), use_tqdm=False)
        restore_key = a.second_save_prefix_key
    restore_params = {"turbobus.do_restore": True, "turbobus.prefix_key": restore_key}
    if a.matched_tokens > 0:
        restore_params["turbobus.matched_tokens"] = a.matched_tokens
    out_restore = llm.generate([TokensPrompt(prompt_token_ids=prompts["restore"])], sp(restore_params),
                               use_tqdm=False)
    out_plain = llm.generate([TokensPrompt(prompt_token_ids=prompts["restore"])], sp({}), use_tqdm=False)
    ev = get_connector_events()
    saves = [e for e in ev if e.get("event") == "save" and e.get("prefix_key", restore_key) == restore_key]
    restores = [e for e in ev if e.get("event") == "restore"]
    matches = [e for e in ev if e.get("event") == "match"]
    toks_r = list(out_restore[0].outputs[0].token_ids)
    toks_p = list(out_plain[0].outputs[0].token_ids)
    s = saves[-1] if saves else {}
    r = restores[-1] if restores else {}
    n = len(prompts["second_save" if a.second_save_prefix_key else "first"])
    layers = SHAPES[a.shape]["num_hidden_layers"] if a.model is None else int(s.get("layers", 0) or 0)
    summary = {"job_id": a.job_id, "session_id": a.session_id, "shape": a.shape if a.model is None else a.model,
               "prompt_tokens": n, "restore_prefix_key": restore_key,
               "matched_tokens": int(matches[-1]["available_tokens"]) if matches else 0,
               "save_blocks": int(s.get("block_count", 0)), "restore_blocks": int(r.get("block_count", 0)),
               "bytes": int(s.get("bytes", 0)), "bytes_completed": int(r.get("bytes", 0)),
               "save_ms": float(s.get("total_ms", 0.0) or 0.0), "save_cuda_ms": float(s.get("cuda_ms", 0.0) or 0.0),
               "restore_ms": float(r.get("transfer_ms", 0.0) or 0.0),
               "restore_cuda_ms": float(r.get("cuda_ms", 0.0) or 0.0), "data_path": a.data_path,
               "relay_gpus": a.relay_gpus, "direct_bytes": 0, "relay_bytes": 0,
               "save_layer_count": layers, "save_layer_ranges": 0,
               "restored_tokens": toks_r, "recomputed_tokens": toks_p,
               "restore_verified": (toks_r == toks_p) if a.restore_enabled else None,
               "engine_init_s": round(init_s, 1), "events": len(ev)}
    return {"config": vars(a), "summary": summary, "events": ev,
            "lines": summary_lines(a, summary, s, r)}


def main(argv=None) -> int:
    a = parse_args(argv)
    res = run(a)
    line = json.dumps(res["summary"])
    print("VLLM_KV_SUMMARY " + line, flush=True)
    for ln in res["lines"]:
        print(ln, flush=True)
    if a.json_output:
        Path(a.json_output).parent.mkdir(parents=True, exist_ok=True)
        out = {k: v for k, v in res.items() if k != "lines"}
        Path(a.json_output).write_text(json.dumps(out, indent=2, default=str) + "\n")
    if a.log_output:
        Path(a.log_output).parent.mkdir(parents=True, exist_ok=True)
        with Path(a.log_output).open("w", encoding="utf-8") as fh:
            for ev in res["events"]:
                fh.write("turbobus_kv_connector_event " + json.dumps(ev, default=str) + "\n")
            fh.write("\n".join(res["lines"]) + "\n")
    ok = res["summary"]["restore_verified"] is not False
    print(f"vllm_kv_connector status {'ok' if ok else 'failed'}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
