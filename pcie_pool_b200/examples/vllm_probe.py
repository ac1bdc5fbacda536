"""Probe vLLM for what the KV connector relies on.

    python -m pcie_pool_b200.examples.vllm_probe            # install probe (one JSON object)
    python -m pcie_pool_b200.examples.vllm_probe --run      # + observe a generation
    python -m pcie_pool_b200.examples.vllm_probe --model DIR --prompt "..."

The install probe reports versions, GPUs, the V1 connector base class and its
method signatures, and whether this package's connector overrides every hook.
``--run`` / ``--model`` also start an engine (a random-init model of the demo
shape unless ``--model`` names a local checkpoint) with wrappers on the
scheduler's KV-cache manager and the model runner, generate once and print
what vLLM does with KV memory: the cache config at initialisation (blocks,
tensors, groups, block size), the runner's cache attributes, the block ids
each request gets and the computed-prefix blocks it is matched to, between
``VLLM_PROBE_BEGIN`` / ``VLLM_PROBE_END`` (the lines the reference's
examples/vllm_probe.py prints).
"""

from __future__ import annotations

import argparse
import functools
import inspect
import json
import os
import time


def probe() -> dict:
    out: dict = {}
    try:
        import torch

        out["torch"] = torch.__version__
        out["cuda_devices"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
    except Exception as exc:  # noqa: BLE001 - reported
        out["torch_error"] = repr(exc)
    try:
        import vllm

        out["vllm"] = vllm.__version__
        from vllm.distributed.kv_transfer.kv_connector.v1 import base

        hooks = ["register_kv_caches", "get_num_new_matched_tokens", "update_state_after_alloc",
                 "build_connector_meta", "start_load_kv", "wait_for_layer_load", "save_kv_layer", "wait_for_save",
                 "get_finished", "request_finished"]
        out["base_signatures"] = {h: str(inspect.signature(getattr(base.KVConnectorBase_V1, h))) for h in hooks}
        from ..adapters.vllm_kv_connector import TurboBusConnector

        out["connector_overrides"] = {h: getattr(TurboBusConnector, h) is not getattr(base.KVConnectorBase_V1, h)
                                      for h in hooks}
        out["connector_is_subclass"] = issubclass(TurboBusConnector, base.KVConnectorBase_V1)
        try:
            from vllm.distributed.kv_transfer.kv_connector.v1.base import SupportsHMA

            out["supports_hma"] = issubclass(TurboBusConnector, SupportsHMA)
        except ImportError:
            out["supports_hma"] = None
    except Exception as exc:  # noqa: BLE001 - reported
        out["vllm_error"] = repr(exc)
    return out


def describe_value(value, depth: int = 0) -> str:
    """Short text form of a cache attribute: tensors by shape/dtype/device,
    containers by their first items."""
    if depth > 2:
        return type(value).__name__
    if isinstance(value, dict):
        return "dict{" + ",".join(f"{k}:{describe_value(v, depth + 1)}" for k, v in list(value.items())[:16]) + "}"
    if isinstance(value, (list, tuple)):
        return f"{type(value).__name__}[" + ",".join(describe_value(v, depth + 1) for v in list(value)[:8]) + "]"
    shape = getattr(value, "shape", None)
    if shape is not None:
        return f"tensor(shape={tuple(shape)},dtype={getattr(value, 'dtype', None)},device={getattr(value, 'device', None)})"
    return type(value).__name__


def describe_blocks(blocks) -> str:
    """Block ids of a ``KVCacheBlocks`` (or the object's type when it has none)."""
    if blocks is None:
        return "None"
    get_ids = getattr(blocks, "get_block_ids", None)
    if get_ids is None:
        return type(blocks).__name__
    try:
        return repr(get_ids(allow_none=True))
    except TypeError:
        return repr(get_ids())


def describe_cache_config(cfg) -> str:
    groups = getattr(cfg, "kv_cache_groups", []) or []
    parts = []
    for i, g in enumerate(groups):
        spec = getattr(g, "kv_cache_spec", None)
        parts.append(f"g{i}:layers={len(getattr(g, 'layer_names', []) or [])} "
                     f"block_size={getattr(spec, 'block_size', '?')} spec={type(spec).__name__}")
    return (f"num_blocks={getattr(cfg, 'num_blocks', '?')} tensor_count={len(getattr(cfg, 'kv_cache_tensors', []) or [])} "
            f"group_count={len(groups)} groups=[{';'.join(parts)}]")


def install_observers(emit=print) -> list:
    """Wrap the runner's cache initialisation and the cache manager's slot
    allocation / prefix lookup so each call reports what it produced.
    Returns (owner, name, original) triples for :func:`remove_observers`."""
    from vllm.v1.core import kv_cache_manager as km
    from vllm.v1.worker import gpu_model_runner as gm

    saved = []

    def wrap(owner, name, after):
        orig = getattr(owner, name)

        @functools.wraps(orig)
        def wrapped(self, *args, **kwargs):
            out = orig(self, *args, **kwargs)
            after(self, args, out)
            return out

        setattr(owner, name, wrapped)
        saved.append((owner, name, orig))

    def on_init(runner, args, _out):
        emit("probe_initialize_kv_cache " + describe_cache_config(args[0] if args else None))
        attrs = [f"{k}={describe_value(v)}" for k, v in vars(runner).items()
                 if "kv" in k.lower() or "cache" in k.lower()]
        if attrs:
            emit("probe_runner_attrs " + "|".join(attrs[:40]))

    def on_alloc(_mgr, args, out):
        emit(f"probe_allocate_slots request_id {getattr(args[0], 'request_id', '?') if args else '?'} "
             f"result {describe_blocks(out)}")

    def on_computed(_mgr, args, out):
        blocks, tokens = (out[0], out[1]) if isinstance(out, tuple) and len(out) > 1 else (out, "?")
        emit(f"probe_get_computed_blocks request_id {getattr(args[0], 'request_id', '?') if args else '?'} "
             f"computed_tokens {tokens} blocks {describe_blocks(blocks)}")

    wrap(gm.GPUModelRunner, "initialize_kv_cache", on_init)
    wrap(km.KVCacheManager, "allocate_slots", on_alloc)
    wrap(km.KVCacheManager, "get_computed_blocks", on_computed)
    return saved


def remove_observers(saved) -> None:
    for owner, name, orig in reversed(saved):
        setattr(owner, name, orig)


def run_generation(a) -> int:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # observers live in this process
    install_observers()
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    from .vllm_kv_connector import SHAPES, byte_token_ids, write_model_dir

    t0 = time.perf_counter()
    if a.model:
        llm = LLM(model=a.model, tensor_parallel_size=a.tensor_parallel_size,
                  gpu_memory_utilization=a.gpu_memory_utilization, enforce_eager=a.enforce_eager)
        prompt = a.prompt
    else:
        ids = byte_token_ids(a.prompt, SHAPES[a.shape]["vocab_size"])
        llm = LLM(model=write_model_dir(a.shape, len(ids) + a.max_tokens + 64), load_format="dummy",
                  skip_tokenizer_init=True, dtype="bfloat16", max_model_len=len(ids) + a.max_tokens + 64,
                  tensor_parallel_size=a.tensor_parallel_size, gpu_memory_utilization=a.gpu_memory_utilization,
                  enforce_eager=a.enforce_eager)
        prompt = TokensPrompt(prompt_token_ids=ids)
    init_ms = (time.perf_counter() - t0) * 1e3
    t0 = time.perf_counter()
    outs = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=a.max_tokens,
                                                 detokenize=bool(a.model)), use_tqdm=False)
    gen_ms = (time.perf_counter() - t0) * 1e3
    print("VLLM_PROBE_BEGIN")
    print("llm_init_ms", f"{init_ms:.3f}")
    print("generate_ms", f"{gen_ms:.3f}")
    for o in outs:
        c = o.outputs[0] if o.outputs else None
        text = (c.text or "") if c is not None and a.model else ",".join(str(t) for t in (c.token_ids if c else []))
        print("output request_id", getattr(o, "request_id", "?"), "prompt_tokens",
              len(getattr(o, "prompt_token_ids", []) or []), "generated", repr(text[:200]))
    print("VLLM_PROBE_END", flush=True)
    return 0


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--run", action="store_true", help="also observe one generation")
    p.add_argument("--model", default=None, help="local checkpoint (implies --run)")
    p.add_argument("--shape", default="tiny", help="random-init model shape when --model is not given")
    p.add_argument("--prompt", default="The capital of France is")
    p.add_argument("--max-tokens", type=int, default=8)
    p.add_argument("--tensor-parallel-size", type=int, default=1)
    p.add_argument("--gpu-memory-utilization", type=float, default=0.5)
    p.add_argument("--enforce-eager", action="store_true")
    return p.parse_args(argv)


def main(argv=None) -> int:
    a = parse_args(argv)
    print(json.dumps(probe(), indent=2, sort_keys=True))
    if a.run or a.model:
        return run_generation(a)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
