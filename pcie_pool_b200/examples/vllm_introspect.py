"""Start a small vLLM engine (dummy weights, no tokenizer) with the pooled
connector and report what vLLM hands the connector: the KV cache tensors
(names, shapes, strides, dtype, the layout ``kv_layout`` infers) and the
block-id structure of one request.  ``python -m
pcie_pool_b200.examples.vllm_introspect``"""

from __future__ import annotations

import json
import os


def main() -> int:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    from vllm import LLM, SamplingParams
    from vllm.config import KVTransferConfig
    from vllm.inputs import TokensPrompt

    from ..adapters import vllm_kv_connector as K
    from ..adapters.vllm import kv_layout
    from .vllm_kv_connector import write_model_dir

    seen: dict = {}
    orig = K.TurboBusConnector.register_kv_caches

    def spy(self, kv_caches):
        seen["layers"] = [{"name": n, "shape": list(t.shape), "stride": list(t.stride()), "dtype": str(t.dtype),
                           "layout": kv_layout(t).__dict__} for n, t in list(kv_caches.items())[:2]]
        seen["layer_count"] = len(kv_caches)
        return orig(self, kv_caches)

    K.TurboBusConnector.register_kv_caches = spy
    llm = LLM(model=write_model_dir("tiny", 1024), load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
              enable_prefix_caching=False, max_model_len=1024, gpu_memory_utilization=0.3,
              kv_transfer_config=KVTransferConfig(kv_connector="TurboBusConnector", kv_role="kv_both",
                                                  kv_connector_module_path="pcie_pool_b200.vllm_kv_connector"))
    llm.generate([TokensPrompt(prompt_token_ids=list(range(100, 164)))],
                 SamplingParams(max_tokens=2, detokenize=False), use_tqdm=False)
    allocs = [e for e in K.get_connector_events() if e.get("event") in ("register_kv_caches",)]
    seen["events"] = allocs
    print(json.dumps(seen, indent=2, default=str))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
