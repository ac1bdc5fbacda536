"""Entry point for vLLM-shaped integrations: map vLLM block ids of a
request onto per-layer byte ranges (``make_vllm_layer_range_refs_from_ids``)
and move them through ``VllmKVSlotAdapter``, or hand the whole block table to
``PagedKVOffloader`` (one pooled transfer per request)."""

from ..vllm import (VllmKVBlockRef, VllmKVGroup, VllmKVSlotAdapter, block_table_units,  # noqa: F401
                    kv_layout, make_vllm_layer_range_refs_from_ids)


if __name__ == "__main__":
    import torch

    kv = torch.zeros(2, 64, 16, 8, 128, dtype=torch.bfloat16)
    refs = make_vllm_layer_range_refs_from_ids("demo", [5, 6, 7, 40], [kv])
    for r in refs:
        print(r)
    print(kv_layout(kv))
