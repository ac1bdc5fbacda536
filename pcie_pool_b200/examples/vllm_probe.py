"""Probe the local vLLM install for what the KV connector relies on:
versions, GPUs, the V1 connector base class and its method signatures, and
whether this package's connector overrides every hook.  Prints one JSON
object.  ``python -m pcie_pool_b200.examples.vllm_probe``"""

from __future__ import annotations

import inspect
import json


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


def main() -> int:
    print(json.dumps(probe(), indent=2, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
