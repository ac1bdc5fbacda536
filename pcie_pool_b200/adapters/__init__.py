"""Framework adapters: inference KV slots, vLLM (block mapping, runtime hooks,
V1 KV connector), model-weight loading and training offload.  Public names as
turbobus/adapters/__init__.py; ``PagedKVOffloader`` is additional (paged-KV
save/restore as one fused engine transfer)."""

from ..offload_store import AdapterTransferContext, ReceiptTransferHandle
from .base import FrameworkAdapter
from .inference import (FrameworkKVSlot, FrameworkKVSlotAdapter, InferenceKVSlot, InferenceKVSlotAdapter,
                        make_contiguous_kv_slots)
from .kv_offload import KVTransferStats, PagedKVOffloader
from .model_loading import ModelLoader, ModelWeightLoader
from .streamed_optimizer import StepStats, StreamedAdamW
from .training_offload import TrainingOffloadManager, TrainingOffloadStore
from .vllm import (VllmKVBlockRef, VllmKVGroup, VllmKVSlotAdapter, block_bytes_from_vllm_kv_tensor,
                   block_table_units, make_vllm_block_refs_from_ids, make_vllm_layer_block_refs_from_ids,
                   make_vllm_layer_groups_from_kv_caches, make_vllm_layer_range_refs_from_ids, vllm_block_name)
from .vllm_integration import (VllmAllocationEvent, VllmIntegrationState, VllmTurboBusIntegration,
                               extract_vllm_block_ids)
from .vllm_kv_connector import (TurboBusConnector, TurboBusConnectorConfig, TurboBusConnectorMetadata,
                                TurboBusRequestMetadata, TurboBusSavedPrefix, clear_connector_events,
                                clear_saved_prefixes, get_connector_events, get_saved_prefix)

__all__ = [
    "AdapterTransferContext", "FrameworkAdapter", "FrameworkKVSlot", "FrameworkKVSlotAdapter", "InferenceKVSlot",
    "InferenceKVSlotAdapter", "KVTransferStats", "ModelLoader", "ModelWeightLoader", "PagedKVOffloader",
    "ReceiptTransferHandle", "TrainingOffloadManager", "TrainingOffloadStore", "TurboBusConnector",
    "TurboBusConnectorConfig", "TurboBusConnectorMetadata", "TurboBusRequestMetadata", "TurboBusSavedPrefix",
    "VllmAllocationEvent", "VllmIntegrationState", "VllmKVBlockRef", "VllmKVGroup", "VllmKVSlotAdapter",
    "StepStats", "StreamedAdamW", "VllmTurboBusIntegration", "block_bytes_from_vllm_kv_tensor", "block_table_units", "clear_connector_events",
    "clear_saved_prefixes", "extract_vllm_block_ids", "get_connector_events", "get_saved_prefix",
    "make_contiguous_kv_slots", "make_vllm_block_refs_from_ids", "make_vllm_layer_block_refs_from_ids",
    "make_vllm_layer_groups_from_kv_caches", "make_vllm_layer_range_refs_from_ids", "vllm_block_name",
]
