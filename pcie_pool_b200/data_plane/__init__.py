"""Data-plane facade: backends, the persistent runtime and the engine."""

from ..backends.base import TransferBackend
from ..backends.cuda import CudaNativeBackend, default_cuda_backend
from ..parallel.engine import PoolEngine
from ..runtime_engine import PoolRuntime, RuntimeOptions

__all__ = ["CudaNativeBackend", "PoolEngine", "PoolRuntime", "RuntimeOptions", "TransferBackend",
           "default_cuda_backend"]
