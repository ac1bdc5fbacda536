"""Backends of the data plane."""

from .base import TransferBackend
from .cuda import CudaNativeBackend, default_cuda_backend

__all__ = ["CudaNativeBackend", "TransferBackend", "default_cuda_backend"]
