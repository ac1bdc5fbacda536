"""ctypes binding of the allocation-free landing entry point
(``ppb_noalloc_land`` in csrc/noalloc.h): the landing kernel over a
device-resident source with all scratch in a static device array."""

from __future__ import annotations

import ctypes
import functools

import numpy as np

from .._native import native

OP_COPY = 0
OP_SCATTER_UNITS = 1


@functools.lru_cache(maxsize=1)
def library() -> ctypes.CDLL:
    lib = ctypes.CDLL(native().__file__)
    u64, u32, vp = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_void_p
    lib.ppb_noalloc_land.argtypes = [ctypes.c_int, ctypes.c_int, vp, u64, vp, u64, vp, u32, u64, u32,
                                     ctypes.c_int, u64, vp]
    lib.ppb_noalloc_land.restype = ctypes.c_int
    lib.ppb_noalloc_result.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), vp, u32, vp]
    lib.ppb_noalloc_result.restype = ctypes.c_int
    lib.ppb_noalloc_setup.argtypes = [ctypes.c_int]
    lib.ppb_noalloc_setup.restype = ctypes.c_int
    lib.ppb_noalloc_strerror.argtypes = [ctypes.c_int]
    lib.ppb_noalloc_strerror.restype = ctypes.c_char_p
    lib.ppb_noalloc_max_chunks.restype = u32
    lib.ppb_noalloc_scratch_bytes.restype = u64
    return lib


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(f"ppb_noalloc: {library().ppb_noalloc_strerror(rc).decode()} (code {rc})")


def setup(device: int) -> None:
    """One-time per-device setup; call before any stream capture."""
    _check(library().ppb_noalloc_setup(int(device)))


def _check_tensors(src, dst, unit_addrs) -> None:
    """The C entry point takes raw device addresses: reject what would make it
    read or write the wrong memory (host tensors, another device, strided
    views, a unit table that is not 64-bit)."""
    import torch

    named = [("src", src)] + ([("dst", dst)] if dst is not None else []) + \
        ([("unit_addrs", unit_addrs)] if unit_addrs is not None else [])
    for name, t in named:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (the unit table too: it is read on the device)")
        if t.device != src.device:
            raise ValueError(f"{name} is on {t.device}, src is on {src.device}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if unit_addrs is not None and unit_addrs.dtype not in (torch.int64, torch.uint64):
        raise ValueError("unit_addrs must be an int64 or uint64 tensor of device addresses")
    if dst is not None and unit_addrs is not None:
        raise ValueError("give dst (copy) or unit_addrs (scatter), not both")


def land(src, dst=None, *, chunk_bytes: int, ctas: int = 4, unit_addrs=None, unit_bytes: int = 0,
         checksum: bool = True, timeout_ns: int = 0, stream=None) -> None:
    """Queue a copy (``dst`` given) or a unit scatter (``unit_addrs`` given) on
    the current torch stream of ``src``'s device; asynchronous."""
    import torch

    _check_tensors(src, dst, unit_addrs)
    if unit_addrs is not None and unit_addrs.numel() * int(unit_bytes or 1) < src.numel() * src.element_size():
        raise ValueError("unit_addrs has fewer entries than src holds units")
    dev = src.device.index
    s = torch.cuda.current_stream(src.device) if stream is None else stream
    op = OP_COPY if unit_addrs is None else OP_SCATTER_UNITS
    nbytes = src.numel() * src.element_size()
    _check(library().ppb_noalloc_land(
        dev, op, src.data_ptr(), nbytes, 0 if dst is None else dst.data_ptr(),
        0 if dst is None else dst.numel() * dst.element_size(),
        None if unit_addrs is None else unit_addrs.data_ptr(), int(unit_bytes), int(chunk_bytes), int(ctas),
        1 if checksum else 0, int(timeout_ns), ctypes.c_void_p(s.cuda_stream)))


def result(device: int, chunks: int, stream=None) -> tuple[list[int], np.ndarray]:
    """Synchronise the stream; (status words, per-chunk checksums [chunks, 2])."""
    import torch

    s = torch.cuda.current_stream(device) if stream is None else stream
    status = (ctypes.c_int * 4)()
    csum = np.zeros((int(chunks), 2), dtype=np.uint64)
    _check(library().ppb_noalloc_result(int(device), status, csum.ctypes.data, int(chunks),
                                        ctypes.c_void_p(s.cuda_stream)))
    return list(status), csum


__all__ = ["OP_COPY", "OP_SCATTER_UNITS", "land", "library", "result", "setup"]
