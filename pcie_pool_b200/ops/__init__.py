"""Torch-facing wrappers of the device-local sm_100a kernels.

All functions run on the tensor's device and the current torch stream.  They
call the native core directly (no fallback): on a machine without the built
extension they raise.
"""

from __future__ import annotations

import numpy as np

from .._native import native


def _torch():
    import torch

    return torch


def _stream(t) -> int:
    torch = _torch()
    return torch.cuda.current_stream(t.device).cuda_stream


def fp8_block_quant(x):
    """bf16 [R, C] (CUDA) -> (e4m3 codes uint8 [R, C], fp32 scales [ceil(R/128), ceil(C/128)])."""
    torch = _torch()
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_cuda:
        raise ValueError("fp8_block_quant expects a 2-D bf16 CUDA tensor")
    x = x.contiguous()
    R, Cc = x.shape
    q = torch.empty((R, Cc), dtype=torch.uint8, device=x.device)
    s = torch.empty(((R + 127) // 128, (Cc + 127) // 128), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        native().fp8_block_quant(x.data_ptr(), R, Cc, q.data_ptr(), s.data_ptr(), _stream(x))
    return q, s


def fp8_block_dequant(q, scales):
    torch = _torch()
    R, Cc = q.shape
    out = torch.empty((R, Cc), dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        native().fp8_block_dequant(q.contiguous().data_ptr(), scales.contiguous().data_ptr(), R, Cc,
                                   out.data_ptr(), _stream(q))
    return out


def unit_addresses(base_tensor, unit_bytes: int, unit_index) -> "torch.Tensor":
    """Device uint64 tensor of ``base + unit_index * unit_bytes``."""
    torch = _torch()
    idx = torch.as_tensor(np.asarray(unit_index, dtype=np.int64), device=base_tensor.device)
    return (idx * int(unit_bytes) + int(base_tensor.data_ptr())).to(torch.int64)


def gather_units(addrs, unit_bytes: int, out):
    """out[u*unit:(u+1)*unit] = bytes at addrs[u] (addrs: int64 CUDA tensor)."""
    torch = _torch()
    with torch.cuda.device(out.device):
        native().gather_units(addrs.data_ptr(), addrs.numel(), int(unit_bytes), out.data_ptr(),
                              _stream(out))
    return out


def scatter_units(src, addrs, unit_bytes: int):
    torch = _torch()
    with torch.cuda.device(src.device):
        native().scatter_units(src.data_ptr(), addrs.data_ptr(), addrs.numel(), int(unit_bytes),
                               _stream(src))


def paged_kv_gather(kv, block_ids, out=None):
    """Gather K/V blocks of one vLLM layer cache ``[2, num_blocks, ...]`` into a
    contiguous buffer laid out [K blocks in order, V blocks in order]."""
    torch = _torch()
    blk = kv.stride(1) * kv.element_size()
    lane = kv.stride(0) * kv.element_size()
    ids = np.asarray(block_ids, dtype=np.int64)
    offs = np.concatenate([ids * blk, lane + ids * blk])
    addrs = torch.as_tensor(offs + kv.data_ptr(), device=kv.device)
    if out is None:
        out = torch.empty(offs.size * blk, dtype=torch.uint8, device=kv.device)
    gather_units(addrs, blk, out)
    return out


def paged_kv_scatter(kv, block_ids, src):
    torch = _torch()
    blk = kv.stride(1) * kv.element_size()
    lane = kv.stride(0) * kv.element_size()
    ids = np.asarray(block_ids, dtype=np.int64)
    offs = np.concatenate([ids * blk, lane + ids * blk])
    addrs = torch.as_tensor(offs + kv.data_ptr(), device=kv.device)
    scatter_units(src, addrs, blk)


def pack_ranges(addrs, sizes, out):
    """Pack variable ranges (device addresses + sizes, int64 CUDA tensors) into ``out``."""
    torch = _torch()
    pos = torch.cumsum(sizes, 0) - sizes
    with torch.cuda.device(out.device):
        native().pack_ranges(addrs.data_ptr(), sizes.data_ptr(), pos.data_ptr(), addrs.numel(),
                             out.data_ptr(), _stream(out))
    return out


def unpack_ranges(src, addrs, sizes):
    torch = _torch()
    pos = torch.cumsum(sizes, 0) - sizes
    with torch.cuda.device(src.device):
        native().unpack_ranges(src.data_ptr(), addrs.data_ptr(), sizes.data_ptr(), pos.data_ptr(),
                               addrs.numel(), _stream(src))


def fused_adamw(master, exp_avg, exp_avg_sq, grad_bf16, param_bf16=None, *, lr=1e-3,
                betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, step=1, grad_scale=1.0):
    """In-place AdamW over fp32 master/moments with a bf16 gradient; writes the
    updated parameters as bf16 into ``param_bf16`` when given."""
    torch = _torch()
    for t in (master, exp_avg, exp_avg_sq):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("master and moments must be contiguous fp32")
    if grad_bf16.dtype != torch.bfloat16:
        raise ValueError("gradient must be bf16")
    C = native()
    p = C.AdamParams()
    p.lr, p.beta1, p.beta2, p.eps = float(lr), float(betas[0]), float(betas[1]), float(eps)
    p.weight_decay, p.step, p.grad_scale = float(weight_decay), int(step), float(grad_scale)
    with torch.cuda.device(master.device):
        C.fused_adamw(master.data_ptr(), exp_avg.data_ptr(), exp_avg_sq.data_ptr(),
                      grad_bf16.contiguous().data_ptr(),
                      0 if param_bf16 is None else param_bf16.data_ptr(), master.numel(), p,
                      _stream(master))


def interference(buf, iters: int = 64, ctas: int = 0):
    """SM/HBM load generator over an fp32 CUDA tensor (ctas 0 = one per SM)."""
    torch = _torch()
    with torch.cuda.device(buf.device):
        native().interference(buf.data_ptr(), buf.numel(), int(iters), int(ctas), _stream(buf))


def checksum(t) -> tuple[int, int]:
    """Chunk checksum of a tensor's bytes (device or host)."""
    torch = _torch()
    nbytes = t.numel() * t.element_size()
    if t.is_cuda:
        out = torch.zeros(2, dtype=torch.int64, device=t.device)
        with torch.cuda.device(t.device):
            native().checksum_device(t.data_ptr(), nbytes, out.data_ptr(), _stream(t))
        a, b = out.cpu().tolist()
        return a & (2**64 - 1), b & (2**64 - 1)
    return tuple(native().checksum_host(t.data_ptr(), nbytes))
