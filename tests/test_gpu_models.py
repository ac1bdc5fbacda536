"""Pooled weight loading on a GPU: a small decoder manifest lands bf16
(byte-exact) and fp8 e4m3 + fp32 128x128 scales (bit-exact against the CPU
oracle built from the OCP FP8 spec), norms as bf16."""

import numpy as np
import pytest
import torch

from pcie_pool_b200.models.llama import DecoderConfig, weight_manifest

pytestmark = pytest.mark.gpu


def _setup(seed=3):
    from pcie_pool_b200._native import native
    from pcie_pool_b200.utils.host_memory import PinnedHostBuffer

    cfg = DecoderConfig("tiny", layers=2, hidden=1024, intermediate=3584, heads=8, kv_heads=2, head_dim=128,
                        vocab=4224)
    m = weight_manifest(cfg)
    host = PinnedHostBuffer(m.total_bytes, fill=None)
    native().fill_normal_bf16(host.ptr, m.total_bytes // 2, 0.0, 0.02, seed, 0)
    return m, host


def _engine(devices=(0,)):
    from pcie_pool_b200.parallel.engine import PoolEngine

    return PoolEngine(list(devices), slot_bytes=4 << 20, slots=3, timeout_s=10.0)


def test_bf16_load_exact(need_gpu):
    from pcie_pool_b200.models.loader import PooledWeightLoader

    m, host = _setup()
    try:
        ld = PooledWeightLoader(_engine(), 0, chunk_bytes=4 << 20)
        out = ld.load_bf16(host.ptr, m.total_bytes, m)
        raw = host.numpy()
        for t in m.tensors:
            got = out.tensors[t.name].view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
            assert np.array_equal(got, raw[t.offset:t.offset + t.nbytes].view(np.uint16)), t.name
        assert out.stats.bytes == m.total_bytes and out.stats.cuda_ms > 0
    finally:
        host.release()


def test_fp8_load_bit_exact(need_gpu):
    from pcie_pool_b200.models.loader import PooledWeightLoader
    from pcie_pool_b200.utils.fp8 import block_quant

    m, host = _setup(seed=11)
    try:
        ld = PooledWeightLoader(_engine(), 0, chunk_bytes=4 << 20)
        out = ld.load_fp8(host.ptr, m.total_bytes, m)
        raw = host.numpy()
        for t in m.matrices():
            rows, cols = t.shape
            w = raw[t.offset:t.offset + t.nbytes].view(np.uint16).reshape(rows, cols)
            f = torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16).float().numpy()
            q_ref, s_ref = block_quant(f)
            assert np.array_equal(out.scales[t.name].cpu().numpy(), s_ref), t.name
            assert np.array_equal(out.tensors[t.name].cpu().numpy(), q_ref), t.name
        for t in m.vectors():
            got = out.tensors[t.name].view(torch.int16).cpu().numpy().view(np.uint16)
            assert np.array_equal(got, raw[t.offset:t.offset + t.nbytes].view(np.uint16))
        assert out.stats.transfers == 2
    finally:
        host.release()


@pytest.mark.multigpu
def test_fp8_load_over_relays(need_two_gpus):
    from pcie_pool_b200.models.loader import PooledWeightLoader
    from pcie_pool_b200.utils.fp8 import block_quant

    m, host = _setup(seed=12)
    try:
        n = torch.cuda.device_count()
        ld = PooledWeightLoader(_engine(range(n)), 0, list(range(1, n)), chunk_bytes=4 << 20)
        out = ld.load_fp8(host.ptr, m.total_bytes, m)
        assert len({d for d, _b, _ms in out.stats.lanes}) == n
        t = m.matrices()[3]
        rows, cols = t.shape
        w = host.numpy()[t.offset:t.offset + t.nbytes].view(np.uint16).reshape(rows, cols)
        q_ref, s_ref = block_quant(torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16).float().numpy())
        assert np.array_equal(out.tensors[t.name].cpu().numpy(), q_ref)
        assert np.array_equal(out.scales[t.name].cpu().numpy(), s_ref)
    finally:
        host.release()
