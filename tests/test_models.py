"""Model shapes and synthetic-data generators (CPU)."""

import numpy as np
import torch

from pcie_pool_b200._native import native
from pcie_pool_b200.models.llama import decoder_7b, llama3_8b, weight_manifest


def test_llama3_8b_manifest_shape():
    m = weight_manifest(llama3_8b())
    assert m.param_count == 8_030_261_248 and m.total_bytes == 16_060_522_496
    assert len(m.matrices()) == 2 + 32 * 7 and len(m.vectors()) == 2 * 32 + 1
    assert all(t.shape[0] % 128 == 0 and t.shape[1] % 128 == 0 for t in m.matrices())
    assert all(t.offset % 4096 == 0 for t in m.tensors)
    names = m.by_name()
    assert names["model.layers.0.self_attn.k_proj.weight"].shape == (1024, 4096)
    assert names["model.layers.31.mlp.down_proj.weight"].shape == (4096, 14336)


def test_decoder_7b_param_count():
    assert weight_manifest(decoder_7b()).param_count == 6_738_415_616


def test_fill_normal_bf16_is_seeded_and_thread_invariant():
    C = native()
    a = np.empty(1 << 21, dtype=np.uint16)
    b = np.empty_like(a)
    C.fill_normal_bf16(a.ctypes.data, a.size, 0.0, 0.02, 5, 0)
    C.fill_normal_bf16(b.ctypes.data, b.size, 0.0, 0.02, 5, 3)
    assert np.array_equal(a, b)
    f = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).float()
    assert abs(float(f.mean())) < 1e-3 and abs(float(f.std()) - 0.02) < 1e-3
    C.fill_normal_bf16(b.ctypes.data, b.size, 0.0, 0.02, 6, 0)
    assert not np.array_equal(a, b)
