"""GPU tests of the device-local ops against host/PyTorch fp32 oracles."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("shape", [(256, 384), (200, 300), (1, 17), (129, 128)])
def test_fp8_block_quant_matches_oracle(need_gpu, shape):
    from pcie_pool_b200.ops import fp8_block_dequant, fp8_block_quant
    from pcie_pool_b200.utils.fp8 import block_dequant, block_quant

    x = (torch.randn(*shape, generator=torch.Generator().manual_seed(1)) * 3).to(torch.bfloat16)
    q, s = fp8_block_quant(x.cuda())
    q_ref, s_ref = block_quant(x.float().numpy())
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    deq = fp8_block_dequant(q, s).float().cpu().numpy()
    ref = block_dequant(q_ref, s_ref)
    np.testing.assert_allclose(deq, ref, rtol=1e-2, atol=1e-6)


def test_fp8_zero_block_scale_is_one(need_gpu):
    from pcie_pool_b200.ops import fp8_block_quant

    q, s = fp8_block_quant(torch.zeros(128, 256, dtype=torch.bfloat16, device="cuda"))
    assert torch.all(s == 1.0) and torch.all(q == 0)


def test_paged_kv_gather_scatter_roundtrip(need_gpu):
    from pcie_pool_b200.ops import paged_kv_gather, paged_kv_scatter

    kv = torch.randn(2, 40, 16, 8, 128, device="cuda").to(torch.bfloat16)
    ids = torch.randperm(40, generator=torch.Generator().manual_seed(2))[:13].numpy()
    flat = paged_kv_gather(kv, ids)
    ref = torch.cat([kv[0, ids].reshape(-1), kv[1, ids].reshape(-1)]).view(torch.uint8)
    assert torch.equal(flat, ref)
    kv2 = torch.zeros_like(kv)
    paged_kv_scatter(kv2, ids, flat)
    assert torch.equal(kv2[:, ids], kv[:, ids])


def test_pack_unpack_ranges(need_gpu):
    from pcie_pool_b200.ops import pack_ranges, unpack_ranges

    src = torch.randint(0, 256, (1 << 16,), dtype=torch.uint8, device="cuda")
    offs = torch.tensor([5, 1000, 4096, 30000, 65000], dtype=torch.int64)
    sizes = torch.tensor([7, 333, 4096, 100, 536], dtype=torch.int64)
    addrs = (offs + src.data_ptr()).cuda()
    out = torch.zeros(int(sizes.sum()), dtype=torch.uint8, device="cuda")
    pack_ranges(addrs, sizes.cuda(), out)
    ref = torch.cat([src[o:o + s] for o, s in zip(offs.tolist(), sizes.tolist())])
    assert torch.equal(out, ref)
    dst = torch.zeros_like(src)
    unpack_ranges(out, (offs + dst.data_ptr()).cuda(), sizes.cuda())
    for o, s in zip(offs.tolist(), sizes.tolist()):
        assert torch.equal(dst[o:o + s], src[o:o + s])


def test_fused_adamw_matches_torch(need_gpu):
    from pcie_pool_b200.ops import fused_adamw

    g = torch.Generator().manual_seed(3)
    n = 100_003
    p0 = torch.randn(n, generator=g)
    grads = [torch.randn(n, generator=g).to(torch.bfloat16) for _ in range(3)]
    ref = p0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    master = p0.clone().cuda()
    m = torch.zeros_like(master)
    v = torch.zeros_like(master)
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    for step, gr in enumerate(grads, 1):
        ref.grad = gr.float()
        opt.step()
        fused_adamw(master, m, v, gr.cuda(), out, lr=1e-2, betas=(0.9, 0.95), eps=1e-8,
                    weight_decay=0.1, step=step)
    torch.testing.assert_close(master.cpu(), ref.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(out.float().cpu(), ref.detach().to(torch.bfloat16).float(),
                               rtol=1e-2, atol=1e-2)


def test_checksum_device_matches_host(need_gpu):
    from pcie_pool_b200.ops import checksum
    from pcie_pool_b200.utils.checksum import checksum_bytes

    for n in (1, 3, 16, 4097, 1 << 20):
        t = torch.randint(0, 256, (n,), dtype=torch.uint8)
        assert checksum(t.cuda()) == checksum_bytes(t.numpy())
        assert checksum(t) == checksum_bytes(t.numpy())


def test_interference_runs(need_gpu):
    from pcie_pool_b200.ops import interference

    buf = torch.ones(1 << 20, device="cuda")
    interference(buf, iters=8, ctas=16)
    torch.cuda.synchronize()
    assert torch.isfinite(buf).all()
