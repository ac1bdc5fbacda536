"""Fused landing ops through the daemon on real GPUs.

A vLLM-layout KV prefix is saved with the fused gather and restored into a
permuted block table with the fused scatter, and a small decoder lands as fp8
e4m3 + fp32 per-128x128 scales -- each as an intent to an in-process daemon
whose executor drives the native engine, so the relay lanes (every other
visible GPU, up to three) come from the daemon's leases.  Bytes are compared
exactly with the source, fp8 codes and scales bit-exactly with the OCP
oracle (utils/fp8.py), and the daemon must hold no lease or chunk quota
afterwards."""

import numpy as np
import pytest
import torch

from pcie_pool_b200 import TurboBusClient

pytestmark = pytest.mark.gpu


def _node(gpus: int):
    from pcie_pool_b200.e2e import build_inprocess_node, nominal_profile
    from pcie_pool_b200.parallel.engine import PoolEngine

    devs = list(range(gpus))
    eng = PoolEngine(devs, slot_bytes=4 << 20, slots=3, timeout_s=10.0)
    daemon, dc = build_inprocess_node(eng, devs, 0, nominal_profile(0, devs[1:]) if gpus > 1 else None)
    sid = dc.register_session(0, devs[1:], max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job("job", session_id=sid).ok
    return daemon, dc, sid, eng


def _no_leaks(dc, relays: bool):
    """Leases were taken (relay lanes ran) and every one was released."""
    d = dc.describe().payload
    quotas = d.get("relay_quotas") or {}
    assert all(int(q.get("active_chunks", 0)) == 0 for q in quotas.values()), quotas
    assert not d.get("reservations"), d.get("reservations")
    assert not (d.get("runtime_resource_state") or {}).get("active_paths")
    if relays:
        used = {int(p.get("relay_device", -1)) for m in (d.get("measured_transfers") or {}).values()
                for p in m.get("path_stats", ())}
        assert used - {-1}, "no transfer ran on a leased relay lane"


def test_kv_save_and_permuted_restore_through_daemon(need_gpu, gpu_count):
    from pcie_pool_b200.adapters.kv_offload import DaemonKVOffloader

    daemon, dc, sid, _ = _node(min(gpu_count, 4))
    g = torch.Generator(device="cuda").manual_seed(21)
    layers, blocks, nreq = 8, 512, 200
    kvs = [torch.randn(2, blocks, 16, 8, 128, device="cuda", dtype=torch.bfloat16, generator=g)
           for _ in range(layers)]
    ref = [kv.clone() for kv in kvs]
    off = DaemonKVOffloader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="job", kv_caches=kvs,
                            units_per_chunk=32)
    cpu = torch.Generator().manual_seed(22)
    src_ids = torch.randperm(blocks, generator=cpu)[:nreq].tolist()
    dst_ids = torch.randperm(blocks, generator=cpu)[:nreq].tolist()
    host = torch.zeros(off.prefix_bytes(nreq), dtype=torch.uint8, pin_memory=True)
    st = off.save(src_ids, host)
    assert st.bytes == host.numel()
    want = torch.cat([r[lane, src_ids].reshape(-1).view(torch.uint8).cpu() for r in ref for lane in range(2)])
    assert torch.equal(host, want)
    for kv in kvs:
        kv.zero_()
    torch.cuda.synchronize()
    rs = off.restore(dst_ids, host)
    torch.cuda.synchronize()
    for kv, r in zip(kvs, ref):
        assert torch.equal(kv[:, dst_ids], r[:, src_ids])
    if gpu_count > 1:
        assert len(rs.lanes) > 1, "the restore should use leased relay lanes"
    _no_leaks(dc, gpu_count > 1)


def test_fp8_load_through_daemon_bit_exact(need_gpu, gpu_count):
    from pcie_pool_b200._native import native
    from pcie_pool_b200.models.llama import DecoderConfig, weight_manifest
    from pcie_pool_b200.models.loader import DaemonWeightLoader
    from pcie_pool_b200.utils.fp8 import block_quant

    daemon, dc, sid, _ = _node(min(gpu_count, 4))
    cfg = DecoderConfig("tiny", layers=2, hidden=1024, intermediate=3584, heads=8, kv_heads=2, head_dim=128,
                        vocab=4224)
    m = weight_manifest(cfg)
    host = torch.empty(m.total_bytes, dtype=torch.uint8, pin_memory=True)
    native().fill_normal_bf16(host.data_ptr(), m.total_bytes // 2, 0.0, 0.02, 5, 0)
    ld = DaemonWeightLoader(TurboBusClient(daemon=dc), dc, session_id=sid, job_id="job", target=0,
                            chunk_bytes=4 << 20)
    out = ld.load_fp8(host, m)
    torch.cuda.synchronize()
    raw = host.numpy()
    for t in m.matrices():
        rows, cols = t.shape
        w = raw[t.offset:t.offset + t.nbytes].view(np.uint16).reshape(rows, cols)
        f = torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16).float().numpy()
        q, sc = block_quant(f)
        assert np.array_equal(out.tensors[t.name].cpu().numpy(), q), t.name
        assert np.array_equal(out.scales[t.name].cpu().numpy(), sc), t.name
    for t in m.vectors():
        got = out.tensors[t.name].contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
        assert np.array_equal(got, raw[t.offset:t.offset + t.nbytes].view(np.uint16)), t.name
    _no_leaks(dc, gpu_count > 1)
