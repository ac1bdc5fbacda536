"""Allocation-free C entry point ``ppb_noalloc_land`` (csrc/noalloc.h), called
through its exported symbol with ctypes and compared with the existing
PoolEngine path that runs the same landing kernel with allocated scratch.

Named to be collected last: it must pass alone and after every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from pcie_pool_b200._native import native

MiB = 1 << 20


def _lib():
    C = native()
    lib = ctypes.CDLL(C.__file__)
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


def test_noalloc_rejects_oversize_before_any_cuda_call():
    lib = _lib()
    assert lib.ppb_noalloc_max_chunks() == 4096
    assert lib.ppb_noalloc_scratch_bytes() == 256 * 1024
    # 4097 chunks of 1 byte: rejected by the argument checks (no device needed)
    rc = lib.ppb_noalloc_land(0, 0, 16, 4097, 16, 4097, None, 0, 1, 1, 1, 0, None)
    assert rc == -2
    assert b"4096 chunks" in lib.ppb_noalloc_strerror(rc)
    assert lib.ppb_noalloc_land(0, 0, 16, 1 << 20, 16, 1 << 20, None, 0, 1 << 32, 1, 1, 0, None) == -2
    assert lib.ppb_noalloc_land(0, 7, 16, 64, 16, 64, None, 0, 64, 1, 1, 0, None) == -1
    assert lib.ppb_noalloc_land(0, 1, 16, 96, None, 0, 16, 64, 64, 1, 1, 0, None) == -1  # 96 % 64


def test_noalloc_scatter_rejects_misalignment_before_any_cuda_call():
    """The scatter path moves units with 16-byte bulk copies: a unit size or a
    source that is not 16-byte aligned is an argument error, not a GPU fault."""
    lib = _lib()
    # unit_bytes = 8: whole units, but not a multiple of 16
    assert lib.ppb_noalloc_land(0, 1, 4096, 64, None, 0, 4096, 8, 64, 1, 1, 0, None) == -1
    # misaligned source (4104 % 16 == 8)
    assert lib.ppb_noalloc_land(0, 1, 4104, 64, None, 0, 4096, 16, 64, 1, 1, 0, None) == -1
    # misaligned unit table pointer
    assert lib.ppb_noalloc_land(0, 1, 4096, 64, None, 0, 4100, 16, 64, 1, 1, 0, None) == -1
    assert b"16-byte aligned" in lib.ppb_noalloc_strerror(-1)


def test_noalloc_python_binding_rejects_host_tensors():
    from pcie_pool_b200.ops import noalloc

    src = torch.zeros(64, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA tensor"):
        noalloc.land(src, torch.zeros(64, dtype=torch.uint8), chunk_bytes=64)
    with pytest.raises(TypeError):
        noalloc.land(np.zeros(64, np.uint8), chunk_bytes=64)


def _land(lib, op, src, dst, chunk, *, unit_addrs=None, unit_bytes=0, ctas=4):
    stream = torch.cuda.current_stream()
    rc = lib.ppb_noalloc_land(0, op, src.data_ptr(), src.numel(), 0 if dst is None else dst.data_ptr(),
                              0 if dst is None else dst.numel(),
                              None if unit_addrs is None else unit_addrs.data_ptr(), unit_bytes, chunk, ctas, 1,
                              0, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.ppb_noalloc_strerror(rc)
    n = -(-src.numel() // chunk)
    status = (ctypes.c_int * 4)()
    csum = np.zeros((n, 2), dtype=np.uint64)
    rc = lib.ppb_noalloc_result(0, status, csum.ctypes.data, n, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.ppb_noalloc_strerror(rc)
    assert list(status) == [0, 0, 0, 0]
    return csum


def _engine_land(op, host, dst_ptr, dst_bytes, chunk, unit_addrs=None, unit_bytes=0):
    from pcie_pool_b200.parallel.engine import H2D, PoolEngine, make_lane

    C = native()
    eng = PoolEngine([0], slot_bytes=chunk, slots=3, ctas_per_lane=4)
    n = host.numel()
    chunks = [(o, o, min(chunk, n - o)) for o in range(0, n, chunk)]
    kw = {}
    if unit_addrs is not None:
        units_per_chunk = chunk // unit_bytes
        kw = dict(unit0=np.arange(len(chunks), dtype=np.uint32) * units_per_chunk)
    lane = make_lane(0, chunks, **kw)
    # the engine runs on its own streams: what torch queued (zero fills,
    # uploads) must be done before it starts
    torch.cuda.synchronize()
    r = eng.run(H2D, 0, host.data_ptr(), n, dst_ptr, dst_bytes, [lane],
                op=C.OP_COPY if unit_addrs is None else C.OP_SCATTER_UNITS, checksum=True,
                stage_direct=True, unit_bytes=unit_bytes, unit_addrs=unit_addrs)
    r.raise_for_status()
    return np.asarray(r.checksums, dtype=np.uint64)


@pytest.mark.gpu
def test_noalloc_copy_matches_engine_twice(need_gpu):
    lib = _lib()
    assert lib.ppb_noalloc_setup(0) == 0
    nbytes, chunk = 24 * MiB + 4100, 4 * MiB  # ragged tail, misaligned tail length
    g = torch.Generator().manual_seed(3)
    host = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=g).pin_memory()
    ref = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    want = _engine_land(None, host, ref.data_ptr(), nbytes, chunk)
    torch.cuda.synchronize()
    src = host.cuda()
    assert torch.equal(ref, src)
    for _ in range(2):  # two calls in a row reuse the same static scratch
        dst = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        got = _land(lib, 0, src, dst, chunk)
        torch.cuda.synchronize()
        assert torch.equal(dst, src)
        assert torch.equal(dst, ref)
        np.testing.assert_array_equal(got, want)


@pytest.mark.gpu
def test_noalloc_scatter_units_matches_engine_twice(need_gpu):
    lib = _lib()
    unit, nunits, blocks = 16 * 1024, 512, 2048
    chunk = 64 * unit
    g = torch.Generator().manual_seed(5)
    host = torch.randint(0, 256, (nunits * unit,), dtype=torch.uint8, generator=g).pin_memory()
    perm = torch.randperm(blocks, generator=g)[:nunits]
    ref_pool = torch.zeros(blocks * unit, dtype=torch.uint8, device="cuda")
    addrs = (ref_pool.data_ptr() + perm.to(torch.int64) * unit).numpy().astype(np.uint64)
    want = _engine_land(1, host, ref_pool.data_ptr(), ref_pool.numel(), chunk, unit_addrs=addrs, unit_bytes=unit)
    torch.cuda.synchronize()
    src = host.cuda()
    expect = torch.zeros_like(ref_pool).view(blocks, unit)
    expect[perm.cuda()] = src.view(nunits, unit)
    assert torch.equal(ref_pool.view(blocks, unit), expect)
    for _ in range(2):
        pool = torch.zeros_like(ref_pool)
        table = (pool.data_ptr() + perm.to(torch.int64) * unit).cuda()  # addresses < 2^63: int64 bits
        got = _land(lib, 1, src, None, chunk, unit_addrs=table, unit_bytes=unit)
        torch.cuda.synchronize()
        assert torch.equal(pool.view(blocks, unit), expect)
        assert torch.equal(pool, ref_pool)
        np.testing.assert_array_equal(got, want)


@pytest.mark.gpu
def test_noalloc_bad_unit_address_reports_status_and_writes_nothing(need_gpu):
    """A unit table entry that is not 16-byte aligned is found on the device
    before any copy: the call reports status 3 (bad argument) with the unit
    index, lands nothing, and the next good call on the same scratch works."""
    lib = _lib()
    unit, nunits = 4096, 64
    src = torch.arange(nunits * unit, dtype=torch.int64, device="cuda").to(torch.uint8)
    pool = torch.zeros(nunits * unit, dtype=torch.uint8, device="cuda")
    table = pool.data_ptr() + torch.arange(nunits, dtype=torch.int64, device="cuda") * unit
    table[37] += 8  # misaligned entry
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    rc = lib.ppb_noalloc_land(0, 1, src.data_ptr(), src.numel(), None, 0, table.data_ptr(), unit, 16 * unit, 4, 1,
                              0, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0
    status = (ctypes.c_int * 4)()
    assert lib.ppb_noalloc_result(0, status, None, 0, ctypes.c_void_p(stream.cuda_stream)) == 0
    assert status[0] == 3 and status[3] == 37
    assert int(pool.count_nonzero()) == 0
    table[37] -= 8
    _land(lib, 1, src, None, 16 * unit, unit_addrs=table, unit_bytes=unit)
    torch.cuda.synchronize()
    assert torch.equal(pool, src)
