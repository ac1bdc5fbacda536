"""The fp8 quantizer's division-free estimate (csrc/fp8_e4m3.cuh) restated
on the host: its codes equal e4m3(fp32(x / scale)) for random blocks, for
quotients placed on e4m3 rounding midpoints, and at the range edges; the
exact division is taken only near boundaries."""

import numpy as np

from pcie_pool_b200.utils.fp8 import E4M3_MAX, _TABLE, e4m3_encode, e4m3_quotient_estimated


def _bf16(x):
    b = np.asarray(x, dtype=np.float32).view(np.uint32)
    b = (b + np.uint32(0x7FFF) + ((b >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return b.view(np.float32)


def _check(x):
    x = _bf16(x)
    amax = np.float32(np.max(np.abs(x)))
    s = np.float32(amax / np.float32(E4M3_MAX)) if amax > 0 else np.float32(1.0)
    want = e4m3_encode((x / s).astype(np.float32))
    got, exact = e4m3_quotient_estimated(x, s)
    assert np.array_equal(got, want), np.flatnonzero(got != want)[:10]
    return exact


def test_random_blocks_match_division():
    rng = np.random.default_rng(0)
    fallback = 0
    for k in range(200):
        scale = 10.0 ** rng.uniform(-30, 30)
        fallback += _check(rng.standard_normal(128 * 128) * scale).sum()
    assert fallback < 200 * 128 * 128 * 0.02  # the exact path stays rare


def test_quotients_on_rounding_midpoints():
    rng = np.random.default_rng(1)
    mids = (_TABLE[:-1] + _TABLE[1:]) / 2.0
    for k in (-20, -3, 0, 7, 40):
        s = np.float32(2.0 ** k)  # exact quotients: every midpoint is hit exactly
        x = np.concatenate([mids, -mids, [E4M3_MAX, -E4M3_MAX]]) * float(s)
        exact = _check(x)
        assert exact.any()
    for _ in range(50):  # near-midpoints under a non-power-of-two scale
        s = np.float32(rng.uniform(0.5, 2.0) * 2.0 ** rng.integers(-20, 20))
        x = np.concatenate([mids * float(s), [E4M3_MAX * float(s)]])
        _check(x * (1 + rng.uniform(-1e-6, 1e-6, x.size)))


def test_edges_zero_signs_and_tiny_blocks():
    _check(np.zeros(64))
    _check(np.array([-0.0, 0.0, 1.0, -1.0]))
    _check(np.array([1e-40, -3e-41, 2e-39]))  # subnormal bf16 inputs, subnormal scale
    _check(np.array([448.0, -448.0, 447.9, 1e-3]))
