"""Host oracle for fp8 e4m3 block quantisation, written from the OCP FP8
specification (E4M3: 1 sign, 4 exponent bits with bias 7, 3 mantissa bits,
no infinities, NaN = S.1111.111, largest finite 448, smallest subnormal 2**-9).

Rounding: round to nearest, ties to the even code; finite values above 448
saturate to +-448 ("satfinite"); NaN stays NaN; the sign of zero is kept.

Block quantisation contract (same as the device kernels): for every 128x128
block of a row-major matrix, ``scale = amax / 448`` in fp32 (1.0 when the block
is all zero) and ``q = e4m3(x / scale)`` with an IEEE fp32 division.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def _e4m3_table() -> np.ndarray:
    """Values of codes 0x00..0x7E (non-negative finite), increasing."""
    vals = np.zeros(127, dtype=np.float64)
    for code in range(127):
        e = code >> 3
        m = code & 7
        vals[code] = (m / 8.0) * 2.0 ** -6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


_TABLE = _e4m3_table()


def e4m3_encode(x) -> np.ndarray:
    """fp32/fp64 array -> uint8 e4m3 codes (RNE, satfinite)."""
    x = np.asarray(x, dtype=np.float64)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.abs(x)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, a)
    # index of the largest table value <= a
    k = np.searchsorted(_TABLE, a, side="right") - 1
    k = np.clip(k, 0, 126)
    lo = _TABLE[k]
    hi = _TABLE[np.minimum(k + 1, 126)]
    mid = (lo + hi) / 2.0
    up = (a > mid) | ((a == mid) & ((k & 1) == 1))
    code = np.where((k < 126) & up, k + 1, k)
    code = np.where(a >= E4M3_MAX, 126, code).astype(np.uint8)
    code = np.where(nan, 0x7F, code).astype(np.uint8)
    return code | sign


def e4m3_decode(code) -> np.ndarray:
    code = np.asarray(code, dtype=np.uint8)
    mag = code & 0x7F
    v = np.where(mag == 0x7F, np.nan, _TABLE[np.minimum(mag, 126)])
    return np.where(code & 0x80, -v, v)


def block_quant(x: np.ndarray, block: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """Quantise a 2-D fp32 array (values exactly representable in bf16 or any
    fp32) into (e4m3 codes [R, C], fp32 scales [ceil(R/128), ceil(C/128)])."""
    x = np.asarray(x, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError("block_quant expects a 2-D array")
    R, C = x.shape
    nrb, ncb = (R + block - 1) // block, (C + block - 1) // block
    q = np.zeros((R, C), dtype=np.uint8)
    scales = np.zeros((nrb, ncb), dtype=np.float32)
    for rb in range(nrb):
        for cb in range(ncb):
            blk = x[rb * block:(rb + 1) * block, cb * block:(cb + 1) * block]
            amax = np.float32(np.max(np.abs(blk))) if blk.size else np.float32(0)
            scale = np.float32(amax / np.float32(E4M3_MAX)) if amax > 0 else np.float32(1.0)
            scales[rb, cb] = scale
            q[rb * block:(rb + 1) * block, cb * block:(cb + 1) * block] = e4m3_encode(
                (blk / scale).astype(np.float32))
    return q, scales


def block_dequant(q: np.ndarray, scales: np.ndarray, block: int = 128) -> np.ndarray:
    R, C = q.shape
    s = np.repeat(np.repeat(scales, block, axis=0), block, axis=1)[:R, :C]
    return (e4m3_decode(q) * s).astype(np.float32)


def e4m3_quotient_estimated(x, scale) -> tuple[np.ndarray, np.ndarray]:
    """The device quantizer's method for ``e4m3(x / scale)``, restated on the
    host (csrc/fp8_e4m3.cuh): estimate q = x * fp32(1/scale), bracket |q| by
    the floats 8 steps below and above it, and divide exactly only where the
    bracket's ends convert to different codes.  Returns (codes, mask of the
    elements that took the exact division)."""
    x = np.asarray(x, dtype=np.float32)
    s = np.float32(scale)
    r = np.float32(1.0) / s
    with np.errstate(over="ignore", invalid="ignore"):
        q = (x * r).astype(np.float32)
    bits = q.view(np.uint32)
    a = bits & np.uint32(0x7FFFFFFF)
    lo = np.where(a > 8, a - np.uint32(8), np.uint32(0)).astype(np.uint32).view(np.float32)
    hi = (a + np.uint32(8)).astype(np.uint32).view(np.float32)
    clo, chi = e4m3_encode(lo), e4m3_encode(hi)
    exact = (clo != chi) | (not np.isfinite(r))
    mag = np.where(exact, e4m3_encode(np.abs(x) / s) & 0x7F, clo & 0x7F).astype(np.uint8)
    sign = ((bits >> 24) & 0x80).astype(np.uint8)
    return mag | sign, exact
