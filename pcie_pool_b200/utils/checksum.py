"""Chunk checksum oracle (host side, numpy).

Definition shared by every kernel of the package: the bytes of a chunk are
read as little-endian 32-bit words ``w_i`` (a final partial word is
zero-padded) and

    checksum = (sum_i w_i  mod 2**64,  sum_i (i + 1) * w_i  mod 2**64)

with ``i`` the word index inside the chunk.  The position weight makes the
value sensitive to swapped or misplaced words; both halves are plain sums, so
partial results of any split add up exactly.
"""

from __future__ import annotations

import numpy as np

_MASK = (1 << 64) - 1


def checksum_bytes(data) -> tuple[int, int]:
    """Checksum of a bytes-like object or a uint8 numpy array."""
    buf = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8) if not isinstance(
        data, np.ndarray
    ) else data.reshape(-1).view(np.uint8)
    n = buf.size
    pad = (-n) % 4
    if pad:
        buf = np.concatenate([buf, np.zeros(pad, dtype=np.uint8)])
    words = buf.view("<u4").astype(np.uint64)
    s = int(words.sum(dtype=np.uint64))
    # (i+1) * w_i summed mod 2**64: numpy uint64 arithmetic wraps modulo 2**64.
    idx = np.arange(1, words.size + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        w = int((idx * words).sum(dtype=np.uint64))
    return s & _MASK, w & _MASK


def combine(parts) -> tuple[int, int]:
    """Sum checksum pairs (mod 2**64)."""
    s = w = 0
    for a, b in parts:
        s = (s + int(a)) & _MASK
        w = (w + int(b)) & _MASK
    return s, w


def checksum_at(data, start_byte: int) -> tuple[int, int]:
    """Checksum of ``data`` as if it started at byte ``start_byte`` (multiple
    of 4) of a longer stream: the weight of word k becomes k + start/4 + 1."""
    if start_byte % 4:
        raise ValueError("start_byte must be a multiple of 4")
    s, w = checksum_bytes(data)
    shift = start_byte // 4
    return s, (w + shift * s) & _MASK


def rebase_chunk_sums(checksums, lanes):
    """Per-chunk checksums (chunk-local word index, in lane order) re-based
    onto the whole host buffer via each chunk's host offset, so that
    ``combine`` of the result equals the checksum of the full buffer when the
    chunks tile it.  ``lanes`` are the H2D lanes of the transfer (``src_off``
    is the host offset, a multiple of 4)."""
    out, i = [], 0
    for lane in lanes:
        for s in lane.src_off:
            a, w = int(checksums[i][0]), int(checksums[i][1])
            out.append((a, (w + (int(s) // 4) * a) & _MASK))
            i += 1
    return out
