"""Philox4x32-10 counter-based generator, restated in numpy (oracle; test infrastructure only).

The algorithm is the published Philox4x32 of Salmon, Moraes, Dror and Shaw,
"Parallel random numbers: as easy as 1, 2, 3" (SC'11): ten rounds of two
32x32->64 multiplies by 0xD2511F53 / 0xCD9E8D57, with the key bumped by the
Weyl constants 0x9E3779B9 / 0xBB67AE85 after every round.  Triton's
``tl.rand`` (triton 3.6.0, ``triton/language/random.py``) is this generator with
counter ``(offset, 0, 0, 0)`` and key ``(seed_lo, seed_hi)``; the reference's
optimizer kernels draw from it (``ecoint8/triton_kernels.py:87,113,116``).

``sr_word`` / ``sr_nudge`` define the stochastic-rounding stream of the CUDA
library (its Philox mode); the CUDA device code implements the same function.
"""

from __future__ import annotations

import numpy as np

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = 0x9E3779B9
W1 = 0xBB67AE85
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32(c0, c1, c2, c3, k0: int, k1: int, rounds: int = 10):
    """Vectorised Philox4x32-R.  Counters are arrays of uint32 values; key is two ints."""
    c0 = np.asarray(c0, dtype=np.uint64) & MASK32
    c1 = np.asarray(c1, dtype=np.uint64) & MASK32
    c2 = np.asarray(c2, dtype=np.uint64) & MASK32
    c3 = np.asarray(c3, dtype=np.uint64) & MASK32
    c0, c1, c2, c3 = np.broadcast_arrays(c0, c1, c2, c3)
    k0 &= 0xFFFFFFFF
    k1 &= 0xFFFFFFFF
    for _ in range(rounds):
        p0 = M0 * c0  # < 2**64, exact in uint64
        p1 = M1 * c2
        n0 = (p1 >> np.uint64(32)) ^ c1 ^ np.uint64(k0)
        n2 = (p0 >> np.uint64(32)) ^ c3 ^ np.uint64(k1)
        c1 = p1 & MASK32
        c3 = p0 & MASK32
        c0, c2 = n0, n2
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return c0, c1, c2, c3


def _words(seed: int, stream: int, rows: np.ndarray, cols: np.ndarray, per: int):
    """Philox outputs for (row, col) with ``per`` columns per call (2: 64-bit, 4: 32-bit words)."""
    rows = np.asarray(rows, dtype=np.uint64)
    cols = np.asarray(cols, dtype=np.uint64)
    rows, cols = np.broadcast_arrays(rows, cols)
    shift = np.uint64(1 if per == 2 else 2)
    x = philox4x32(cols >> shift, rows, stream & 0xFFFFFFFF, (stream >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF,
                   (seed >> 32) & 0xFFFFFFFF)
    return cols, x


def _full_width(rows, cols):
    """``(row column vector, n)`` when ``cols`` is the row vector ``0 .. n-1`` (a whole-width
    block, where one Philox call per counter serves all its columns), else None."""
    r = np.asarray(rows)
    c = np.asarray(cols)
    if c.ndim == 2 and c.shape[0] == 1 and r.ndim == 2 and r.shape[1] == 1 and c.shape[1] > 0:
        n = c.shape[1]
        if c[0, 0] == 0 and c[0, -1] == n - 1 and np.array_equal(c[0], np.arange(n, dtype=c.dtype)):
            return r.astype(np.uint64), n
    return None


def _interleave(words, n):
    """Words ``[rows, calls]`` each -> ``[rows, len(words) * calls]``, call-major, cut to ``n`` columns."""
    out = np.stack(words, axis=-1)
    return out.reshape(out.shape[0], -1)[:, :n]


def _blocks(r, calls: int, n: int, fn):
    """``fn(row block, call indices)`` -> its ``[block rows, n]`` words, over blocks of about
    256 K calls (numpy temporaries that stay in cache)."""
    out = np.empty((r.shape[0], n), dtype=np.uint64)
    idx = np.arange(calls, dtype=np.uint64)[None, :]
    step = max(1, (1 << 18) // max(calls, 1))
    for i in range(0, r.shape[0], step):
        out[i:i + step] = fn(r[i:i + step], idx)
    return out


def sr_word(seed: int, stream: int, rows: np.ndarray, cols: np.ndarray) -> np.ndarray:
    """64 random bits for element ``(row, col)`` of site ``stream`` (uint64).

    Counter ``(col >> 1, row, stream_lo, stream_hi)``, key ``(seed_lo, seed_hi)``;
    an even column takes words ``(x1:x0)``, an odd column ``(x3:x2)``.
    """
    fw = _full_width(rows, cols)
    if fw is not None:  # one call per column pair
        r, n = fw

        def words(rb, pairs):
            x0, x1, x2, x3 = philox4x32(pairs, rb, stream & 0xFFFFFFFF, (stream >> 32) & 0xFFFFFFFF,
                                        seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
            return _interleave([(x1 << np.uint64(32)) | x0, (x3 << np.uint64(32)) | x2], n)

        return _blocks(r, (n + 1) // 2, n, words)
    cols, (x0, x1, x2, x3) = _words(seed, stream, rows, cols, 2)
    lo = np.where((cols & np.uint64(1)) == 0, x0, x2)
    hi = np.where((cols & np.uint64(1)) == 0, x1, x3)
    return (hi << np.uint64(32)) | lo


def sr_field(seed: int, stream: int, rows: np.ndarray, cols: np.ndarray) -> np.ndarray:
    """32 random bits for element ``(row, col)``: word ``col & 3`` of counter ``(col >> 2, row, stream)``."""
    fw = _full_width(rows, cols)
    if fw is not None:  # one call per column quad
        r, n = fw

        def words(rb, quads):
            return _interleave(list(philox4x32(quads, rb, stream & 0xFFFFFFFF, (stream >> 32) & 0xFFFFFFFF,
                                               seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)), n)

        return _blocks(r, (n + 3) // 4, n, words)
    cols, (x0, x1, x2, x3) = _words(seed, stream, rows, cols, 4)
    k = cols & np.uint64(3)
    return np.select([k == 0, k == 1, k == 2], [x0, x1, x2], x3).astype(np.uint64)


def low_bits(word: np.ndarray, nbits: int) -> np.ndarray:
    """``word mod 2**nbits`` as int64 (0 <= nbits <= 63)."""
    if nbits <= 0:
        return np.zeros(np.shape(word), dtype=np.int64)
    return (np.asarray(word, dtype=np.uint64) & np.uint64((1 << nbits) - 1)).astype(np.int64)


STREAM_ALT = 1 << 63  # the tie-break stream of a site is its stream id with the top bit set


def sr_nudge(seed: int, stream: int, shape, shift: int, row_base: int = 0) -> np.ndarray:
    """``U[0, 2**shift)`` nudges of a requant site, ``[rows, cols]`` (rows offset by ``row_base``).

    The top bits are the element's 32-bit field; for ``shift > 32`` the low
    ``shift - 32`` bits come from the field of the tie-break stream.  The CUDA
    kernels draw the tie-break field only when the rounding depends on it
    (probability 2**-32), which gives the same result.
    """
    rows, cols = (shape if len(shape) == 2 else (int(np.prod(shape[:-1])), shape[-1]))
    r = np.arange(rows, dtype=np.uint64)[:, None] + np.uint64(row_base)
    c = np.arange(cols, dtype=np.uint64)[None, :]
    f = sr_field(seed, stream, r, c)
    if shift <= 32:
        u = low_bits(f, shift)
    else:
        lo = shift - 32
        t = low_bits(sr_field(seed, stream | STREAM_ALT, r, c), lo)
        u = ((f.astype(np.int64) << np.int64(lo)) | t)
    return u.reshape(shape)


def step_nudges(seed: int, stream: int, rows: int, cols: int, com_mm: int):
    """Weight (12-bit) and momentum (``com_mm``-bit) nudges of one I8ECO layer step.

    One 32-bit field per element: the weight nudge is its low 12 bits and the
    momentum nudge's top bits are its high 20 bits; for ``com_mm > 20`` the low
    ``com_mm - 20`` bits come from the 64-bit word of the tie-break stream
    (drawn by the kernel only when the rounding depends on them).
    """
    r = np.arange(rows, dtype=np.uint64)[:, None]
    c = np.arange(cols, dtype=np.uint64)[None, :]
    f = sr_field(seed, stream, r, c)
    nw = low_bits(f, 12)
    mf = (f >> np.uint64(12)).astype(np.uint64)
    if com_mm < 0:
        nm = None
    elif com_mm <= 20:
        nm = low_bits(mf, com_mm)
    else:
        lo = com_mm - 20
        t = low_bits(sr_word(seed, stream | STREAM_ALT, r, c), lo)
        nm = (mf.astype(np.int64) << np.int64(lo)) | t
    return nw, nm


def tl_rand(seed: int, offsets: np.ndarray) -> np.ndarray:
    """``tl.rand(seed, offsets)`` for int32 offsets: uniform fp32 in [0, 1).

    Counter ``(offset, 0, 0, 0)``; the first output word, viewed as int32 and
    folded (``x < 0 -> -x - 1``), times fp32 4.6566127342e-10.
    """
    off = np.asarray(offsets, dtype=np.int64).astype(np.uint64) & MASK32
    x0, _, _, _ = philox4x32(off, 0, 0, 0, seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    xi = x0.astype(np.uint32).view(np.int32).astype(np.int64)
    xi = np.where(xi < 0, -xi - 1, xi).astype(np.int32)
    return (xi.astype(np.float32) * np.float32(4.6566127342e-10)).astype(np.float32)
