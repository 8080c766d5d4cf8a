"""Integer fixed-point core, restated in numpy (oracle; test infrastructure only).

Follows ``ecoint8/fixedpoint.py`` of the reference.  All tensor math is int64
with two's-complement wrap-around, exactly as PyTorch's int64 kernels behave:

* ``a * b`` wraps modulo 2**64;
* ``a << s`` is ``(uint64(a) << s)`` for ``0 <= s < 64`` and 0 for ``s >= 64``;
* ``a >> s`` is an arithmetic shift, and for ``s >= 64`` it equals ``a >> 63``;
* ``torch.div(p, 2**s, rounding_mode="floor")`` equals ``p >> s``.

Stochastic-rounding draws are explicit ``nudge`` arrays, so the caller decides
whether they replay the reference's ``torch.randint`` stream or come from the
Philox stream of the CUDA kernels (``oracle/philox.py``).
"""

from __future__ import annotations

import math

import numpy as np

INT8_LO, INT8_HI = -127, 127


def shl64(a: np.ndarray, s: int) -> np.ndarray:
    """Left shift with PyTorch int64 semantics (wraps; 0 when ``s >= 64``)."""
    a = np.asarray(a, dtype=np.int64)
    if s >= 64:
        return np.zeros_like(a)
    return (a.view(np.uint64) << np.uint64(s)).view(np.int64)


def sar64(a: np.ndarray, s: int) -> np.ndarray:
    """Arithmetic right shift with PyTorch int64 semantics (``s >= 64`` -> sign)."""
    a = np.asarray(a, dtype=np.int64)
    return a >> np.int64(min(s, 63))


def mul64(a, b) -> np.ndarray:
    """int64 product with wrap-around (PyTorch int64 ``*``)."""
    with np.errstate(over="ignore"):
        return (np.asarray(a, dtype=np.int64).view(np.uint64)
                * np.asarray(b, dtype=np.int64).view(np.uint64)).view(np.int64)


def add64(a, b) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (np.asarray(a, dtype=np.int64).view(np.uint64)
                + np.asarray(b, dtype=np.int64).view(np.uint64)).view(np.int64)


def sub64(a, b) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (np.asarray(a, dtype=np.int64).view(np.uint64)
                - np.asarray(b, dtype=np.int64).view(np.uint64)).view(np.int64)


def quantize_multiplier(r: float) -> tuple[int, int]:
    """``r -> (mult, shift)`` with ``mult`` in [2**30, 2**31).  fixedpoint.py:26-37."""
    assert r >= 0.0, "scale ratios must be non-negative"
    if r == 0.0:
        return 0, 0
    mantissa, exponent = math.frexp(r)
    shift = exponent
    mult = round(mantissa * (1 << 31))  # Python round: half to even
    if mult == (1 << 31):
        mult //= 2
        shift += 1
    return mult, 31 - shift


def pad_mm_dims(m: int, k: int, n: int) -> tuple[int, int, int]:
    """fixedpoint.py:91-102."""
    p8 = lambda v: (v + 7) // 8 * 8  # noqa: E731
    return max(32, p8(m)), p8(k), p8(n)


def dynamic_scale_from_int(acc_amax: int, real_gain: float) -> float:
    """fixedpoint.py:105-114."""
    real_amax = acc_amax * real_gain
    if real_amax <= 0.0:
        return 1.0
    return real_amax / 127.0


def sr_nudge_dtype(denom: int):
    """Dtype the reference draws a nudge in (fixedpoint.py:48)."""
    return np.int32 if denom <= (1 << 31) else np.int64


def apply_mult_shift(x, mult, shift: int, stochastic: bool = False, nudge=None) -> np.ndarray:
    """``floor((x*mult + nudge) / 2**shift)`` or ``(x*mult) << -shift``.  fixedpoint.py:52-76.

    ``mult`` is a Python int or an integer array that broadcasts against ``x``.
    ``nudge`` (stochastic only) is the ``U[0, 2**shift)`` draw, shaped like the product.
    """
    xi = np.asarray(x).astype(np.int64)
    if isinstance(mult, np.ndarray):
        prod = mul64(xi, mult.astype(np.int64))
    else:
        prod = mul64(xi, np.int64(mult)) if mult != 1 else xi
    if shift >= 0:
        denom = 1 << shift
        if stochastic:
            assert nudge is not None, "stochastic rounding needs a nudge array"
            nudge = np.asarray(nudge).astype(np.int64)
            assert nudge.shape == prod.shape, (nudge.shape, prod.shape)
            assert nudge.min(initial=0) >= 0 and nudge.max(initial=0) < denom
            prod = add64(prod, nudge)
        else:
            prod = add64(prod, np.int64(denom >> 1))
        return sar64(prod, shift)
    return shl64(prod, -shift)


def to_int8_sat(x) -> np.ndarray:
    """fixedpoint.py:79-82."""
    return np.clip(np.asarray(x), INT8_LO, INT8_HI).astype(np.int8)


def int_amax(x) -> int:
    """fixedpoint.py:85-88 (abs with int64 wrap, like torch)."""
    a = np.asarray(x).astype(np.int64)
    return int(np.abs(a).max())


def int_mm(a8: np.ndarray, b8: np.ndarray) -> np.ndarray:
    """Exact int8 x int8 -> int32 product (``torch._int_mm``, ilayer.py:40-54).

    float64 BLAS is exact here: every partial sum is an integer of magnitude at
    most K * 128**2 < 2**53.  The int32 result wraps like int32 accumulation.
    """
    a = np.asarray(a8, dtype=np.int8)
    b = np.asarray(b8, dtype=np.int8)
    assert a.ndim == 2 and b.ndim == 2 and a.shape[1] == b.shape[0]
    acc = a.astype(np.float64) @ b.astype(np.float64)
    return acc.astype(np.int64).astype(np.int32)


def col_mults(ratios) -> tuple[np.ndarray, int]:
    """Per-channel ``(mult, shift)`` with one common (minimum) shift.

    ``ilayer.py:66-68`` and ``iopt.py:51-53``: ``mults = m >> (s - com)``.
    Returns int32 multipliers and the common shift.
    """
    ms = [quantize_multiplier(r) for r in ratios]
    com = min(s for _, s in ms)
    return np.array([m >> (s - com) for m, s in ms], dtype=np.int32), com
