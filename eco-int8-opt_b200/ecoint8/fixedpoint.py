"""Integer-only fixed-point helpers (drop-in for ``ecoint8/fixedpoint.py`` v0.4.9).

Scalar bookkeeping (``quantize_multiplier``, ``pad_mm_dims``,
``dynamic_scale_from_int``) is the reference's own Python arithmetic, line
for line, so every ``(mult, shift)`` is bit-identical.  Tensor functions run
on the B200 library: ``apply_mult_shift`` is one int64 register pass
(``eco_apply_mult_shift``) instead of eager int64 temporaries, and
``int_amax`` a device reduction.  CUDA tensors only; no CPU path.
"""

from __future__ import annotations

import math

import torch

from . import _native, _ops, _sr

_INT8_LO, _INT8_HI = -127, 127

__all__ = ["quantize_multiplier", "apply_mult_shift", "to_int8_sat", "int_amax", "pad_mm_dims",
           "dynamic_scale_from_int"]


def _check_int(t: torch.Tensor, name: str = "tensor") -> torch.Tensor:
    """fixedpoint.py:19-23."""
    assert t.dtype in (torch.int8, torch.int32, torch.int64), (
        f"{name} must be integral, got {t.dtype} — fp32 leaked into the int path"
    )
    return t


def quantize_multiplier(r: float) -> tuple[int, int]:
    """``r ~= mult / 2**shift`` with ``mult`` in [2**30, 2**31).  fixedpoint.py:26-37."""
    assert r >= 0.0, "scale ratios must be non-negative"
    if r == 0.0:
        return 0, 0
    mantissa, exponent = math.frexp(r)
    shift = exponent
    mult = round(mantissa * (1 << 31))
    if mult == (1 << 31):
        mult //= 2
        shift += 1
    return mult, 31 - shift


def _sr_nudge(shape: torch.Size, denom: int, device: torch.device) -> torch.Tensor:
    """``U[0, denom)`` draw in the narrowest dtype (fixedpoint.py:40-49)."""
    dtype = torch.int32 if denom <= (1 << 31) else torch.int64
    return torch.randint(0, denom, shape, dtype=dtype, device=device)


def _check_shift(shift: int, stochastic: bool) -> None:
    """The reference's int64 tensor arithmetic cannot represent 2**shift beyond 62."""
    if shift > 62:
        if stochastic:
            raise ValueError("Overflow when unpacking long long")  # torch.randint(0, 2**shift)
        raise RuntimeError(f"value cannot be converted to type int64_t without overflow (shift {shift})")


def apply_mult_shift(x: torch.Tensor, mult, shift: int, stochastic: bool = False) -> torch.Tensor:
    """Integer ``y = round(x * mult / 2**shift)`` -> int64.  fixedpoint.py:52-76.

    ``mult`` is a Python int or an integer tensor broadcastable against ``x``
    (one shared shift).  A per-column ``[cols]`` or per-row ``[rows, 1]``
    multiplier is read in place; any other broadcast is expanded first.  The
    stochastic draw has the shape of the product, as in the reference.
    """
    _check_int(x, "x")
    if shift >= 0:
        _check_shift(shift, stochastic)
    shape = x.shape
    kind, m = 0, mult
    if isinstance(mult, torch.Tensor):
        _check_int(mult, "mult")
        shape = torch.broadcast_shapes(x.shape, mult.shape)
        m32 = mult.to(device=x.device, dtype=torch.int32)
        if m32.numel() == 1:
            kind, m = 0, int(m32.reshape(()).item())
        else:
            kind, m = 1, m32.expand(shape).contiguous().reshape(-1)
    # kind 1 treats the product as one row with a multiplier per element
    x2 = x.expand(shape).reshape(1, -1) if kind == 1 else x.reshape(-1, shape[-1] if len(shape) else 1)
    if stochastic:
        site = _sr.draw(tuple(shape), shift, x.device, batch=False, kind="apply_mult_shift")
        if site.nudge is not None:
            site.nudge = site.nudge.reshape(x2.shape)
            site.spec.nudge = site.nudge.data_ptr()
            site.spec.nudge_ld = x2.shape[1]
    else:
        site = _sr.Site(_native.sr_spec(_native.SR_NEAREST), None)
    return _ops.apply_mult_shift(x2, m, kind, shift, site).reshape(shape)


def to_int8_sat(x: torch.Tensor) -> torch.Tensor:
    """Clamp an integral tensor into int8 (symmetric, [-127, 127]).  fixedpoint.py:79-82."""
    _check_int(x, "x")
    return torch.clamp(x, _INT8_LO, _INT8_HI).to(torch.int8)


def int_amax(x: torch.Tensor) -> int:
    """Max abs as a plain Python int (one device reduction + one read).  fixedpoint.py:85-88."""
    _check_int(x, "x")
    return int(_ops.amax(x).item())


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def pad_mm_dims(m: int, k: int, n: int) -> tuple[int, int, int]:
    """Padded dims the reference used for CUDA ``torch._int_mm`` (fixedpoint.py:95-102).

    Kept as API; the B200 GEMMs take any M, N, K and never pad.
    """
    return max(32, _pad8(m)), _pad8(k), _pad8(n)


def dynamic_scale_from_int(acc_amax: int, real_gain: float) -> float:
    """fixedpoint.py:105-114."""
    real_amax = acc_amax * real_gain
    if real_amax <= 0.0:
        return 1.0
    return real_amax / 127.0
