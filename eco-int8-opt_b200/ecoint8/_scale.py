"""Scales that live on the device.

When ``I8Sequential.backward_i8`` queues a whole backward pass (Philox mode), each
layer's dX and dW scales are computed by ``eco_scale_from_amax`` from the device
maxima, in the reference's IEEE double arithmetic, and the requants read their
multiplier and shift in place: no host round trip per layer.  A ``DevScale`` is
the result -- an int64 ``[3]`` tensor ``(double bits of s, mult, shift)`` -- and
becomes the reference's Python float the first time it is read (one device
synchronisation).  Kernels that consume it (the next layer's scale, the I8ECO
step) read the double in place.

Overflow: where the reference raises inside ``backward_i8`` (a stochastic-rounding
shift beyond 62), the scale kernel raises a flag in a per-device word instead; the
flag is checked, and the same ``ValueError`` raised, whenever a ``DevScale`` is
read and at every ``I8ECO.step``.
"""

from __future__ import annotations

import struct

import torch

from . import _native as nat

_FLAGS: dict = {}  # device -> int32 [1] flag word of the scale kernels


def flags(device) -> torch.Tensor:
    t = _FLAGS.get(device)
    if t is None:
        t = _FLAGS[device] = torch.zeros(1, dtype=torch.int32, device=device)
    return t


def raise_flags(device) -> None:
    """Raise the reference's error if a device scale overflowed (synchronises)."""
    t = _FLAGS.get(device)
    if t is None:
        return
    f = int(t.item())
    if f:
        t.zero_()
        if f & nat.FLAG_SHIFT_OVERFLOW:
            # the reference raises here from torch.randint(0, 2**shift) with shift >= 63
            raise ValueError("Overflow when unpacking long long (a backward requant shift exceeded 62)")
        raise AssertionError("scale ratios must be non-negative")


class DevScale:
    """A scale on the device; ``float(s)`` reads it."""

    __slots__ = ("t", "_v")

    def __init__(self, t: torch.Tensor):
        self.t = t
        self._v: float | None = None

    def value(self) -> float:
        if self._v is None:
            raise_flags(self.t.device)
            self._v = struct.unpack("<d", struct.pack("<q", int(self.t[0].item())))[0]
        return self._v

    def __float__(self) -> float:
        return self.value()

    def ptr(self) -> int:
        return self.t.data_ptr()  # the double bits of s


def as_float(s) -> float:
    return s.value() if isinstance(s, DevScale) else float(s)


def gain_args(s):
    """``(device pointer or None, host value)`` of a scale for ``eco_scale_from_amax``."""
    if isinstance(s, DevScale):
        return s.ptr(), 0.0
    return None, float(s)


def from_amax(amax: torch.Tensor, s_in, gain1: float) -> DevScale:
    """``dynamic_scale_from_int(amax, s_in * gain1)`` and its multiplier, on the device."""
    out = torch.empty(3, dtype=torch.int64, device=amax.device)
    g0, g0v = gain_args(s_in)
    bits = 32 if amax.dtype == torch.int32 else 64
    nat.call("eco_scale_from_amax", amax.data_ptr(), bits, g0, g0v, float(gain1), out.data_ptr(),
             flags(amax.device).data_ptr(), nat.stream())
    return DevScale(out)
