"""Stochastic-rounding draw sites.

Every place where the reference draws ``_sr_nudge(shape, 2**shift)``
(``ecoint8/fixedpoint.py:40-49``) is a *site* here.  A site is served in one of
two ways:

* Philox (default): the kernel generates the nudges itself from a 64-bit key
  and the element's (row, column).  Each site takes a fresh key from
  ``torch``'s default CPU generator (or from the generator set with
  ``set_generator``), so ``torch.manual_seed`` makes runs reproducible and
  data-parallel ranks that make the same calls draw the same keys.  Rows that
  are batch rows are numbered globally (``row_base``), so a batch split across
  ranks draws exactly the nudges the unsplit batch would.
* Replay: inside ``with replay(fn):`` every site calls ``fn(shape, denom,
  device)`` in the reference's order and the kernels consume the returned
  int32/int64 tensor.  With ``fn`` drawing ``torch.randint`` from the CPU
  generator, the draws are the reference's own, which makes the whole path
  bit-exact against a seeded CPU run of the reference.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch

from . import _native as nat

_REPLAY = None
_GEN: torch.Generator | None = None
_ROW_BASE = 0
LOG: list | None = None  # when a list, every Philox site appends (kind, seed, stream, shape, shift, row_base)


def reference_draw(shape, denom, device):
    """The reference's ``_sr_nudge`` draw, taken from the CPU generator (fixedpoint.py:48-49)."""
    dt = torch.int32 if denom <= (1 << 31) else torch.int64
    return torch.randint(0, denom, tuple(shape), dtype=dt)


@contextlib.contextmanager
def replay(fn=reference_draw):
    """Serve every SR site from ``fn(shape, denom, device)`` (verification mode)."""
    global _REPLAY
    prev, _REPLAY = _REPLAY, fn
    try:
        yield
    finally:
        _REPLAY = prev


def replaying() -> bool:
    return _REPLAY is not None


def set_generator(gen: torch.Generator | None) -> None:
    """Take Philox keys from ``gen`` instead of torch's default CPU generator."""
    global _GEN
    _GEN = gen


@contextlib.contextmanager
def batch_rows(row_base: int):
    """Number batch rows from ``row_base`` (this rank's first global sample)."""
    global _ROW_BASE
    prev, _ROW_BASE = _ROW_BASE, int(row_base)
    try:
        yield
    finally:
        _ROW_BASE = prev


def row_base() -> int:
    return _ROW_BASE


def new_key():
    """A site's Philox key: drawn now from the generator, or -- while a ``StepGraph`` is
    being captured -- a word of its table that every replay fills with a fresh draw."""
    from . import graphs

    g = graphs.capturing()
    if g is not None:
        return g.table.key()
    return int(torch.randint(0, 1 << 62, (1,), generator=_GEN).item())


@dataclass
class Site:
    spec: nat.SRSpec
    nudge: torch.Tensor | None  # keeps a replay tensor alive until the launch


def draw(shape, shift: int, device, batch: bool, kind: str = "requant") -> Site:
    """One SR site of a ``[rows, cols]`` requant with common shift ``shift``."""
    if shift < 0:  # left shift: the reference draws nothing
        return Site(nat.sr_spec(nat.SR_NEAREST), None)
    if _REPLAY is not None:
        t = _REPLAY(torch.Size(shape), 1 << shift, device)
        t = t.to(device=device).contiguous()
        mode = nat.SR_REPLAY32 if t.dtype == torch.int32 else nat.SR_REPLAY64
        return Site(nat.sr_spec(mode, t), t)
    key = new_key()
    rb = _ROW_BASE if batch else 0
    if LOG is not None:
        LOG.append((kind, key, 0, tuple(shape), shift, rb))
    return Site(nat.sr_spec(nat.SR_PHILOX, seed=key, stream_id=0, row_base=rb), None)


_RESERVED: dict = {}  # key -> its place in LOG, filled in by site_from_key


def reserve_key() -> int | None:
    """Take a site's Philox key now and build the site later (None in replay mode).
    ``LOG`` keeps the site at the position of the reservation."""
    if _REPLAY is not None:
        return None
    key = new_key()
    if LOG is not None:
        _RESERVED[key] = (LOG, len(LOG))
        LOG.append(None)
    return key


def site_from_key(key: int, shape, shift: int, row_base: int, kind: str = "requant") -> Site:
    """The Philox site of a key taken earlier with ``reserve_key``."""
    log, pos = _RESERVED.pop(key, (None, None))
    if shift < 0:
        if log is not None:  # no draw: the site leaves the log
            log[pos] = ("none", key, 0, tuple(shape), shift, row_base)
        return Site(nat.sr_spec(nat.SR_NEAREST), None)
    entry = (kind, key, 0, tuple(shape), shift, row_base)
    if log is not None:
        log[pos] = entry
    elif LOG is not None:
        LOG.append(entry)
    return Site(nat.sr_spec(nat.SR_PHILOX, seed=key, stream_id=0, row_base=row_base), None)


def replay_draw(shape, denom, device) -> torch.Tensor:
    """A raw draw from the active replay function (the step assembles its chunks)."""
    return _REPLAY(torch.Size(shape), denom, device).to(device=device)
