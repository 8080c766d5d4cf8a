"""A training step captured once as a CUDA graph and replayed.

The strict step issues a few dozen library launches and small torch operations per
step.  On one GPU the device is the bottleneck; under data parallelism each GPU's
share of the work shrinks while the host's does not, and eight processes issuing
launches one by one cannot keep eight B200s busy.  ``StepGraph`` records one step --
any callable that runs this package on device tensors of fixed shape -- into a CUDA
graph and replays it: a step then costs one graph launch and one small copy.

Values that change from step to step are read by the recorded kernels from a table of
64-bit words in device memory, refreshed before every replay by one host-to-device copy:

* Philox keys: every stochastic-rounding site of the captured step owns a key word
  (``ECO_SR_PHILOX_DEV``).  Before a replay the host draws the keys from the generator
  the eager step draws from (``ecoint8._sr``), as many and in the same order, so a
  replayed step is bit for bit the step an uncaptured call would have made;
* the ``I8ECO`` step's hyper-parameters (so ``set_lr`` between replays takes effect);
* the epochs of the data-parallel peer exchange's flag barriers, advanced on the host
  exactly as the eager calls advance them.

Host bookkeeping that the captured code did once (the optimizer's step count, its
error-flag read-back, the statistics it will report) is redone after every replay by
hooks that the components register while they are being captured.

Rules for the captured callable: inputs and outputs are tensors whose storage stays
fixed (copy new data into the inputs before ``replay``); it runs in Philox mode (not
inside ``sr_replay`` and with no site log); layer shapes, scales and the optimizer's
layer list do not change between capture and replay (capture again if they do).
"""

from __future__ import annotations

import ctypes

import torch

_ACTIVE: "StepGraph | None" = None


def capturing() -> "StepGraph | None":
    """The graph being captured by this process, or None."""
    return _ACTIVE


class DevKey:
    """A Philox key word of a captured graph's table (``ptr``: its device address)."""

    __slots__ = ("ptr", "off")

    def __init__(self, ptr: int, off: int):
        self.ptr = ptr
        self.off = off

    def __int__(self):
        raise TypeError("a captured graph's Philox key lives on the device; it has no host value at capture")

    def __repr__(self):
        return f"DevKey(word {self.off})"


class _Table:
    """The per-replay words: pinned host halves (alternating) and their device copy."""

    def __init__(self, device: torch.device, words: int = 16384):
        self.device = device
        self.words = words
        self.dev = torch.zeros(words, dtype=torch.int64, device=device)
        self.host = [torch.zeros(words, dtype=torch.int64).pin_memory() for _ in range(2)]
        self.copied = [None, None]
        self.turn = 0
        self.n = 0
        self.keys: list[int] = []  # word offsets of Philox keys, in draw order
        self.fills: list = []  # (offset, words, fn(host_view, table) -> None), in capture order

    def alloc(self, words: int) -> int:
        off = self.n
        self.n += words
        if self.n > self.words:
            raise RuntimeError(f"captured step needs more than {self.words} table words")
        return off

    def ptr(self, off: int) -> int:
        return self.dev.data_ptr() + 8 * off

    def key(self) -> DevKey:
        off = self.alloc(1)
        self.keys.append(off)
        return DevKey(self.ptr(off), off)

    def word(self, fn) -> int:
        """A word whose value ``fn()`` gives at every refresh (run in capture order)."""
        off = self.alloc(1)
        self.fills.append((off, 1, lambda view, t, fn=fn: view.__setitem__(0, int(fn()))))
        return self.ptr(off)

    def block(self, words: int, fn) -> int:
        """``words`` words that ``fn(view, table)`` fills at every refresh."""
        off = self.alloc(words)
        self.fills.append((off, words, fn))
        return self.ptr(off)

    def refresh(self) -> None:
        from . import _sr

        h = self.host[self.turn]
        ev = self.copied[self.turn]
        if ev is not None:
            ev.synchronize()  # that half's previous copy has left the host (two replays ago)
        if self.keys:
            if getattr(self, "_key_idx", None) is None or self._key_idx.numel() != len(self.keys):
                self._key_idx = torch.tensor(self.keys, dtype=torch.int64)
            # one draw of all the step's keys: the sequence of single draws the eager step makes
            h[self._key_idx] = torch.randint(0, 1 << 62, (len(self.keys),), generator=_sr._GEN)
        self._h = h
        for off, words, fn in self.fills:
            fn(h[off:off + words], self)
        self.dev[:self.n].copy_(h[:self.n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.copied[self.turn] = ev
        self.turn ^= 1

    def value(self, off: int) -> int:
        """A word's value in the refresh under way (for fills that embed a key)."""
        return int(self._h[off])


def struct_fill(struct_fn):
    """A ``block`` filler that writes the bytes of the ctypes structure ``struct_fn(table)``."""

    def fill(view: torch.Tensor, table: _Table) -> None:
        st = struct_fn(table)
        raw = bytes(st)
        words = (len(raw) + 7) // 8
        buf = (ctypes.c_int64 * words)()
        ctypes.memmove(buf, raw, len(raw))
        view[:words] = torch.tensor(list(buf), dtype=torch.int64)

    return fill


class StepGraph:
    """One step of ``fn`` (no arguments; returns a tensor or a tuple of tensors)
    captured as a CUDA graph.

    ``capture()`` runs ``warmup`` eager steps (they build every launch plan, exchange
    buffer and cached multiplier; they are real training steps), then records one step.
    ``replay()`` refreshes the per-step words, launches the graph on the current stream
    and returns the outputs of the recorded step (the same tensors every time).
    """

    def __init__(self, fn, warmup: int = 1):
        self.fn = fn
        self.warmup = int(warmup)
        self.graph = None
        self.table: _Table | None = None
        self.hooks: list = []  # run after every replay, in registration order
        self.joins: list = []  # side streams to join before the capture ends
        self.outputs = None
        self.replays = 0

    # -- used by the components while they are captured --------------------------------
    def on_replay(self, fn) -> None:
        self.hooks.append(fn)

    def join(self, stream: torch.cuda.Stream) -> None:
        if all(s is not stream for s in self.joins):
            self.joins.append(stream)

    # -- capture and replay ---------------------------------------------------------------
    def capture(self):
        """Run the warm-up steps, record one step; returns the last warm-up step's outputs."""
        global _ACTIVE
        from . import _sr, parallel

        if _sr.replaying() or _sr.LOG is not None:
            raise RuntimeError("StepGraph captures Philox-mode steps only (no sr_replay, no site log)")
        if parallel.active() and parallel.exchange() != "peer":
            raise RuntimeError("capturing a data-parallel step needs the peer exchange (dw_exchange='peer')")
        if self.warmup < 1:
            raise ValueError("StepGraph needs at least one warm-up step (it builds the launch plans)")
        out = None
        for _ in range(self.warmup):
            out = self.fn()
        dev = torch.device("cuda", torch.cuda.current_device())
        torch.cuda.synchronize(dev)
        self.table = _Table(dev)
        self.graph = torch.cuda.CUDAGraph()
        if _ACTIVE is not None:
            raise RuntimeError("another StepGraph is being captured")
        _ACTIVE = self
        try:
            with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
                self.outputs = self.fn()
                cur = torch.cuda.current_stream()
                for s in self.joins:
                    cur.wait_stream(s)
        finally:
            _ACTIVE = None
        torch.cuda.synchronize(dev)
        return out

    def replay(self):
        if self.graph is None:
            raise RuntimeError("StepGraph.replay before capture()")
        self.table.refresh()
        self.graph.replay()
        self.replays += 1
        for h in self.hooks:
            h()
        return self.outputs

    __call__ = replay

    @property
    def keys_per_step(self) -> int:
        return len(self.table.keys) if self.table is not None else 0
