"""I8ECO: integer-only ECO step (drop-in for ``ecoint8/strict/iopt.py`` v0.4.9).

The reference runs ~15 eager int64 kernels per 64-row chunk with two host
synchronisations per chunk and builds every per-row multiplier in Python.
Here ``step()`` is ONE kernel launch for all layers (``eco_i8eco_step``): the
per-row (mult, shift) columns of iopt.py:134-148 are derived on the device in
IEEE double (bit-identical to Python's float arithmetic), the gradient clip
reads the square sum that the dW requant produced, weights and momentum are
updated in place in one pass (read w, m, g; write w, m), the momentum scale
``s_m`` is updated on the device from the row maxima, and per-row sums of |e|
are kept for ``stats``.  No host synchronisation.

Host-visible state keeps the reference's names and types:
``m_i8`` (int8 tensors), ``s_m`` (a list of Python floats, read from the
device when accessed), ``step_count``, ``stats`` (``mean_abs_e`` computed from
the row sums on first access, with the reference's summation order), ``lr``,
``beta``, ``grad_clip``, ``chunk_rows``.  ``chunk_rows`` no longer changes the
arithmetic; in the verification (replay) mode it orders the consumed draws
exactly like the reference's chunk loop.

Errors: where the reference raises inside ``step`` (a stochastic-rounding
shift of 63 or more, ``torch.randint``'s ValueError), this step raises the same
ValueError.  The bias shift is known on the host and checked before the launch
(state untouched); a momentum / gradient shift overflow is detected by the
kernel, which leaves that layer untouched, and is raised at the next ``step``,
``s_m`` or ``stats`` access.
"""

from __future__ import annotations

import ctypes
import math
import struct
import time

import torch

from .. import _native as nat
from .. import _ops, _scale, _sr, parallel
from ..fixedpoint import _check_int, quantize_multiplier
from .ilayer import _ScaleList

layer_values = _ScaleList.values

__all__ = ["I8ECO"]

FRAC_BITS = 12
HOST_WAIT_S = [0.0]  # seconds step() spent waiting for the device (the previous step's flags)
BETA_Q = 1 << 16  # beta in 16-bit fixed-point
LR_Q = 1 << 16  # lr in 16-bit fixed-point (requires lr < 2)


def _bits(v: float) -> int:
    return struct.unpack("<q", struct.pack("<d", float(v)))[0]


def _float(b: int) -> float:
    return struct.unpack("<d", struct.pack("<q", int(b)))[0]


def _col_mults(ratios: list[float], dev: torch.device) -> tuple[torch.Tensor, int]:
    """Per-row ``(mult, shift)`` pairs sharing one common shift (iopt.py:42-54)."""
    ms = [quantize_multiplier(r) for r in ratios]
    com = min(s for _, s in ms)
    mults = torch.tensor([m >> (s - com) for m, s in ms], dtype=torch.int32, device=dev)
    return mults.unsqueeze(1), com


def _common_shift(ratios) -> int:
    return min(quantize_multiplier(r)[1] for r in ratios)


class _ScaleView(list):
    """``s_m`` as a list of floats; item assignment writes through to the optimizer."""

    def __init__(self, opt, values):
        super().__init__(values)
        self._opt = opt

    def __setitem__(self, i, v):
        super().__setitem__(i, v)
        self._opt.s_m = list(self)


class I8ECO:
    """Fully integer ECO-SGDM for ``I8Linear`` layers.  Zero fp32 state or temporaries."""

    def __init__(self, layers, lr: float = 0.5, momentum: float = 0.9, grad_clip: float | None = 1.0,
                 chunk_rows: int = 64):
        assert momentum > 0, "ECO requires beta > 0"
        assert 0.0 < lr < 2.0, "lr must fit 16-bit fixed-point (0, 2)"
        assert chunk_rows >= 1, "chunk_rows must be positive"
        self.layers = list(layers)
        self.lr = float(lr)
        self.beta = float(momentum)
        self.grad_clip = grad_clip
        self.chunk_rows = int(chunk_rows)
        self.m_i8 = [torch.zeros_like(layer.w_i8) for layer in self.layers]
        self._s_m_host = [1.0 for _ in self.layers]
        self._state = None  # device int64 [L, 4]: s_m bits, row-max accumulator, error flags, spare
        self._counter = None
        self._rowsum: list[torch.Tensor | None] = [None] * len(self.layers)
        self._pending_stats = None
        self._err = None  # (event, pinned flags) of the last launch
        self.step_count = 0
        self._stats = {"skipped": 0, "mean_abs_e": 0.0}

    # -- checkpointing (torch.save of the optimizer, as of the reference's plain object) --
    def __getstate__(self):
        """The reference's state (layers, hyper-parameters, ``m_i8``, ``s_m``, ``stats``,
        ``step_count``); device bookkeeping and launch caches are rebuilt after loading.
        Under data parallelism, call ``parallel.synchronize`` and ``gather_momentum`` first."""
        d = dict(self.__dict__)
        if self._state is not None:
            d["_s_m_host"] = [float(v) for v in self.s_m]  # reads the device (raises pending errors)
            d["_stats"] = dict(self.stats)
        for k in ("_plan_cache", "_keep_plan", "_flag_bufs", "_flag_turn", "_err", "_keep", "_rowsum_work"):
            d.pop(k, None)
        d.update(_state=None, _counter=None, _pending_stats=None, _err=None,
                 _rowsum=[None] * len(self.layers))
        return d

    def __setstate__(self, d):
        self.__dict__.update(d)

    # -- reference attributes ----------------------------------------------
    @property
    def s_m(self) -> list[float]:
        if self._state is None:
            return _ScaleView(self, self._s_m_host)
        self._raise_pending(block=True)
        return _ScaleView(self, [_float(b) for b in self._state[:, 0].tolist()])

    @s_m.setter
    def s_m(self, values) -> None:
        values = [float(v) for v in values]
        assert len(values) == len(self.layers)
        if self._state is None:
            self._s_m_host = values
        else:
            self._state[:, 0].copy_(torch.tensor([_bits(v) for v in values], dtype=torch.int64))

    @property
    def stats(self) -> dict:
        if self._pending_stats is not None:
            work = getattr(self, "_rowsum_work", None)
            if work is not None:  # row sums of other ranks (data parallel)
                work.wait()
                self._rowsum_work = None
            self._raise_pending(block=True)
            tot_e, n_e = 0.0, 0
            for src, token, rowlen, out in self._pending_stats:
                sw = layer_values(token)
                rowsum = src if isinstance(src, torch.Tensor) else src[0][:, src[1]:src[1] + src[2]].reshape(-1)
                rs = rowsum.tolist()
                tot_e += sum(s * sw_o for s, sw_o in zip(rs, sw)) / rowlen / (1 << FRAC_BITS)  # iopt.py:183
                n_e += out
            if n_e:
                self._stats["mean_abs_e"] = tot_e / n_e
            self._pending_stats = None
        return self._stats

    @stats.setter
    def stats(self, value: dict) -> None:
        self._pending_stats = None
        self._stats = value

    def set_lr(self, lr: float):
        assert 0.0 < lr < 2.0, "lr must fit 16-bit fixed-point (0, 2)"
        self.lr = float(lr)

    # -- device state ------------------------------------------------------
    def _ensure_state(self, dev: torch.device) -> None:
        if self._state is not None and self._state.device == dev:
            return
        s_m = self._s_m_host if self._state is None else self.s_m
        st = torch.zeros((len(self.layers), 4), dtype=torch.int64)
        st[:, 0] = torch.tensor([_bits(v) for v in s_m], dtype=torch.int64)
        self._state = st.to(dev)
        self._counter = torch.zeros(1, dtype=torch.int32, device=dev)

    def _raise_pending(self, block: bool, idle: bool = False) -> None:
        """Raise the error a finished step flagged.  ``idle``: the device is known to be
        idle (no event calls, e.g. while a graph is being captured)."""
        if self._err is None:
            return
        event, flags, sflags = self._err
        if not idle:
            if not block and not event.query():
                return
            event.synchronize()
        self._err = None
        if int(sflags[0]):  # a device scale of the queued backward overflowed (the reference raises there)
            _scale.raise_flags(self._state.device)
        bad = [(i, int(f)) for i, f in enumerate(flags.tolist()) if f]
        if bad:
            self._state[:, 2].zero_()
            i, f = bad[0]
            if f & nat.FLAG_SHIFT_OVERFLOW:
                # the reference raises here from torch.randint(0, 2**shift) with shift >= 63
                raise ValueError(f"Overflow when unpacking long long (I8ECO layer {i}: a requant shift "
                                 "exceeded 62; that layer was left unchanged)")
            raise ValueError(f"I8ECO layer {i}: invalid scale ratio (flags {f}); layer left unchanged")

    def _gsq(self, layer, g: torch.Tensor) -> torch.Tensor:
        """sum g^2 on the device: the dW requant's by-product, or one reduction."""
        if getattr(layer, "_gw_sumsq_of", None) is g and getattr(layer, "_gw_sumsq", None) is not None:
            return layer._gw_sumsq
        return _ops.sumsq(g)

    # -- step ------------------------------------------------------------
    def _hyper(self, replay: bool, dp: bool) -> "nat.I8ECOHyper":
        """The launch's hyper-parameters from the current lr and momentum (iopt.py:104-110)."""
        b = self.beta
        alpha = (1.0 / self.lr) * (1.0 - 1.0 / b)
        hyper = nat.I8ECOHyper()
        hyper.lr = self.lr
        hyper.grad_clip = -1.0 if self.grad_clip is None else float(self.grad_clip)
        hyper.b_q, hyper.nb_q = round(b * BETA_Q), round((1.0 - b) * BETA_Q)
        hyper.lr_q, hyper.a_q = round(self.lr * LR_Q), round(alpha * BETA_Q)
        hyper.sr_mode = nat.SR_REPLAY32 if replay else nat.SR_PHILOX
        hyper.finalize = 0 if dp else 1  # under data parallelism: max over the row shards first
        hyper.done_counter = self._counter.data_ptr()
        return hyper

    @torch.no_grad()
    def step(self):
        from .. import graphs

        graph = graphs.capturing()
        t0 = time.perf_counter()
        if graph is None:
            self._raise_pending(block=True)  # the previous step's flags (long since copied back)
        else:  # capture starts on an idle device: the last eager step's flags are in
            self._raise_pending(block=True, idle=True)
        HOST_WAIT_S[0] += time.perf_counter() - t0
        if graph is None:
            self.step_count += 1
        active = [(i, layer) for i, layer in enumerate(self.layers) if layer._gw_i8 is not None]
        if not active:
            return
        dev = nat.require_cuda(*[layer.w_i8 for _, layer in active])
        self._ensure_state(dev)
        replay = _sr.replaying()
        if replay:
            s_m_now = [_float(v) for v in self._state[:, 0].tolist()]
        dp = parallel.active()
        plan = self._plan(active, dev, dp)
        keep = []  # tensors that must outlive the launch
        for (i, layer), d, rows in zip(active, plan["descs"], plan["rows"]):
            g = layer._gw_i8
            _check_int(g, "weight grad")
            w = layer.w_i8
            lo, hi = (0, w.shape[0]) if rows is None else rows
            if g.dtype != torch.int8 or not g.is_contiguous() or tuple(g.shape) != (hi - lo, w.shape[1]):
                raise RuntimeError("I8ECO: weights, momentum and gradient must be contiguous int8 of one shape")
            nat.require_cuda(g)
            out, rowlen = w.shape
            s_g_raw = layer.__dict__.get("_gw_s_store")  # a float, or a device scale of a queued backward
            queued_g = isinstance(s_g_raw, _scale.DevScale) and not replay
            s_g = 0.0 if queued_g else _scale.as_float(s_g_raw)
            gsq = self._gsq(layer, g) if self.grad_clip is not None else None
            d.g, d.gsq, d.s_g = g.data_ptr(), nat.ptr(gsq), s_g
            d.s_g_dev = s_g_raw.ptr() if queued_g else None
            d.s_gb_dev = None
            d.nudge_w = d.nudge_m = d.nudge_b = None
            d.nudge_m_bits = d.nudge_b_bits = 32
            if layer.use_bias:
                gb = layer._gb_sum
                if gb.dtype != torch.int64 or gb.device != dev or not gb.is_contiguous():
                    gb = gb.to(device=dev, dtype=torch.int64).contiguous()
                s_gb_raw = layer.__dict__.get("_gb_s_store")
                if isinstance(s_gb_raw, _scale.DevScale) and not replay:
                    # on the device: the kernel flags a bias shift beyond 62 and leaves the layer
                    d.s_gb, d.s_gb_dev = 0.0, s_gb_raw.ptr()
                    keep.append(s_gb_raw.t)
                else:
                    s_gb = _scale.as_float(s_gb_raw)
                    com_b = _common_shift([self.lr * s_gb / (layer.sx * d.sw_min)])  # = min over rows
                    if com_b > 62:  # the reference's torch.randint(0, 2**com_b) raises (iopt.py:194)
                        raise ValueError("Overflow when unpacking long long")
                    d.s_gb = s_gb
                d.gb_sum = gb.data_ptr() + 8 * lo
                keep.append(gb)
            if replay:
                keep += self._replay_nudges(d, layer, s_m_now[i], s_g, gsq, (out, rowlen), lo)
            keep += [g, gsq] + ([s_g_raw.t] if queued_g else [])
        hyper = self._hyper(replay, dp)
        key = 0 if replay else _sr.new_key()
        if isinstance(key, graphs.DevKey):
            # a replayed step reads the lr and key of the moment from the graph's table
            def image(table, key=key, replay=replay, dp=dp):
                h = self._hyper(replay, dp)
                h.seed = table.value(key.off)
                return h

            hyper.seed = 0
            hyper.dev = graph.table.block((ctypes.sizeof(nat.I8ECOHyper) + 7) // 8, graphs.struct_fill(image))
        else:
            hyper.seed = key
        if _sr.LOG is not None and not replay:
            _sr.LOG.append(("i8eco_step", hyper.seed, [(i, 2 * i, 2 * i + 1) for i, _ in active]))
        self._keep_plan = plan
        nat.call("eco_i8eco_step", plan["arr"], len(active), ctypes.byref(hyper), nat.stream())
        self._rowsum_work = None
        if dp:
            parallel.combine_step_state(self._state)
            nat.call("eco_i8eco_finalize", self._state.data_ptr(), self._state.shape[0], nat.stream())
            for (_, layer), rows in zip(active, plan["rows"]):
                if rows is not None:
                    parallel.gather_rows(layer, rows)
            if plan["flat"] is not None:
                self._rowsum_work = parallel.gather_flat(plan["flat"])
        pending = [(src, layer.sw.snapshot(), layer.w_i8.shape[1], layer.out_features)
                   for (_, layer), src in zip(active, plan["rowsum"])]
        # error flags come back asynchronously into one of two persistent pinned buffers
        # (allocating pinned memory every step can stall the host); a third one is a
        # captured graph's
        if getattr(self, "_flag_bufs", None) is None or self._flag_bufs[0][0].numel() != len(self.layers):
            self._flag_bufs = [(torch.empty(len(self.layers), dtype=torch.int64, pin_memory=True),
                                torch.empty(1, dtype=torch.int32, pin_memory=True),
                                torch.cuda.Event()) for _ in range(3)]
            self._flag_turn = 0
        if graph is not None:
            flags, sflags, _ = self._flag_bufs[2]
            flags.copy_(self._state[:, 2], non_blocking=True)
            sflags.copy_(_scale.flags(dev), non_blocking=True)
            work = self._rowsum_work

            def after_replay(flags=flags, sflags=sflags, pending=pending, work=work, keep=keep):
                if self._err is not None:  # the previous replay's flags (bounds the host's lead)
                    t0 = time.perf_counter()
                    self._raise_pending(block=True)
                    HOST_WAIT_S[0] += time.perf_counter() - t0
                self.step_count += 1
                ev = torch.cuda.Event()
                ev.record()
                self._err = (ev, flags, sflags)
                self._pending_stats = pending
                self._rowsum_work = work
                self._keep = keep

            graph.on_replay(after_replay)
            return
        self._pending_stats = pending
        flags, sflags, ev = self._flag_bufs[self._flag_turn]
        self._flag_turn ^= 1
        t0 = time.perf_counter()
        ev.synchronize()  # its previous copy finished a step ago
        HOST_WAIT_S[0] += time.perf_counter() - t0
        flags.copy_(self._state[:, 2], non_blocking=True)
        sflags.copy_(_scale.flags(dev), non_blocking=True)
        ev.record()
        self._err = (ev, flags, sflags)
        self._keep = keep  # released at the next step (stream-ordered reuse is safe)

    def _plan(self, active, dev, dp):
        """The step's layer descriptors with every field that does not change between
        steps filled in; rebuilt only when a layer, its storage, its row shard or its
        scales change.  Under data parallelism the row sums of the sharded layers live
        in one rank-major ``[world, sum of shard rows]`` buffer (one all-gather)."""
        world = parallel.world() if dp else 1
        rank = parallel.rank() if dp else 0
        key = [dp, world, rank, str(dev), self._state.data_ptr()]
        for i, layer in active:
            if self.m_i8[i].device != layer.w_i8.device:  # layer moved after construction: follow it
                self.m_i8[i] = self.m_i8[i].to(layer.w_i8.device)
            key.append((i, id(layer), layer.w_i8.data_ptr(), tuple(layer.w_i8.shape), self.m_i8[i].data_ptr(),
                        getattr(layer, "_gw_rows", None), layer.use_bias,
                        layer.b_acc.data_ptr() if layer.use_bias else 0, layer._sw_key(), layer.sx))
        plan = getattr(self, "_plan_cache", None)
        if plan is not None and plan["key"] == key:
            return plan
        shard_total = sum(r[1] - r[0] for r in (getattr(l, "_gw_rows", None) for _, l in active) if r is not None)
        flat = parallel.flat_buffer((world, shard_total), dev) if dp and shard_total else None
        descs, rows_l, rowsum_l = [], [], []
        off = 0
        for i, layer in active:
            w, m = layer.w_i8, self.m_i8[i]
            nat.require_cuda(w, m)
            if not (w.dtype == torch.int8 and m.dtype == torch.int8 and w.is_contiguous() and m.is_contiguous()
                    and m.shape == w.shape):
                raise RuntimeError("I8ECO: weights, momentum and gradient must be contiguous int8 of one shape")
            rows = getattr(layer, "_gw_rows", None)  # this rank's row shard under data parallelism
            lo, hi = (0, w.shape[0]) if rows is None else rows
            out, rowlen = w.shape
            sw_bits, sw_min, sw_max = layer._sw_device(dev)
            d = nat.I8ECOLayer()
            d.w, d.m = w.data_ptr() + lo * rowlen, m.data_ptr() + lo * rowlen
            d.sw = sw_bits.data_ptr() + 8 * lo
            if rows is not None and flat is not None:
                d.rowsum = flat[rank, off:off + hi - lo].data_ptr()
                rowsum_l.append((flat, off, hi - lo))
                off += hi - lo
            else:
                if self._rowsum[i] is None or self._rowsum[i].numel() != out or self._rowsum[i].device != dev:
                    self._rowsum[i] = torch.empty(out, dtype=torch.int64, device=dev)
                d.rowsum = self._rowsum[i].data_ptr()
                rowsum_l.append(self._rowsum[i])
            d.state = self._state[i].data_ptr()
            d.rows, d.cols, d.row_base = hi - lo, rowlen, lo
            d.sw_min, d.sw_max = sw_min, sw_max
            d.stream_w, d.stream_b = 2 * i, 2 * i + 1
            d.bias_rows = 0
            if layer.use_bias:
                assert isinstance(layer.sx, float)
                d.b_acc, d.sx = layer.b_acc.data_ptr() + 4 * lo, layer.sx
                if rows is not None:  # every rank steps every bias (gb_sum is complete on each rank)
                    d.bias_rows = out
            descs.append(d)
            rows_l.append(rows)
        arr = (nat.I8ECOLayer * len(descs))(*descs)
        plan = {"key": key, "arr": arr, "descs": list(arr), "rows": rows_l, "rowsum": rowsum_l, "flat": flat,
                "sw": [layer._sw_device(dev)[0] for _, layer in active]}
        self._plan_cache = plan
        return plan

    def _replay_nudges(self, d, layer, s_m: float, s_g: float, gsq, shape, lo: int = 0):
        """Verification mode: draw in the reference's order (iopt.py:152-197), consume whole.

        Host scalars follow the reference expressions; the kernel recomputes the
        same shifts on the device.
        """
        F = FRAC_BITS
        out, rowlen = shape
        dev = layer.w_i8.device
        if self.grad_clip is not None:
            sq_sum = int(gsq.item())
            n_real = math.sqrt(sq_sum) * s_g
            if n_real > self.grad_clip:
                s_g = s_g * (self.grad_clip / n_real)
        com_mm = _common_shift([(sw_o / (1 << F)) / s_m if s_m > 0 else 0.0 for sw_o in layer.sw])
        ws, ms = [], []
        for c in range(0, out, self.chunk_rows):
            rows = min(c + self.chunk_rows, out) - c
            ws.append(_sr.replay_draw((rows, rowlen), 1 << F, dev).to(torch.int32))
            if com_mm >= 0:
                ms.append(_sr.replay_draw((rows, rowlen), 1 << com_mm, dev))
        nw = torch.cat(ws).contiguous()
        nm = torch.cat(ms).contiguous() if ms else torch.zeros(1, dtype=torch.int32, device=dev)
        d.nudge_m_bits = 64 if nm.dtype == torch.int64 else 32
        d.nudge_w = nw.data_ptr() + 4 * lo * rowlen  # a row shard consumes its rows of the layer's draws
        d.nudge_m = nm.data_ptr() + (d.nudge_m_bits // 8) * lo * rowlen if ms else nm.data_ptr()
        kept = [nw, nm]
        if layer.use_bias:
            com_b = _common_shift([self.lr * _scale.as_float(layer.__dict__.get("_gb_s_store")) / (layer.sx * sw_o)
                                   for sw_o in layer.sw])
            if com_b >= 0:
                nb = _sr.replay_draw((out, 1), 1 << com_b, dev).reshape(out).contiguous()
            else:
                nb = torch.zeros(1, dtype=torch.int32, device=dev)
            d.nudge_b_bits = 64 if nb.dtype == torch.int64 else 32
            d.nudge_b = nb.data_ptr() + ((d.nudge_b_bits // 8) * lo if com_b >= 0 else 0)
            kept.append(nb)
        return kept

    @torch.no_grad()
    def zero_grad(self):
        for layer in self.layers:
            layer._gw_i8 = None

    def memory_bytes(self) -> int:
        """Stored integer state in bytes (int8 weights live on layers; int8 momentum here)."""
        return sum(m.numel() for m in self.m_i8)
