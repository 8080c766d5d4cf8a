"""Strict integer-only linear layers (drop-in for ``ecoint8/strict/ilayer.py`` v0.4.9).

Same classes, methods, attributes and scale bookkeeping as the reference; the
tensor work runs on the B200 library:

* ``forward_i8`` is ONE kernel: the int8 tcgen05 GEMM with the bias add,
  per-channel (mult, shift) requant, stochastic rounding, int8 saturation and
  -- when ``I8Sequential`` sees an ``I8ReLU`` next -- the ReLU in its
  epilogue.  The int32 accumulator never reaches HBM.
* ``backward_i8`` runs the dX and dW GEMMs with a fused max|acc|, then one
  requant kernel each; the maxima come back on a side stream, so the host
  reads the dX maximum while the dW GEMM runs and the device never waits for
  the host; the dW requant also produces the square sum that ``I8ECO``'s
  gradient clip needs, and the dX requant applies the mask of the preceding
  ``I8ReLU``.
* Scales stay plain Python floats computed by the reference's expressions, so
  every multiplier and shift is bit-identical.

Persist modules with ``torch.save(model)`` as in the reference (scales are
Python floats, not ``state_dict`` entries).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import _native, _ops, _scale, _sr, parallel
from ..fixedpoint import (
    _check_int,
    _check_shift,
    apply_mult_shift,
    dynamic_scale_from_int,
    pad_mm_dims,  # noqa: F401  (kept importable from this module, as in the reference)
    quantize_multiplier,
    to_int8_sat,
)

__all__ = ["I8Linear", "I8ReLU", "I8Sequential"]


class _ScaleList(list):
    """The per-row weight steps ``sw``: a plain list of floats that counts its edits."""

    def __init__(self, it=()):
        super().__init__(it)
        self.version = 0

    def _edited(self):
        # unpickling appends the items before it restores __dict__
        self.version = getattr(self, "version", 0) + 1

    def _before_edit(self):
        snap = self.__dict__.pop("_snap", None)
        if snap is not None:  # an outstanding snapshot keeps the values it was taken with
            snap[0] = list(self)

    def snapshot(self):
        """The current values, copied only if the list is edited before ``values(token)``."""
        snap = self.__dict__.get("_snap")
        if snap is None:
            snap = self.__dict__["_snap"] = [None]
        return self, snap

    @staticmethod
    def values(token) -> list:
        lst, snap = token
        return lst if snap[0] is None else snap[0]


for _name in ("__setitem__", "__delitem__", "__iadd__", "__imul__", "append", "extend", "insert", "pop",
              "remove", "clear", "sort", "reverse"):
    def _wrap(name=_name):
        base = getattr(list, name)

        def method(self, *a, **k):
            self._before_edit()
            r = base(self, *a, **k)
            self._edited()
            return self if name in ("__iadd__", "__imul__") else r

        method.__name__ = name
        return method

    setattr(_ScaleList, _name, _wrap())


def _int_mm(a8: torch.Tensor, b8: torch.Tensor) -> torch.Tensor:
    """int8 x int8 -> int32 on tcgen05 (ilayer.py:40-54); any M, K, N, no padding."""
    _check_int(a8, "mm lhs")
    _check_int(b8, "mm rhs")
    _native.require_cuda(a8, b8)
    M, K = a8.shape
    N = b8.shape[1]
    # b8 [K, N]: a transposed view of a contiguous [N, K] tensor is K-major already
    if b8.dim() == 2 and b8.stride(0) == 1 and b8.stride(1) >= K:
        return _ops.gemm_s32(a8, 0, b8.t(), 0, M, N, K)
    return _ops.gemm_s32(a8, 0, b8, 1, M, N, K)


def _requant_site(shape, shift, device, batch, kind):
    _check_shift(shift, True)
    return _sr.draw(shape, shift, device, batch=batch, kind=kind)


def _common_shift_requant(acc: torch.Tensor, ratios: list[float], stochastic: bool) -> torch.Tensor:
    """Requantize ``acc`` [N, out] with per-channel ratios -> int8 (ilayer.py:57-70)."""
    _check_int(acc, "acc")
    ms = [quantize_multiplier(r) for r in ratios]
    com = min(s for _, s in ms)
    mults = torch.tensor([m >> (s - com) for m, s in ms], dtype=torch.int32, device=acc.device)
    if acc.dtype != torch.int32 or acc.dim() != 2:
        return to_int8_sat(apply_mult_shift(acc.to(torch.int64), mults, com, stochastic))
    if stochastic:
        site = _requant_site(acc.shape, com, acc.device, True, "requant")
    else:
        _check_shift(com, False)
        site = _sr.Site(_native.sr_spec(_native.SR_NEAREST), None)
    return _ops.requant(acc, mults, com, site)


def i8_relu(x_i8: torch.Tensor) -> torch.Tensor:
    """ReLU on int8: integer clamp.  ilayer.py:73-76."""
    _check_int(x_i8, "relu input")
    return torch.clamp(x_i8, min=0)


class I8Linear(nn.Module):
    """Integer-only linear layer: int8 in -> int8 out, int32 accumulate (ilayer.py:79-170).

    ``headroom`` (default 4.0): the frozen grids cover ``headroom``x the init
    ranges so training does not slam into the +-127 rails.
    """

    def __init__(self, in_f: int, out_f: int, bias: bool = True, headroom: float = 4.0):
        super().__init__()
        assert headroom >= 1.0, "headroom must cover at least the init range"
        self.headroom = float(headroom)
        # float initialisation outside the strict region (ilayer.py:96-101)
        w_fp = torch.randn(out_f, in_f) * (2.0 / in_f) ** 0.5
        amax = w_fp.abs().amax(dim=1)
        sw = (amax / 127.0 * self.headroom).clamp_min(1e-8)
        w_i8 = torch.clamp(torch.round(w_fp / sw.unsqueeze(1)), -127, 127).to(torch.int8)
        self.register_buffer("w_i8", w_i8)
        self.sw = [float(v) for v in sw]  # plain floats, NOT a tensor
        self.register_buffer("b_acc", torch.zeros(out_f, dtype=torch.int32))
        self.use_bias = bias
        self.sx: float | None = None
        self.sy: float | None = None
        self._cache_x: torch.Tensor | None = None
        self._gw_i8 = None
        self._gw_rows = None  # (lo, hi) when the stashed gradient is this rank's row shard
        self._dw_pending = None
        self._fwd_cache = None
        self._sw_cache = None

    # Per-call bookkeeping attributes bypass nn.Module.__setattr__ (none is a
    # parameter, buffer or submodule; properties still apply).
    _PLAIN_ATTRS = frozenset({"_cache_x", "_dw_pending", "_dw_event", "_fwd_cache", "_gb_s", "_gb_sum",
                              "_gw_rows", "_gw_s", "_gw_i8", "_gw_sumsq", "_gw_sumsq_of", "_sw_cache",
                              "_input_gather", "_gather_works"})

    def __setattr__(self, name, value):
        if name in I8Linear._PLAIN_ATTRS:
            object.__setattr__(self, name, value)
        else:
            super().__setattr__(name, value)

    def __getstate__(self):
        """Module state for ``torch.save(model)`` (the reference's way to persist): the
        launch caches and in-flight exchange handles are dropped (rebuilt on use); device
        scales of a queued backward are stored as their float values."""
        ev = self.__dict__.get("_dw_event")
        if ev is not None:  # a queued backward's dW branch finishes before the tensors are copied
            self.__dict__["_dw_event"] = None
            torch.cuda.current_stream(self.w_i8.device).wait_event(ev)
        d = nn.Module.__getstate__(self) if hasattr(nn.Module, "__getstate__") else dict(self.__dict__)
        d = dict(d)
        for k in ("_fwd_cache", "_sw_cache", "_input_gather", "_gather_works", "_sw_mean_cache", "_dw_event"):
            d.pop(k, None)
        if d.get("_dw_pending") is not None:
            raise RuntimeError("a data-parallel dW reduction is in flight: read a gradient or call "
                               "ecoint8.parallel.synchronize() before saving")
        for k in ("_gw_s_store", "_gb_s_store"):
            if isinstance(d.get(k), _scale.DevScale):
                d[k] = d[k].value()
        d["_fwd_cache"] = None
        d["_sw_cache"] = None
        return d

    # Gradient stashes of the reference (ilayer.py:155-156, 168-169).  Under data
    # parallelism the dW reduction is still in flight when backward_i8 returns;
    # reading any of them completes every pending layer at once.
    def _grad_get(self, name):
        if self.__dict__.get("_dw_pending") is not None:
            parallel.finalize_pending()
        ev = self.__dict__.get("_dw_event")
        if ev is not None:  # a queued backward's dW branch: order the reader's stream after it
            self.__dict__["_dw_event"] = None
            torch.cuda.current_stream(self.w_i8.device).wait_event(ev)
        return self.__dict__.get(name + "_store")

    _gw_i8 = property(lambda self: self._grad_get("_gw_i8"),
                      lambda self, v: self.__dict__.__setitem__("_gw_i8_store", v))
    _gw_s = property(lambda self: _scale.as_float(self._grad_get("_gw_s")) if self._grad_get("_gw_s") is not None
                     else None,
                     lambda self, v: self.__dict__.__setitem__("_gw_s_store", v))
    # the bias gradient's scale (ilayer.py:169); a device scale while a queued backward runs
    _gb_s = property(lambda self: _scale.as_float(self.__dict__["_gb_s_store"])
                     if self.__dict__.get("_gb_s_store") is not None else None,
                     lambda self, v: self.__dict__.__setitem__("_gb_s_store", v))
    _gb_sum = property(lambda self: self._grad_get("_gb_sum"),
                       lambda self, v: self.__dict__.__setitem__("_gb_sum_store", v))

    # ``sw`` is a list of floats like the reference's; edits invalidate the device copies
    @property
    def sw(self) -> list[float]:
        return self.__dict__["_sw"]

    @sw.setter
    def sw(self, values) -> None:
        self.__dict__["_sw"] = values if isinstance(values, _ScaleList) else _ScaleList(values)

    @property
    def out_features(self) -> int:
        return self.w_i8.shape[0]

    def _sw_key(self):
        return id(self.sw), self.sw.version, len(self.sw)

    def _fwd_mults(self, device):
        """Per-channel multipliers and common shift of the frozen forward (ilayer.py:140, :66-68)."""
        key = (self.sx, self.sy, self._sw_key(), device)
        if self._fwd_cache is None or self._fwd_cache[0] != key:
            ratios = [(self.sx * sw) / self.sy for sw in self.sw]
            ms = [quantize_multiplier(r) for r in ratios]
            com = min(s for _, s in ms)
            mults = torch.tensor([m >> (s - com) for m, s in ms], dtype=torch.int32, device=device)
            self._fwd_cache = (key, mults, com)
        return self._fwd_cache[1], self._fwd_cache[2]

    def _sw_mean(self) -> float:
        """``sum(self.sw) / len(self.sw)`` (ilayer.py:160), cached until ``sw`` is edited."""
        key = self._sw_key()
        cached = self.__dict__.get("_sw_mean_cache")
        if cached is None or cached[0] != key:
            cached = (key, sum(self.sw) / len(self.sw))
            self.__dict__["_sw_mean_cache"] = cached
        return cached[1]

    def _sw_device(self, device):
        """``sw`` on the device as int64 bit patterns of the doubles, plus its min and max."""
        key = (self._sw_key(), device)
        if self._sw_cache is None or self._sw_cache[0] != key:
            import struct

            raw = struct.pack(f"<{len(self.sw)}d", *self.sw)
            bits = torch.frombuffer(bytearray(raw), dtype=torch.int64).to(device)
            self._sw_cache = (key, bits, min(self.sw), max(self.sw))
        return self._sw_cache[1], self._sw_cache[2], self._sw_cache[3]

    # -- calibration (once) -------------------------------------------------
    def calibrate_forward(self, x_i8: torch.Tensor, s_x: float) -> tuple[torch.Tensor, float]:
        """First-and-only dynamic pass: freeze ``sx``/``sy`` (ilayer.py:113-123)."""
        _check_int(x_i8, "calibration input")
        self.sx = float(s_x)
        _native.require_cuda(x_i8, self.w_i8)
        N, K = x_i8.shape
        amax = torch.empty(1, dtype=torch.int32, device=x_i8.device)
        acc = _ops.gemm_s32(x_i8, 0, self.w_i8, 0, N, self.out_features, K,
                            bias=self.b_acc if self.use_bias else None, amax=amax)
        acc_amax = int(amax.item())
        if parallel.active():
            acc_amax = parallel.allreduce_max_int(acc_amax)
        gain = self.sx * max(self.sw)
        self.sy = dynamic_scale_from_int(acc_amax, gain) * self.headroom
        ratios = [(self.sx * sw) / self.sy for sw in self.sw]
        return _common_shift_requant(acc, ratios, stochastic=True), self.sy

    def set_bias_acc(self, b_acc: torch.Tensor) -> None:
        """Install a bias already quantized to the acc domain (int32)."""
        _check_int(b_acc, "bias acc")
        self.b_acc.copy_(b_acc)

    # -- static forward / explicit backward ---------------------------------
    def forward_i8(self, x_i8: torch.Tensor, _relu: bool = False) -> tuple[torch.Tensor, float]:
        """Static integer forward (ilayer.py:131-141): one fused GEMM + requant kernel."""
        assert self.sx is not None and self.sy is not None, "calibrate first"
        _check_int(x_i8, "layer input")
        _native.require_cuda(x_i8, self.w_i8)
        assert isinstance(self.sx, float) and isinstance(self.sy, float)
        if parallel.peer_bufs(self, x_i8.shape[0]) is not None:
            parallel.peer_forward(self, x_i8)  # weight rows in, input rows out ("peer" exchange)
        else:
            parallel.wait_gathers(self)
            if parallel.gathers_input(self):
                parallel.gather_input(self, x_i8)  # the global-batch input of this layer's dW ("gather" exchange)
        mults, com = self._fwd_mults(x_i8.device)
        N, K = x_i8.shape
        out = self.out_features
        site = _requant_site((N, out), com, x_i8.device, True, "forward")
        y = _ops.gemm_requant(x_i8, 0, self.w_i8, 0, N, out, K, self.b_acc if self.use_bias else None, mults, com,
                              _relu, site)
        self._cache_x = x_i8
        return y, self.sy

    def backward_i8(self, g_i8: torch.Tensor, s_g: float, _mask: torch.Tensor | None = None
                    ) -> tuple[torch.Tensor, float]:
        """Integer backward (ilayer.py:143-170).  Returns ``(dx_i8, s_dx)``; stashes
        ``_gw_i8``/``_gw_s`` and ``_gb_sum``/``_gb_s``.  ``_mask`` (internal): zero the
        rows/cols of dX where it is <= 0 (the preceding ReLU's mask)."""
        _check_int(g_i8, "grad output")
        assert self._cache_x is not None, "call forward_i8 before backward_i8"
        x_i8 = self._cache_x
        assert isinstance(self.sx, float)
        s_x = self.sx
        s_g = _scale.as_float(s_g)  # a device scale (the fused loss boundary's) is read here
        dev = _native.require_cuda(g_i8, x_i8, self.w_i8)
        N, out = g_i8.shape
        in_f = x_i8.shape[1]
        if parallel.active():
            return self._backward_dp(g_i8, float(s_g), x_i8, _mask, dev)
        amax = torch.empty(2, dtype=torch.int32, device=dev)
        # dX first: its maximum gates the next layer, and the host reads it while the dW GEMM runs
        # dX = g w: A = g [M=N, K=out], B = w stored [K=out, N=in]
        dx_acc = _ops.gemm_s32(g_i8, 0, self.w_i8, 1, N, in_f, out, amax=amax[1:2])
        rd_dx = _ops.read_later(amax[1:2])
        # dW = g^T x: A = g stored [K=N, M=out], B = x stored [K=N, N=in]
        dw_acc = _ops.gemm_s32(g_i8, 1, x_i8, 1, out, in_f, N, amax=amax[0:1])
        rd_dw = _ops.read_later(amax[0:1])
        self._gb_sum = _ops.colsum(g_i8)  # dBias: integer column sums (torch's int32 .sum(0) is int64)
        self._gb_s = float(s_g)
        key_w = _sr.reserve_key()  # the dW site's key, in the reference's draw order

        def requant_dw(a_dw):
            # dW: exact scales (both per-tensor) -> int8 grad for the optimizer
            s_gw = dynamic_scale_from_int(a_dw, s_g * s_x)
            m_gw, sh_gw = quantize_multiplier((s_g * s_x) / s_gw)
            if key_w is not None:
                _check_shift(sh_gw, True)
                site = _sr.site_from_key(key_w, (out, in_f), sh_gw, 0, "dw")
            else:
                site = _requant_site((out, in_f), sh_gw, dev, False, "dw")
            self._gw_sumsq = torch.empty(1, dtype=torch.int64, device=dev)
            self._gw_i8 = _ops.requant(dw_acc, m_gw, sh_gw, site, sumsq=self._gw_sumsq)
            self._gw_sumsq_of = self._gw_i8
            self._gw_s = s_gw
            self._gw_rows = None

        def requant_dx(a_dx):
            # dX: per-channel s_w approximated by its mean
            sw_mean = self._sw_mean()
            s_dx = dynamic_scale_from_int(a_dx, s_g * sw_mean)
            m_dx, sh_dx = quantize_multiplier((s_g * sw_mean) / s_dx)
            site = _requant_site((N, in_f), sh_dx, dev, True, "dx")
            return _ops.requant(dx_acc, m_dx, sh_dx, site, mask=_mask), s_dx

        if key_w is None:  # replay: the dW site draws first, and its draw needs the dW shift
            requant_dw(rd_dw.value()[0])
            return requant_dx(rd_dx.value()[0])
        dx_i8, s_dx = requant_dx(rd_dx.value()[0])  # queued behind the dW GEMM: no idle gap
        requant_dw(rd_dw.value()[0])
        return dx_i8, s_dx

    def _backward_queued(self, g_i8: torch.Tensor, s_g, _mask: torch.Tensor | None = None):
        """``backward_i8`` for a pass queued without host round trips (Philox mode):
        ``s_g`` is a float or a device scale, the dX and dW scales are computed on the
        device (``_scale``) and the returned ``s_dx`` is a device scale.  Same keys,
        draws and results as ``backward_i8``."""
        _check_int(g_i8, "grad output")
        assert self._cache_x is not None, "call forward_i8 before backward_i8"
        x_i8 = self._cache_x
        assert isinstance(self.sx, float)
        dev = _native.require_cuda(g_i8, x_i8, self.w_i8)
        N, out = g_i8.shape
        in_f = x_i8.shape[1]
        if parallel.active():
            return self._backward_dp(g_i8, s_g, x_i8, _mask, dev, queued=True)
        # The dW branch (GEMM, bias column sums, scale, requant) runs on a side stream forked
        # here: nothing of the dX chain waits for it, and its memory-bound kernels share the
        # SMs with the next layer's dX GEMM.  The optimizer (any read of the stashed
        # gradient) joins it through ``_dw_event``.
        cur = torch.cuda.current_stream(dev)
        side = _dw_stream(dev)
        side.wait_stream(cur)
        key_w = _sr.reserve_key()  # the dW site's key, then the dX site's (the reference's order)
        with torch.cuda.stream(side):
            amax_w = torch.empty(1, dtype=torch.int32, device=dev)
            dw_acc = _ops.gemm_s32(g_i8, 1, x_i8, 1, out, in_f, N, amax=amax_w)
            gb_sum = _ops.colsum(g_i8)
            s_gw = _scale.from_amax(amax_w, s_g, self.sx)
            gw_sumsq = torch.empty(1, dtype=torch.int64, device=dev)
            gw_i8 = _ops.requant_dev(dw_acc, s_gw, key_w, 0, sumsq=gw_sumsq)
            done = torch.cuda.Event()
            done.record(side)
        g_i8.record_stream(side)  # the main stream may free these while the side stream reads them
        x_i8.record_stream(side)
        from .. import graphs

        g = graphs.capturing()
        if g is not None:
            g.join(side)
        amax_x = torch.empty(1, dtype=torch.int32, device=dev)
        dx_acc = _ops.gemm_s32(g_i8, 0, self.w_i8, 1, N, in_f, out, amax=amax_x)
        s_dx = _scale.from_amax(amax_x, s_g, self._sw_mean())
        dx_i8 = _ops.requant_dev(dx_acc, s_dx, _sr.new_key(), _sr.row_base(), mask=_mask)
        self._gb_sum = gb_sum
        self._gb_s = s_g
        self._gw_sumsq = gw_sumsq
        self._gw_i8 = gw_i8
        self._gw_sumsq_of = gw_i8
        self._gw_s = s_gw
        self._gw_rows = None
        self._dw_event = done
        return dx_i8, s_dx

    def _backward_dp(self, g_i8, s_g, x_i8, mask, dev, queued: bool = False):
        """Data-parallel backward: dW rows formed asynchronously (reduce-scatter of the
        int32 accumulators, or one GEMM over the gathered global batch) and finalized
        when the gradient is read; global dX maximum over ranks; dX requant.  Same
        draws and results as the single-device backward on the concatenated batch."""
        N, out = g_i8.shape
        in_f = x_i8.shape[1]
        peer = parallel.peer_bufs(self) is not None
        gathered = self.__dict__.get("_input_gather") is not None
        if peer:  # dY columns out, then the dW GEMM on the exchange's stream once all have arrived
            parallel.start_dw_rows_peer(self, g_i8, s_g)
        elif gathered:
            dy_cols, a2a = parallel.exchange_grad_columns(g_i8)
        else:
            dw_acc = _ops.gemm_s32(g_i8, 1, x_i8, 1, out, in_f, N)
            gb_sum = _ops.colsum(g_i8)
        key_w = _sr.reserve_key()  # the dW site's key, in the reference's draw order
        if peer:
            self._dw_pending["key"] = key_w
        elif not gathered:
            parallel.start_dw_reduction(self, dw_acc, gb_sum, s_g)
            self._dw_pending["key"] = key_w
        self._gb_s = s_g
        amax_dx = torch.empty(1, dtype=torch.int32, device=dev)
        dx_acc = _ops.gemm_s32(g_i8, 0, self.w_i8, 1, N, in_f, out, amax=amax_dx)
        t, work = parallel.start_max(amax_dx)
        if queued:  # the dX scale from the global maximum, on the device
            if gathered:
                parallel.start_dw_rows(self, dy_cols, a2a, s_g)
                self._dw_pending["key"] = key_w
            self._dw_pending["queued"] = True
            work.wait()
            s_dx = _scale.from_amax(t, s_g, self._sw_mean())
            return _ops.requant_dev(dx_acc, s_dx, _sr.new_key(), _sr.row_base(), mask=mask), s_dx
        rd_dx = _ops.read_later(t, work)
        if gathered:  # the dW GEMM runs while the host waits for the dX maximum
            parallel.start_dw_rows(self, dy_cols, a2a, s_g)
            self._dw_pending["key"] = key_w
        if key_w is None:  # replay mode draws in order: finish this layer's dW now
            parallel.finalize_pending()
        a_dx = rd_dx.value()[0]
        sw_mean = self._sw_mean()
        s_dx = dynamic_scale_from_int(a_dx, s_g * sw_mean)
        m_dx, sh_dx = quantize_multiplier((s_g * sw_mean) / s_dx)
        site = _requant_site((N, in_f), sh_dx, dev, True, "dx")
        dx_i8 = _ops.requant(dx_acc, m_dx, sh_dx, site, mask=mask)
        return dx_i8, s_dx

    def _finalize_dw_queued(self, amax: torch.Tensor, sumsq_out: torch.Tensor) -> None:
        """``_finalize_dw`` with the global maximum on the device (a queued backward)."""
        p = self.__dict__["_dw_pending"]
        self._dw_pending = None
        s_gw = _scale.from_amax(amax, p["s_g"], self.sx)
        rows = p["rows"]
        self._gw_i8 = _ops.requant_dev(p["red"], s_gw, p["key"], 0 if rows is None else rows[0], sumsq=sumsq_out)
        self._gw_s = s_gw
        self._gw_rows = rows
        self._gb_sum = p["gb"]

    def _finalize_dw(self, a_dw: int, sumsq_out: torch.Tensor) -> None:
        """Requantize this rank's rows of the summed dW with the global maximum."""
        p = self.__dict__["_dw_pending"]
        self._dw_pending = None
        s_g, s_x = p["s_g"], self.sx
        out, in_f = p["shape"]
        s_gw = dynamic_scale_from_int(a_dw, s_g * s_x)
        m_gw, sh_gw = quantize_multiplier((s_g * s_x) / s_gw)
        _check_shift(sh_gw, True)
        rows = p["rows"]
        lo = 0 if rows is None else rows[0]
        if p.get("key") is not None:
            site = _sr.site_from_key(p["key"], (out, in_f), sh_gw, lo, "dw")
        else:
            site = _sr.draw((out, in_f), sh_gw, p["red"].device, batch=False, kind="dw")
            if site.nudge is not None and rows is not None:
                site.nudge = site.nudge[rows[0]:rows[1]].contiguous()
                site.spec.nudge = site.nudge.data_ptr()
        self._gw_i8 = _ops.requant(p["red"], m_gw, sh_gw, site, sumsq=sumsq_out)
        self._gw_s = s_gw
        self._gw_rows = rows
        self._gb_sum = p["gb"]


_DW_STREAMS: dict = {}


def _dw_stream(dev: torch.device) -> torch.cuda.Stream:
    """The side stream of the single-device queued backward's dW branches (one per device)."""
    st = _DW_STREAMS.get(dev.index)
    if st is None:
        st = _DW_STREAMS[dev.index] = torch.cuda.Stream(dev)
    return st


class I8ReLU(nn.Module):
    """ReLU block for I8Sequential with integer mask caching (ilayer.py:173-188).

    Inside ``I8Sequential`` the clamp runs in the preceding layer's GEMM
    epilogue and the mask is its output's sign, materialised only if read.
    """

    def __setattr__(self, name, value):
        if name in ("_mask", "_relu_out"):  # bookkeeping, not parameters or buffers
            object.__setattr__(self, name, value)
        else:
            super().__setattr__(name, value)

    def __init__(self):
        super().__init__()
        self._mask = None
        self._relu_out = None

    @property
    def mask_cache(self) -> torch.Tensor | None:
        if self._mask is None and self._relu_out is not None:
            self._mask = (self._relu_out > 0).to(torch.int8)
        return self._mask

    @mask_cache.setter
    def mask_cache(self, value) -> None:
        self._mask = value
        self._relu_out = None

    def _mask_source(self) -> torch.Tensor | None:
        return self._relu_out if self._relu_out is not None else self._mask

    def _fused_output(self, y: torch.Tensor) -> None:
        self._relu_out = y
        self._mask = None

    def apply_forward(self, x_i8: torch.Tensor) -> torch.Tensor:
        self.mask_cache = (x_i8 > 0).to(torch.int8)
        return i8_relu(x_i8)

    def backward_mask(self, g_i8: torch.Tensor) -> torch.Tensor:
        _check_int(g_i8, "relu grad")
        mask = self.mask_cache
        assert mask is not None
        gm = g_i8.to(torch.int32) * mask.to(torch.int32)
        return torch.clamp(gm, -127, 127).to(torch.int8)


class I8Sequential(nn.Module):
    """Manual int8 pipeline: threads int8 tensors + scalar scales, explicit backward (ilayer.py:191-245)."""

    def __init__(self, *blocks: nn.Module):
        super().__init__()
        self.blocks = nn.ModuleList(blocks)

    def int8_layers(self) -> list[I8Linear]:
        return [b for b in self.blocks if isinstance(b, I8Linear)]

    def quantize_input(self, x_fp: torch.Tensor) -> tuple[torch.Tensor, float]:
        """Quantize a float batch onto the FROZEN entry scale (ilayer.py:201-213)."""
        first = self.int8_layers()[0]
        assert first.sx is not None, "calibrate first"
        s = float(first.sx)
        return torch.clamp(torch.round(x_fp / s), -127, 127).to(torch.int8), s

    def calibrate(self, x_i8: torch.Tensor, s_x: float) -> tuple[torch.Tensor, float]:
        """One dynamic pass that freezes every layer's scales (ilayer.py:215-224)."""
        _check_int(x_i8, "calibration input")
        s = float(s_x)
        for blk in self.blocks:
            if isinstance(blk, I8Linear):
                x_i8, s = blk.calibrate_forward(x_i8, s)
            elif isinstance(blk, I8ReLU):
                x_i8 = blk.apply_forward(x_i8)
        return x_i8, s

    def forward_i8(self, x_i8: torch.Tensor) -> tuple[torch.Tensor, float]:
        """Static integer forward (ilayer.py:226-236); Linear+ReLU pairs run as one kernel."""
        _check_int(x_i8, "net input")
        s: float | None = None
        blocks = list(self.blocks)
        i = 0
        while i < len(blocks):
            blk = blocks[i]
            if isinstance(blk, I8Linear):
                nxt = blocks[i + 1] if i + 1 < len(blocks) else None
                if isinstance(nxt, I8ReLU):
                    x_i8, s = blk.forward_i8(x_i8, _relu=True)
                    nxt._fused_output(x_i8)
                    i += 2
                    continue
                x_i8, s = blk.forward_i8(x_i8)
            elif isinstance(blk, I8ReLU):
                x_i8 = blk.apply_forward(x_i8)
            i += 1
        assert s is not None
        return x_i8, s

    def backward_i8(self, g_i8: torch.Tensor, s_g: float) -> None:
        """Explicit reverse pass (ilayer.py:238-245); a ReLU mask rides in the dX requant."""
        _check_int(g_i8, "net grad")
        blocks = list(self.blocks)
        # Philox mode queues the whole pass: scales stay on the device between layers
        # (the per-layer site log and the replay mode need host shifts: layer by layer)
        queued = not _sr.replaying() and _sr.LOG is None and g_i8.is_cuda
        i = len(blocks) - 1
        while i >= 0:
            blk = blocks[i]
            if isinstance(blk, I8Linear):
                step = blk._backward_queued if queued else blk.backward_i8
                prev = blocks[i - 1] if i > 0 else None
                if isinstance(prev, I8ReLU) and prev._mask_source() is not None:
                    g_i8, s_g = step(g_i8, s_g, _mask=prev._mask_source())
                    i -= 2
                    continue
                g_i8, s_g = step(g_i8, s_g)
            elif isinstance(blk, I8ReLU):
                g_i8 = blk.backward_mask(g_i8)
            i -= 1
