"""Strict int8 layers and the integer ECO optimizer, restated in numpy (oracle; test only).

Follows ``ecoint8/strict/ilayer.py`` and ``ecoint8/strict/iopt.py`` of the
reference.  Stochastic-rounding draws come from a ``draw(shape, denom)``
callable, called in exactly the order the reference calls ``_sr_nudge``:

* ``TorchDraws`` replays the reference's own stream (``torch.randint`` on the
  global CPU generator, ``fixedpoint.py:40-49``), so a seeded run of this
  oracle reproduces a seeded run of the reference bit for bit;
* ``ListDraws`` replays recorded arrays;
* ``RecordingDraws`` wraps another source and keeps what it handed out, so the
  same nudges can be fed to the CUDA kernels in their replay mode.
"""

from __future__ import annotations

import math

import numpy as np

from .fixedpoint import (
    add64,
    apply_mult_shift,
    col_mults,
    dynamic_scale_from_int,
    int_amax,
    int_mm,
    mul64,
    quantize_multiplier,
    sar64,
    shl64,
    sub64,
    to_int8_sat,
)

FRAC_BITS = 12  # iopt.py:37
BETA_Q = 1 << 16  # iopt.py:38
LR_Q = 1 << 16  # iopt.py:39


class TorchDraws:
    """The reference's draw stream: ``torch.randint(0, denom, shape)`` (fixedpoint.py:48-49)."""

    def __call__(self, shape, denom):
        import torch

        dt = torch.int32 if denom <= (1 << 31) else torch.int64
        return torch.randint(0, denom, tuple(shape), dtype=dt).numpy().astype(np.int64)


class ListDraws:
    def __init__(self, arrays):
        self.arrays = list(arrays)
        self.pos = 0

    def __call__(self, shape, denom):
        a = np.asarray(self.arrays[self.pos]).astype(np.int64)
        self.pos += 1
        assert tuple(a.shape) == tuple(shape), (a.shape, shape)
        assert a.min(initial=0) >= 0 and a.max(initial=0) < denom
        return a


class RecordingDraws:
    def __init__(self, inner):
        self.inner = inner
        self.log: list[tuple[tuple, int, np.ndarray]] = []

    def __call__(self, shape, denom):
        a = self.inner(shape, denom)
        self.log.append((tuple(shape), denom, a))
        return a


def _sr(x, mult, shift, draw, shape):
    """``apply_mult_shift(x, mult, shift, stochastic=True)`` with a draw when ``shift >= 0``."""
    nudge = draw(shape, 1 << shift) if shift >= 0 else None
    return apply_mult_shift(x, mult, shift, True, nudge)


def common_shift_requant(acc, ratios, draw) -> np.ndarray:
    """ilayer.py:57-70 (always stochastic at every call site of the reference)."""
    mults, com = col_mults(ratios)
    y64 = _sr(acc.astype(np.int64), mults, com, draw, acc.shape)
    return to_int8_sat(y64)


def init_params(in_f: int, out_f: int, headroom: float = 4.0):
    """ilayer.py:96-101: float init outside the strict region (uses torch's CPU stream)."""
    import torch

    w_fp = torch.randn(out_f, in_f) * (2.0 / in_f) ** 0.5
    amax = w_fp.abs().amax(dim=1)
    sw = (amax / 127.0 * float(headroom)).clamp_min(1e-8)
    w_i8 = torch.clamp(torch.round(w_fp / sw.unsqueeze(1)), -127, 127).to(torch.int8)
    return w_i8.numpy().copy(), [float(v) for v in sw]


class I8Linear:
    """ilayer.py:79-170."""

    def __init__(self, w_i8: np.ndarray, sw: list[float], headroom: float = 4.0,
                 bias: bool = True, b_acc: np.ndarray | None = None):
        self.w_i8 = np.array(w_i8, dtype=np.int8)
        self.sw = [float(v) for v in sw]
        self.headroom = float(headroom)
        self.use_bias = bias
        out_f = self.w_i8.shape[0]
        self.b_acc = (np.zeros(out_f, dtype=np.int32) if b_acc is None
                      else np.array(b_acc, dtype=np.int32))
        self.sx: float | None = None
        self.sy: float | None = None
        self._cache_x = None
        self._gw_i8 = None
        self._gw_s = None
        self._gb_sum = None
        self._gb_s = None

    @classmethod
    def seeded(cls, in_f, out_f, headroom=4.0, bias=True):
        w, sw = init_params(in_f, out_f, headroom)
        return cls(w, sw, headroom, bias)

    def _acc(self, x_i8):
        acc = int_mm(x_i8, self.w_i8.T)
        if self.use_bias:
            with np.errstate(over="ignore"):
                acc = (acc.astype(np.int64) + self.b_acc.astype(np.int64)).astype(np.int32)
        return acc

    def calibrate_forward(self, x_i8, s_x, draw):
        """ilayer.py:113-123."""
        self.sx = float(s_x)
        acc = self._acc(x_i8)
        gain = self.sx * max(self.sw)
        self.sy = dynamic_scale_from_int(int_amax(acc), gain) * self.headroom
        ratios = [(self.sx * sw) / self.sy for sw in self.sw]
        return common_shift_requant(acc, ratios, draw), self.sy

    def forward_i8(self, x_i8, draw):
        """ilayer.py:131-141."""
        acc = self._acc(x_i8)
        self._cache_x = np.asarray(x_i8, dtype=np.int8)
        ratios = [(self.sx * sw) / self.sy for sw in self.sw]
        return common_shift_requant(acc, ratios, draw), self.sy

    def backward_i8(self, g_i8, s_g, draw):
        """ilayer.py:143-170."""
        g_i8 = np.asarray(g_i8, dtype=np.int8)
        x_i8 = self._cache_x
        s_x = self.sx
        dw_acc = int_mm(g_i8.T, x_i8)
        s_gw = dynamic_scale_from_int(int_amax(dw_acc), s_g * s_x)
        m_gw, sh_gw = quantize_multiplier((s_g * s_x) / s_gw)
        self._gw_i8 = to_int8_sat(_sr(dw_acc.astype(np.int64), m_gw, sh_gw, draw, dw_acc.shape))
        self._gw_s = s_gw
        dx_acc = int_mm(g_i8, self.w_i8)
        sw_mean = sum(self.sw) / len(self.sw)
        s_dx = dynamic_scale_from_int(int_amax(dx_acc), s_g * sw_mean)
        m_dx, sh_dx = quantize_multiplier((s_g * sw_mean) / s_dx)
        dx_i8 = to_int8_sat(_sr(dx_acc.astype(np.int64), m_dx, sh_dx, draw, dx_acc.shape))
        # torch.sum of an int32 tensor accumulates and returns int64 (ilayer.py:168)
        self._gb_sum = g_i8.astype(np.int64).sum(axis=0)
        self._gb_s = float(s_g)
        return dx_i8, s_dx


class I8ReLU:
    """ilayer.py:173-188."""

    def __init__(self):
        self.mask_cache = None

    def apply_forward(self, x_i8):
        x_i8 = np.asarray(x_i8, dtype=np.int8)
        self.mask_cache = (x_i8 > 0).astype(np.int8)
        return np.maximum(x_i8, 0).astype(np.int8)

    def backward_mask(self, g_i8):
        gm = np.asarray(g_i8).astype(np.int32) * self.mask_cache.astype(np.int32)
        return np.clip(gm, -127, 127).astype(np.int8)


class I8Sequential:
    """ilayer.py:191-245."""

    def __init__(self, *blocks):
        self.blocks = list(blocks)

    def int8_layers(self):
        return [b for b in self.blocks if isinstance(b, I8Linear)]

    def calibrate(self, x_i8, s_x, draw):
        s = float(s_x)
        for blk in self.blocks:
            if isinstance(blk, I8Linear):
                x_i8, s = blk.calibrate_forward(x_i8, s, draw)
            else:
                x_i8 = blk.apply_forward(x_i8)
        return x_i8, s

    def forward_i8(self, x_i8, draw):
        s = None
        for blk in self.blocks:
            if isinstance(blk, I8Linear):
                x_i8, s = blk.forward_i8(x_i8, draw)
            else:
                x_i8 = blk.apply_forward(x_i8)
        return x_i8, s

    def backward_i8(self, g_i8, s_g, draw):
        for blk in reversed(self.blocks):
            if isinstance(blk, I8Linear):
                g_i8, s_g = blk.backward_i8(g_i8, s_g, draw)
            else:
                g_i8 = blk.backward_mask(g_i8)


def fixed_point_consts(lr: float, beta: float):
    """iopt.py:105-110: (b_q, nb_q, lr_q, a_q) with Python's half-to-even round."""
    alpha = (1.0 / lr) * (1.0 - 1.0 / beta)
    return (round(beta * BETA_Q), round((1.0 - beta) * BETA_Q), round(lr * LR_Q),
            round(alpha * BETA_Q))


def eco_rows(w, m, g, mults_m, com_m, mults_g, com_g, b_q, nb_q, lr_q, a_q, nudge_w):
    """Per-element body of iopt.py:154-170 on a block of rows.

    Returns ``(w_new int64, m_new int64, eU int64)``.  ``mults_*`` are ``[rows, 1]``.
    """
    F = FRAC_BITS
    mU = apply_mult_shift(m.astype(np.int64), mults_m, com_m, False)
    gU = apply_mult_shift(g.astype(np.int64), mults_g, com_g, False)
    m_t = sar64(add64(mul64(mU, b_q), mul64(gU, nb_q)), 16)
    thU = sub64(shl64(w.astype(np.int64), F), sar64(mul64(m_t, lr_q), 16))
    w_new = np.clip(sar64(add64(thU, nudge_w), F), -127, 127)
    eU = sub64(thU, shl64(w_new, F))
    m_new = add64(m_t, sar64(mul64(eU, a_q), 16))
    return w_new, m_new, eU


class I8ECO:
    """iopt.py:57-209, with the chunked draw order of iopt.py:152-176."""

    def __init__(self, layers, lr=0.5, momentum=0.9, grad_clip=1.0, chunk_rows=64):
        assert momentum > 0
        assert 0.0 < lr < 2.0
        self.layers = list(layers)
        self.lr = float(lr)
        self.beta = float(momentum)
        self.grad_clip = grad_clip
        self.chunk_rows = int(chunk_rows)
        self.m_i8 = [np.zeros_like(layer.w_i8) for layer in self.layers]
        self.s_m = [1.0 for _ in self.layers]
        self.step_count = 0
        self.stats = {"skipped": 0, "mean_abs_e": 0.0}
        self.last_rowmax: list = []
        self.last_rowsum: list = []

    def set_lr(self, lr):
        assert 0.0 < lr < 2.0
        self.lr = float(lr)

    def clip_grad(self, g_i8, s_g):
        """iopt.py:90-101."""
        if self.grad_clip is None:
            return g_i8, s_g
        sq_sum = int((g_i8.astype(np.int64) ** 2).sum())
        n_real = math.sqrt(sq_sum) * s_g
        if n_real > self.grad_clip:
            return g_i8, s_g * (self.grad_clip / n_real)
        return g_i8, s_g

    def layer_mults(self, i, s_g):
        """The three per-row multiplier columns of iopt.py:134-148."""
        F = FRAC_BITS
        s_m = self.s_m[i]
        sw = self.layers[i].sw
        mm, cm = col_mults([s_m * (1 << F) / sw_o for sw_o in sw])
        mg, cg = col_mults([s_g * (1 << F) / sw_o for sw_o in sw])
        mmm, cmm = col_mults([(sw_o / (1 << F)) / s_m if s_m > 0 else 0.0 for sw_o in sw])
        return (mm[:, None], cm), (mg[:, None], cg), (mmm[:, None], cmm)

    def step(self, draw=None, nudges=None, philox=None):
        """iopt.py:103-200.

        Either ``draw`` (consumed in the reference's chunk order), ``nudges``: a
        list with one ``(nudge_w [out,in], nudge_m [out,in] | None, nudge_b
        [out,1] | None)`` per layer, consumed whole (the CUDA single-pass order),
        or ``philox=(seed, {layer: (stream_w, stream_b)})``: the CUDA library's
        Philox stream (``oracle/philox.py:step_nudges``).
        """
        if philox is not None:
            nudges = self._philox_nudges(*philox)
        F = FRAC_BITS
        b_q, nb_q, lr_q, a_q = fixed_point_consts(self.lr, self.beta)
        self.step_count += 1
        tot_e, n_e = 0.0, 0
        self.last_rowmax, self.last_rowsum = [], []
        for i, layer in enumerate(self.layers):
            g_i8 = layer._gw_i8
            if g_i8 is None:
                continue
            s_g = float(layer._gw_s)
            g_i8, s_g = self.clip_grad(g_i8, s_g)
            sw = layer.sw
            out, rowlen = g_i8.shape
            (mm, cm), (mg, cg), (mmm, cmm) = self.layer_mults(i, s_g)
            w, m = layer.w_i8, self.m_i8[i]
            rowmax_all: list[int] = []
            rowsum_all: list[int] = []
            chunk = self.chunk_rows if nudges is None else out
            for c in range(0, out, chunk):
                sl = slice(c, min(c + chunk, out))
                nrows = sl.stop - sl.start
                if nudges is None:
                    nw = draw((nrows, rowlen), 1 << F)
                else:
                    nw = nudges[i][0]
                w_new, m_new, eU = eco_rows(w[sl], m[sl], g_i8[sl], mm[sl], cm, mg[sl], cg,
                                            b_q, nb_q, lr_q, a_q, nw)
                rowmax_all.extend(np.abs(m_new).max(axis=1).tolist())
                with np.errstate(over="ignore"):
                    rowsum_all.extend(np.abs(eU).sum(axis=1).tolist())
                w[sl] = w_new.astype(np.int8)
                if cmm >= 0:
                    nm = draw((nrows, rowlen), 1 << cmm) if nudges is None else nudges[i][1]
                else:
                    nm = None
                m[sl] = to_int8_sat(apply_mult_shift(m_new, mmm[sl], cmm, True, nm))
            amax_real = max(r * sw_o / (1 << F) for r, sw_o in zip(rowmax_all, sw))
            self.s_m[i] = amax_real / 127.0 if amax_real > 0 else 1.0
            tot_e += sum(s * sw_o for s, sw_o in zip(rowsum_all, sw)) / rowlen / (1 << F)
            n_e += out
            self.last_rowmax.append(rowmax_all)
            self.last_rowsum.append(rowsum_all)
            if layer.use_bias:
                gb = np.asarray(layer._gb_sum).astype(np.int64)
                s_gb = float(layer._gb_s)
                mb, cb = col_mults([self.lr * s_gb / (layer.sx * sw_o) for sw_o in sw])
                if cb >= 0:
                    nb = draw((out, 1), 1 << cb) if nudges is None else nudges[i][2]
                else:
                    nb = None
                delta = apply_mult_shift(gb[:, None], mb[:, None], cb, True, nb)
                with np.errstate(over="ignore"):
                    layer.b_acc = (layer.b_acc.astype(np.int64)
                                   - delta[:, 0].astype(np.int32).astype(np.int64)).astype(np.int32)
        if n_e:
            self.stats["mean_abs_e"] = tot_e / n_e

    def _philox_nudges(self, seed, streams):
        """Whole-layer nudges of the Philox stream, with this step's shifts."""
        from . import philox as ph

        res = []
        for i, layer in enumerate(self.layers):
            if layer._gw_i8 is None or i not in streams:
                res.append(None)
                continue
            s_g = float(layer._gw_s)
            _, s_g = self.clip_grad(layer._gw_i8, s_g)
            (_, _), (_, _), (_, cmm) = self.layer_mults(i, s_g)
            out, cols = layer._gw_i8.shape
            sw_, sb_ = streams[i]
            nw, nm = ph.step_nudges(seed, sw_, out, cols, cmm)
            nb = None
            if layer.use_bias:
                _, cb = col_mults([self.lr * float(layer._gb_s) / (layer.sx * sw_o) for sw_o in layer.sw])
                if cb >= 0:
                    r = np.arange(out, dtype=np.uint64)[:, None]
                    nb = ph.low_bits(ph.sr_word(seed, sb_, r, np.zeros_like(r)), cb)
            res.append((nw, nm, nb))
        return res

    def zero_grad(self):
        for layer in self.layers:
            layer._gw_i8 = None
