"""ECO optimizers without master weights (API of ``ecoint8/eco.py`` v0.4.9).

``EcoInt8SGDM`` -- int8 weights, int8 momentum, fp32 only as a transient -- runs
its step as the library's fused CUDA kernels (``triton_eco_step_`` seam,
eco.py:330-362).  There is one backend: ``backend`` is accepted for
compatibility; ``"auto"``, ``"triton"`` and ``"cuda"`` select the fused CUDA
step and ``"torch"`` (the reference's eager fallback) raises, as does any
layer that is not on an sm_100 GPU.

``EcoSGDM`` and ``EcoAdam`` (fp32 optimizer state) run their weight steps as the
library's fused two-launch kernel pair for all layers (``eco_fp32_eco_step``).
"""

from __future__ import annotations

import ctypes
import random

import torch

from .quant import EPS  # noqa: F401  (re-exported like the reference)

__all__ = ["EcoSGDM", "EcoAdam", "EcoInt8SGDM"]

TILE = 64 * 1024  # elements per tile of eco_fp32_eco_step's statistics


def _get_grad_w(layer) -> torch.Tensor | None:
    """The stashed fp32 weight gradient, or None if absent / non-finite (eco.py:39-47)."""
    g = layer._grad_w
    if g is None:
        return None
    g = g.clone()
    if not torch.isfinite(g).all():
        return None
    return g


class _FusedFp32:
    """The fused step shared by EcoSGDM and EcoAdam: every layer with a gradient in two
    launches (``eco_fp32_eco_step``), no host synchronisation; ``stats`` is read from the
    device when accessed.

    Rounding: the library's Philox stream (a fresh key per step from ``ecoint8._sr``), or,
    inside ``ecoint8.sr_replay()``, one ``torch.rand_like`` draw per stepped layer on its
    device, in layer order -- the draws the reference's ``quantize_symmetric`` makes, which
    makes the step bit for bit the reference's PyTorch arithmetic on that device.  The
    gradient norm is computed in double and rounded to fp32; PyTorch's fp32 ``g.norm()`` can
    differ from it in the last bit, which matters only when clipping is active."""

    _KIND = 0

    def _fused_step(self, hyper_fn) -> None:
        from . import _native as nat
        from . import _sr

        active = [(i, layer) for i, layer in enumerate(self.layers) if layer._grad_w is not None]
        self._pending = None
        if not active:
            return
        dev = nat.require_cuda(*[layer.w_i8 for _, layer in active])
        replay = _sr.replaying()
        descs, keep, stepped_layers = [], [], []
        n = len(active)
        if getattr(self, "_flags_dev", None) is None or self._flags_dev[0].numel() < len(self.layers):
            self._flags_dev = (torch.zeros(len(self.layers), dtype=torch.float32, device=dev),
                               torch.zeros(len(self.layers), dtype=torch.int32, device=dev))
        norms, stepped = self._flags_dev
        for i, layer in active:
            w = layer.w_i8
            if not (w.is_cuda and w.dtype == torch.int8 and w.is_contiguous()):
                raise RuntimeError("Eco optimizers (B200 build): int8 contiguous CUDA weights only")
            for name in ("m", "v", "s_fixed"):
                lst = getattr(self, name, None)
                if lst is not None and lst[i].device != w.device:  # layer moved after opt creation: follow it
                    lst[i] = lst[i].to(w.device)
            g = layer._grad_w
            if g.dtype != torch.float32 or g.device != w.device or g.shape != w.shape:
                raise RuntimeError("Eco optimizers: layer._grad_w must be fp32 with the weights' shape and device")
            g = g.contiguous()
            d = nat.Fp32Layer()
            d.w, d.m, d.g = w.data_ptr(), self.m[i].data_ptr(), g.data_ptr()
            d.v = self.v[i].data_ptr() if self._KIND == 1 else None
            sw = layer.s_w.reshape(-1).contiguous()
            sf = self.s_fixed[i].reshape(-1).contiguous()
            d.sw, d.s_fixed = sw.data_ptr(), sf.data_ptr()
            d.rows, d.cols = w.shape
            d.stream = i
            d.norm_out = norms[i:].data_ptr()
            d.stepped_out = stepped[i:].data_ptr()
            u = None
            if replay:
                # the reference draws torch.rand_like only for a layer it steps (eco.py:44-46)
                if bool(torch.isfinite(g).all()):
                    u = torch.rand_like(g)
                    d.u = u.data_ptr()
                else:
                    d.u = g.data_ptr()  # not read: the layer is skipped on the device as well
            keep += [g, sw, sf, u]
            descs.append(d)
            stepped_layers.append((i, w.numel()))
        hyper = hyper_fn()
        hyper.kind = self._KIND
        hyper.sr_mode = nat.SR_REPLAY_F32 if replay else nat.SR_PHILOX
        hyper.seed = 0 if replay else _sr.new_key()
        self._last_key = hyper.seed  # the step's Philox key (tests reproduce its uniforms)
        pending = []
        for c0 in range(0, n, 64):
            arr = (nat.Fp32Layer * min(64, n - c0))(*descs[c0:c0 + 64])
            need = nat.load().eco_fp32_eco_scratch_len(arr, len(arr))
            key = (c0, str(dev))
            buf = self._scratch.get(key)
            if buf is None or buf.numel() < need:
                buf = self._scratch[key] = torch.empty(need, dtype=torch.float64, device=dev)
            nat.call("eco_fp32_eco_step", arr, len(arr), ctypes.byref(hyper), buf.data_ptr(), need, nat.stream())
            tiles = need // 3
            off = 2 * tiles
            for (i, numel) in stepped_layers[c0:c0 + 64]:
                nt = (numel + TILE - 1) // TILE
                pending.append((i, numel, buf, off, nt))
                off += nt
        self._keep = keep
        self._pending = pending

    def _read_stats(self) -> None:
        pending, self._pending = self._pending, None
        if not pending:
            return
        stepped = self._flags_dev[1].tolist()
        tot_e, n_e = 0.0, 0
        for i, numel, buf, off, nt in pending:
            if not stepped[i]:
                continue
            tot_e += sum(buf[off:off + nt].tolist()) / numel  # e.abs().mean() (eco.py:128, :225)
            n_e += 1
        if n_e:
            self._stats["mean_abs_e"] = tot_e / n_e

    @property
    def stats(self) -> dict:
        if getattr(self, "_pending", None):
            self._read_stats()
        return self._stats

    @stats.setter
    def stats(self, value: dict) -> None:
        self._pending = None
        self._stats = value

    def last_norms(self) -> list[float]:
        """The gradient norms of the last step (fp32, as a list; reads the device)."""
        return self._flags_dev[0].tolist()

    def set_lr(self, lr: float):
        self.lr = lr
        if self._bias_opt is not None:
            for pg in self._bias_opt.param_groups:
                pg["lr"] = lr

    @torch.no_grad()
    def zero_grad(self):
        for layer in self.layers:
            layer._grad_w = None
            if layer.bias is not None and layer.bias.grad is not None:
                layer.bias.grad.zero_()
        if self._bias_opt is not None:
            self._bias_opt.zero_grad()


class EcoSGDM(_FusedFp32):
    """SGD with momentum + ECO error injection, no master weights (eco.py:50-137).

    int8 weights on a frozen grid and an fp32 momentum buffer; the weight step is the
    fused two-launch kernel pair (``_FusedFp32``), the biases take ``torch.optim.SGD``
    as in the reference.  ``m = beta * m + (1 - beta) * g`` form: pass ``lr / (1 - beta)``
    to match torch SGD step sizes."""

    _KIND = 0

    def __init__(self, int8_layers, lr: float = 1e-2, momentum: float = 0.9, weight_decay: float = 0.0,
                 grad_clip: float | None = 1.0, bias_lr: float | None = None):
        assert momentum > 0, "ECO requires beta > 0 (alpha = (1/lr)(1-1/beta) is undefined otherwise)"
        self.layers = list(int8_layers)
        self.lr = lr
        self.beta = momentum
        self.wd = weight_decay
        self.grad_clip = grad_clip
        self.m = [torch.zeros_like(layer.w_i8, dtype=torch.float32) for layer in self.layers]
        self.s_fixed = [layer.s_w.clone() for layer in self.layers]  # frozen grid
        bparams = [layer.bias for layer in self.layers if layer.bias is not None]
        self._bias_opt = torch.optim.SGD(bparams, lr=bias_lr or lr, momentum=momentum) if bparams else None
        self.step_count = 0
        self._stats = {"skipped": 0, "mean_abs_e": 0.0}
        self._scratch: dict = {}

    @torch.no_grad()
    def step(self):
        from . import _native as nat

        self.step_count += 1

        def hyper():
            h = nat.Fp32Hyper()
            h.lr, h.beta1, h.weight_decay = float(self.lr), float(self.beta), float(self.wd)
            h.grad_clip = -1.0 if self.grad_clip is None else float(self.grad_clip)
            h.bc1 = h.bc2 = 1.0
            return h

        self._fused_step(hyper)
        if self._bias_opt is not None:
            self._bias_opt.step()


class EcoAdam(_FusedFp32):
    """Adam + ECO error injection (paper Algorithm 3), no master weights (eco.py:140-235).

    int8 weights on a frozen grid plus fp32 ``m`` / ``v``; the injection uses Adam's
    element-wise step ``m += e * (1 - 1/beta1) / eta_t``.  The weight step is the fused
    kernel pair; the biases take ``torch.optim.Adam`` as in the reference."""

    _KIND = 1

    def __init__(self, int8_layers, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, grad_clip: float | None = 1.0, bias_lr: float | None = None):
        b1, b2 = betas
        assert b1 > 0, "ECO requires beta1 > 0"
        self.layers = list(int8_layers)
        self.lr = lr
        self.b1, self.b2, self.eps = b1, b2, eps
        self.wd = weight_decay
        self.grad_clip = grad_clip
        self.m = [torch.zeros_like(layer.w_i8, dtype=torch.float32) for layer in self.layers]
        self.v = [torch.zeros_like(layer.w_i8, dtype=torch.float32) for layer in self.layers]
        self.s_fixed = [layer.s_w.clone() for layer in self.layers]  # frozen grid
        bparams = [layer.bias for layer in self.layers if layer.bias is not None]
        self._bias_opt = (torch.optim.Adam(bparams, lr=bias_lr or lr, betas=betas, eps=eps) if bparams else None)
        self.t = 0
        self._stats = {"skipped": 0, "mean_abs_e": 0.0}
        self._scratch: dict = {}

    @torch.no_grad()
    def step(self):
        from . import _native as nat

        self.t += 1

        def hyper():
            h = nat.Fp32Hyper()
            h.lr, h.beta1, h.beta2, h.eps = float(self.lr), float(self.b1), float(self.b2), float(self.eps)
            h.weight_decay = float(self.wd)
            h.grad_clip = -1.0 if self.grad_clip is None else float(self.grad_clip)
            h.bc1, h.bc2 = 1.0 - self.b1 ** self.t, 1.0 - self.b2 ** self.t  # eco.py:184
            return h

        self._fused_step(hyper)
        if self._bias_opt is not None:
            self._bias_opt.step()


class EcoInt8SGDM:
    """Fully-int8 ECO: int8 weights, int8 gradients, int8 momentum (eco.py:238-446)."""

    def __init__(self, int8_layers, lr: float = 1e-2, momentum: float = 0.9, weight_decay: float = 0.0,
                 grad_clip: float | None = 1.0, bias_lr: float | None = None, backend: str = "auto"):
        assert momentum > 0, "ECO requires beta > 0"
        assert backend in ("auto", "torch", "triton", "cuda"), "backend: auto | triton | cuda"
        self.layers = list(int8_layers)
        self.lr = lr
        self.beta = momentum
        self.wd = weight_decay
        self.grad_clip = grad_clip  # a no-op for this optimizer, as in the reference (eco.py:264-265)
        self.backend = backend
        self.m_i8 = [torch.zeros_like(layer.w_i8) for layer in self.layers]
        self.s_m = [1.0 for _ in self.layers]  # left stale by the fused step, as in the reference
        self.s_fixed = [layer.s_w.clone() for layer in self.layers]
        bparams = [layer.bias for layer in self.layers if layer.bias is not None]
        self._bias_opt = torch.optim.SGD(bparams, lr=bias_lr or lr, momentum=momentum) if bparams else None
        self.step_count = 0
        self.stats = {"skipped": 0, "dead_grads": 0, "sat_ratio": 0.0, "mean_abs_e": 0.0, "fused_steps": 0}
        self.last_step_backend = "cuda"
        self._scratch: dict[str, torch.Tensor] = {}
        self._sm: dict[int, torch.Tensor] = {}

    def set_lr(self, lr: float):
        self.lr = lr
        if self._bias_opt is not None:
            for pg in self._bias_opt.param_groups:
                pg["lr"] = lr

    def _scratch_for(self, device: torch.device) -> torch.Tensor:
        key = str(device)
        buf = self._scratch.get(key)
        if buf is None:
            buf = torch.zeros(4, dtype=torch.int32, device=device)
            self._scratch[key] = buf
        return buf

    @torch.no_grad()
    def _step_fused(self, i: int, layer, g: torch.Tensor) -> bool:
        """One fused step for one layer (eco.py:330-362)."""
        from .triton_kernels import triton_eco_step_

        dev = layer.w_i8.device
        sw = self.s_fixed[i]
        if sw.device != dev:
            sw = sw.to(dev)
            self.s_fixed[i] = sw
        m = self.m_i8[i]
        if m.device != dev:
            m = m.to(dev)
            self.m_i8[i] = m
        sm_t = self._sm.get(i)
        if sm_t is None or sm_t.device != dev:
            sm_t = torch.ones((), dtype=torch.float32, device=dev)
            self._sm[i] = sm_t
        res = triton_eco_step_(layer.w_i8, m, g.contiguous(), sw.reshape(-1).contiguous(), sm_t, lr=float(self.lr),
                               beta=float(self.beta), wd=float(self.wd), seed=random.getrandbits(31),
                               scratch=self._scratch_for(dev))
        return res == "ok"

    @torch.no_grad()
    def step(self):
        self.step_count += 1
        if self.backend == "torch":
            raise RuntimeError("backend='torch' is not available: the ecoint8 B200 build has only the "
                               "fused CUDA step (backend='auto' | 'triton' | 'cuda')")
        for layer in self.layers:
            if not layer.w_i8.is_cuda:
                raise RuntimeError("EcoInt8SGDM (B200 build) needs every layer on a CUDA device "
                                   f"(cuda={[l.w_i8.is_cuda for l in self.layers]})")
        self.last_step_backend = "cuda"
        for i, layer in enumerate(self.layers):
            g = _get_grad_w(layer)
            if g is None:
                continue
            if self._step_fused(i, layer, g):
                self.stats["fused_steps"] += 1
        if self._bias_opt is not None:
            self._bias_opt.step()

    @torch.no_grad()
    def zero_grad(self):
        for layer in self.layers:
            layer._grad_w = None
            if layer.bias is not None and layer.bias.grad is not None:
                layer.bias.grad.zero_()
        if self._bias_opt is not None:
            self._bias_opt.zero_grad()

    def memory_bytes(self) -> int:
        """Stored state in bytes over all layers (int8 weights + int8 momentum)."""
        return sum(layer.w_i8.numel() + m.numel() for layer, m in zip(self.layers, self.m_i8))
