"""ECO optimizers without master weights (API of ``ecoint8/eco.py`` v0.4.9).

``EcoInt8SGDM`` -- int8 weights, int8 momentum, fp32 only as a transient -- runs
its step as the library's fused CUDA kernels (``triton_eco_step_`` seam,
eco.py:330-362).  There is one backend: ``backend`` is accepted for
compatibility; ``"auto"``, ``"triton"`` and ``"cuda"`` select the fused CUDA
step and ``"torch"`` (the reference's eager fallback) raises, as does any
layer that is not on an sm_100 GPU.

``EcoSGDM`` and ``EcoAdam`` (fp32 optimizer state) are outside this build's
scope; their names raise ``NotImplementedError`` on construction.
"""

from __future__ import annotations

import random

import torch

from .quant import EPS  # noqa: F401  (re-exported like the reference)

__all__ = ["EcoSGDM", "EcoAdam", "EcoInt8SGDM"]


def _get_grad_w(layer) -> torch.Tensor | None:
    """The stashed fp32 weight gradient, or None if absent / non-finite (eco.py:39-47)."""
    g = layer._grad_w
    if g is None:
        return None
    g = g.clone()
    if not torch.isfinite(g).all():
        return None
    return g


class EcoSGDM:
    """Not part of the B200 build (fp32 momentum state; eco.py:50-137)."""

    def __init__(self, *args, **kwargs):
        raise NotImplementedError("EcoSGDM (fp32 state) is not part of the ecoint8 B200 build; "
                                  "use I8ECO or EcoInt8SGDM")


class EcoAdam:
    """Not part of the B200 build (fp32 moment state; eco.py:140-235)."""

    def __init__(self, *args, **kwargs):
        raise NotImplementedError("EcoAdam (fp32 state) is not part of the ecoint8 B200 build; "
                                  "use I8ECO or EcoInt8SGDM")


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
