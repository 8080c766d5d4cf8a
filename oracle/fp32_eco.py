"""EcoSGDM / EcoAdam steps restated op by op in PyTorch (oracle; test infrastructure only).

Follows ``ecoint8/eco.py`` (v0.4.9): ``_get_grad_w`` (:39-47), ``EcoSGDM.step``
(:94-131), ``EcoAdam.step`` (:182-228) and ``quantize_symmetric`` (``quant.py:19-28``),
one weight layer at a time, with the same PyTorch operations in the same order, so
on a given device it computes what the reference computes there.  Two inputs the
reference makes itself can be supplied instead:

* ``u``: the uniforms of the stochastic rounding (the reference draws them with
  ``torch.rand_like``; passing that draw reproduces it);
* ``norm``: the gradient norm used for clipping (the reference's ``g.norm().item()``;
  the B200 kernel sums the squares in double, so a test can hand its value in to check
  everything downstream of it bit for bit).

Returns the new ``w_i8``, ``m`` (and ``v``), the ``|e|`` mean (``e.abs().mean().item()``)
and whether the layer was stepped (False when the gradient has a non-finite value).
"""

from __future__ import annotations

import torch

EPS = 1e-8  # quant.py:7


def quantize_symmetric_sr(x: torch.Tensor, scale: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """quant.py:19-28 with stochastic=True and the uniform draw given."""
    s = scale + EPS
    v = x / s
    q = torch.floor(v + u)
    return torch.clamp(q, -127, 127).to(torch.int8)


def _grad(g: torch.Tensor, w_fp32: torch.Tensor, grad_clip, wd, norm=None):
    """eco.py:39-47 and the clip / weight-decay lines of both steps."""
    g = g.clone()
    if not torch.isfinite(g).all():
        return None, None
    n = g.norm().item() if norm is None else float(norm)
    if grad_clip is not None and n > grad_clip:
        g.mul_(grad_clip / (n + EPS))
    if wd:
        g.add_(w_fp32, alpha=wd)
    return g, n


def sgdm_layer(w_i8, s_w, s_fixed, m, g, u, *, lr, beta, wd=0.0, grad_clip=1.0, norm=None):
    """One layer of EcoSGDM.step (eco.py:94-131)."""
    w_fp32 = w_i8.to(torch.float32) * s_w  # Int8Linear.w_fp32 (layers.py:103-105)
    g, n = _grad(g, w_fp32, grad_clip, wd, norm)
    if g is None:
        return w_i8.clone(), m.clone(), None, False, None
    b = beta
    alpha = (1.0 / lr) * (1.0 - 1.0 / b)
    m_tilde = m * b + g * (1.0 - b)
    th_tilde = w_fp32 - lr * m_tilde
    w_new = quantize_symmetric_sr(th_tilde, s_fixed, u)
    e = th_tilde - w_new.float() * s_fixed
    m_new = m_tilde + alpha * e
    return w_new, m_new, e.abs().mean().item(), True, n


def adam_layer(w_i8, s_w, s_fixed, m, v, g, u, *, t, lr, b1, b2, eps, wd=0.0, grad_clip=1.0, norm=None):
    """One layer of EcoAdam.step at step ``t`` (eco.py:182-228)."""
    bc1, bc2 = 1.0 - b1 ** t, 1.0 - b2 ** t
    w_fp32 = w_i8.to(torch.float32) * s_w
    g, n = _grad(g, w_fp32, grad_clip, wd, norm)
    if g is None:
        return w_i8.clone(), m.clone(), v.clone(), None, False, None
    m = m.clone()
    v = v.clone()
    m.mul_(b1).add_(g, alpha=1.0 - b1)
    v.mul_(b2).addcmul_(g, g, value=1.0 - b2)
    v_hat = (v / bc2).sqrt() + eps
    eta_t = lr / (bc1 * v_hat)
    th_tilde = w_fp32 - eta_t * (m / bc1)
    w_new = quantize_symmetric_sr(th_tilde, s_fixed, u)
    e = th_tilde - w_new.float() * s_fixed
    m.add_(e * ((1.0 - 1.0 / b1) / eta_t))
    return w_new, m, v, e.abs().mean().item(), True, n
