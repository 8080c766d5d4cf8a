"""fp32 boundary quantizers (same API and arithmetic as ``ecoint8/quant.py`` v0.4.9).

These sit outside the strict integer region: entry quantization of the input
batch and of the loss gradient, and the dequantization the autograd layer
uses.  They are plain PyTorch on whatever device the tensor lives on, exactly
as in the reference, so a harness that calls them consumes the global
generator the same way.
"""

from __future__ import annotations

import torch

INT8_MAX = 127.0
EPS = 1e-8


def calc_scale(amax: float, clip: float | None = None) -> float:
    """scale = amax / 127; amax below EPS gives 1.0 (quant.py:9-16)."""
    a = float(amax)
    if clip is not None:
        a = min(a, clip)
    if a < EPS:
        return 1.0
    return a / INT8_MAX


def quantize_symmetric(x: torch.Tensor, scale, stochastic: bool = False) -> torch.Tensor:
    """fp32 -> int8 on ``scale``; stochastic = floor(v + U[0,1)) (quant.py:19-28)."""
    s = scale + EPS
    v = x / s
    if stochastic:
        q = torch.floor(v + torch.rand_like(v))
    else:
        q = torch.round(v)
    return torch.clamp(q, -127, 127).to(torch.int8)


def dequantize(q: torch.Tensor, scale) -> torch.Tensor:
    return q.to(torch.float32) * scale


def quantize_tensor_dynamic(x: torch.Tensor, stochastic: bool = False) -> tuple[torch.Tensor, float]:
    """Per-tensor quantization with a dynamic amax scale (quant.py:35-38)."""
    amax = x.detach().abs().max().item()
    return quantize_symmetric(x, calc_scale(amax), stochastic), calc_scale(amax)


def quantize_per_channel(x: torch.Tensor, axis: int = 0, stochastic: bool = False):
    """Per-channel quantization (quant.py:41-45)."""
    amax = x.detach().abs().amax(dim=tuple(i for i in range(x.dim()) if i != axis), keepdim=True)
    s = torch.clamp(amax / INT8_MAX, min=EPS)
    return quantize_symmetric(x, s, stochastic), s


def saturation_ratio(q: torch.Tensor) -> float:
    """Fraction of values at +-127 (quant.py:48-50)."""
    return ((q == 127) | (q == -127)).float().mean().item()


def is_dead_grad(q: torch.Tensor) -> bool:
    return bool((q == 0).all())
