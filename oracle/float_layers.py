"""``Int8LinearFunc`` restated op by op in PyTorch (oracle; test infrastructure only).

Follows ``ecoint8/layers.py`` (v0.4.9): ``_int_mm`` (:26-42, the padding wrapper around
``torch._int_mm``), ``Int8LinearFunc.forward`` (:45-57) and ``.backward`` (:59-75), and
``quantize_tensor_dynamic`` / ``calc_scale`` / ``quantize_symmetric`` (``quant.py:9-38``),
with the same PyTorch operations in the same order, so on a given device it computes what
the reference computes there.
"""

from __future__ import annotations

import torch

INT8_MAX = 127.0
EPS = 1e-8


def calc_scale(amax: float) -> float:
    a = float(amax)
    if a < EPS:
        return 1.0
    return a / INT8_MAX


def quantize_tensor_dynamic(x: torch.Tensor):
    amax = x.detach().abs().max().item()
    s = calc_scale(amax)
    v = x / (s + EPS)
    return torch.clamp(torch.round(v), -127, 127).to(torch.int8), s


def _pad8(v: int) -> int:
    return (v + 7) // 8 * 8


def int_mm(a8: torch.Tensor, b8: torch.Tensor) -> torch.Tensor:
    """layers.py:26-42 (``pad_mm_dims``: M to at least 32 and a multiple of 8, K and N to 8)."""
    a8 = a8.contiguous()
    b8 = b8.contiguous()
    if a8.is_cuda:
        M, K = a8.shape
        N = b8.shape[1]
        M8, K8, N8 = max(32, _pad8(M)), _pad8(K), _pad8(N)
        if (M8, K8, N8) != (M, K, N):
            a8 = torch.nn.functional.pad(a8, (0, K8 - K, 0, M8 - M))
            b8 = torch.nn.functional.pad(b8, (0, N8 - N, 0, K8 - K))
            return torch._int_mm(a8, b8)[:M, :N]
    return torch._int_mm(a8, b8)


def forward(x_f32, w_i8, s_w, bias):
    """Returns (y, x_i8, s_x)."""
    x_i8, s_x = quantize_tensor_dynamic(x_f32)
    acc = int_mm(x_i8, w_i8.t())
    y = acc.to(torch.float32) * s_x * s_w.t()
    if bias is not None:
        y = y + bias
    return y, x_i8, float(s_x)


def backward(grad_out, x_i8, w_i8, s_w, s_x, has_bias):
    """Returns (grad_x, grad_w, grad_bias)."""
    g_i8, s_g = quantize_tensor_dynamic(grad_out)
    dw_acc = int_mm(g_i8.t(), x_i8)
    grad_w = dw_acc.to(torch.float32) * (s_g * s_x)
    dx_acc = int_mm(g_i8, w_i8)
    grad_x = dx_acc.to(torch.float32) * (s_g * s_w.mean().item())
    grad_bias = grad_out.sum(0) if has_bias else None
    return grad_x, grad_w, grad_bias
