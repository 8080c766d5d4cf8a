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


def int_mm(a8: torch.Tensor, b8: torch.Tensor) -> torch.Tensor:
    """layers.py:26-42: the exact int8 x int8 -> int32 product.  On CPU it is the reference's
    ``torch._int_mm``; on CUDA the reference pads (``pad_mm_dims``) and calls cuBLASLt, which
    rejects some padded shapes (e.g. M 33, K 17, N 70), so here the product is taken in float64
    on the device -- exact, like every int8 GEMM, since each partial sum is an integer far
    below 2^53 -- and the int32 result is the same."""
    a8 = a8.contiguous()
    b8 = b8.contiguous()
    if a8.is_cuda:
        return (a8.to(torch.float64) @ b8.to(torch.float64)).to(torch.int32)
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
