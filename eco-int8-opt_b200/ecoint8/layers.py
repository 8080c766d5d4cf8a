"""Autograd int8 layer (API of ``ecoint8/layers.py`` v0.4.9).

``Int8Linear`` keeps fp32 activations at its boundary (dynamic per-tensor
quantization in, float dequantization out) and feeds fp32 weight gradients to
the ECO optimizers through ``layer._grad_w``.  Its three int8 GEMMs run on the
B200 tcgen05 kernels (no padding) with the fp32 epilogue fused (layers.py:45-75).
"""

from __future__ import annotations

import weakref

import torch
import torch.nn as nn

from . import _native, _ops
from .quant import dequantize, quantize_per_channel, quantize_tensor_dynamic


def _int_mm(a8: torch.Tensor, b8: torch.Tensor) -> torch.Tensor:
    """int8 x int8 -> int32 on tcgen05 (layers.py:26-42), any M, K, N."""
    _native.require_cuda(a8, b8)
    M, K = a8.shape
    N = b8.shape[1]
    if b8.stride(0) == 1 and b8.stride(1) >= K:  # b8 is a transposed view of [N, K]
        return _ops.gemm_s32(a8, 0, b8.t(), 0, M, N, K)
    return _ops.gemm_s32(a8, 0, b8, 1, M, N, K)


class Int8LinearFunc(torch.autograd.Function):
    """layers.py:45-75 with every int8 GEMM's fp32 epilogue fused into it and the dynamic
    scales kept on the device (no ``.item()`` per call): the input and the output gradient
    are quantized by ``eco_quantize_dynamic_f32`` (quant.py:35-38), and ``eco_gemm_s8_dequant``
    computes ``acc.to(float32) * s_x * s_w.t() + bias``, ``dw_acc.float() * (s_g * s_x)`` and
    ``dx_acc.float() * (s_g * s_w.mean())`` in PyTorch's fp32 operation order, bit for bit.
    ``s_w.mean()`` is read once per layer (it is a frozen buffer) and cached."""

    @staticmethod
    def forward(ctx, x_f32, w_i8, s_w, bias, layer_ref):
        if x_f32.dtype != torch.float32 or x_f32.dim() != 2:
            raise RuntimeError("Int8Linear (B200 build): 2-D fp32 input")
        x_i8, s_x = _ops.quantize_dynamic(x_f32)
        M, K = x_i8.shape
        N = w_i8.shape[0]
        y = _ops.gemm_dequant(x_i8, 0, w_i8, 0, M, N, K, s_x, 1.0, col_scale=s_w.reshape(-1).contiguous(),
                              bias=None if bias is None else bias.detach().contiguous())
        ctx.save_for_backward(x_i8, w_i8, s_w)
        ctx.s_x = s_x  # a device scale (the reference's float(s_x))
        ctx.has_bias = bias is not None
        ctx.layer_ref = layer_ref
        return y

    @staticmethod
    def backward(ctx, grad_out):
        x_i8, w_i8, s_w = ctx.saved_tensors
        g_i8, s_g = _ops.quantize_dynamic(grad_out.to(torch.float32))
        M, N = g_i8.shape
        # dW: exact, both scales per-tensor (layers.py:63-64): g^T x
        grad_w = _ops.gemm_dequant(g_i8, 1, x_i8, 1, N, x_i8.shape[1], M, s_g, ctx.s_x)
        # dX: the per-channel s_w replaced by its mean (:66-67): g w
        grad_x = _ops.gemm_dequant(g_i8, 0, w_i8, 1, M, w_i8.shape[1], N, s_g, _sw_mean(s_w))
        grad_bias = grad_out.sum(0) if ctx.has_bias else None
        layer = ctx.layer_ref()
        if layer is not None:
            layer._grad_w = grad_w
        return grad_x, None, None, grad_bias, None


_SW_MEAN: dict = {}  # (storage, version) -> float(s_w.mean())


def _sw_mean(s_w: torch.Tensor) -> float:
    """``s_w.mean().item()`` (PyTorch's own fp32 reduction), cached while the buffer is unchanged."""
    key = (s_w.data_ptr(), s_w._version, s_w.numel())
    v = _SW_MEAN.get(key)
    if v is None:
        if len(_SW_MEAN) > 4096:
            _SW_MEAN.clear()
        v = _SW_MEAN[key] = s_w.mean().item()
    return v


class Int8Linear(nn.Module):
    """Drop-in ``nn.Linear`` with int8 weights and int8 GEMMs (layers.py:78-111)."""

    def __init__(self, in_f: int, out_f: int, bias: bool = True):
        super().__init__()
        w_fp = torch.randn(out_f, in_f) * (2.0 / in_f) ** 0.5
        w_i8, s_w = quantize_per_channel(w_fp, axis=0)
        self.register_buffer("w_i8", w_i8)
        self.register_buffer("s_w", s_w)
        self.bias = nn.Parameter(torch.zeros(out_f)) if bias else None
        self._grad_w: torch.Tensor | None = None

    @classmethod
    def from_float(cls, lin: nn.Linear) -> "Int8Linear":
        m = cls(lin.in_features, lin.out_features, lin.bias is not None)
        w_i8, s_w = quantize_per_channel(lin.weight.detach(), axis=0)
        m.w_i8.copy_(w_i8)
        m.s_w.copy_(s_w)
        if lin.bias is not None:
            m.bias.data.copy_(lin.bias.detach())
        return m

    def forward(self, x):
        return Int8LinearFunc.apply(x, self.w_i8, self.s_w, self.bias, weakref.ref(self))

    def extra_repr(self):
        return f"in={self.w_i8.shape[1]}, out={self.w_i8.shape[0]}, int8=True"

    def w_fp32(self) -> torch.Tensor:
        """Transient fp32 view of the weights."""
        return dequantize(self.w_i8, self.s_w)

    def memory_bytes(self) -> int:
        return self.w_i8.numel()


def to_int8(model: nn.Module) -> nn.Module:
    """Recursively swap ``nn.Linear`` for ``Int8Linear`` (layers.py:114-121)."""
    for name, child in list(model.named_children()):
        if isinstance(child, nn.Linear):
            setattr(model, name, Int8Linear.from_float(child))
        else:
            to_int8(child)
    return model
