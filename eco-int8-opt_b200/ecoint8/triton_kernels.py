"""The optimizer seam of ``ecoint8/triton_kernels.py`` v0.4.9, served by CUDA.

The reference fuses ``EcoInt8SGDM``'s step into two Triton kernels plus three
torch reductions (triton_kernels.py:127-170).  This build has no Triton:
``triton_eco_step_`` keeps the same signature and semantics and runs the
library's ``eco_sgdm_step`` (max|g|, pass 1, pass 2 and the scale update as
three stream-ordered kernels, no host synchronisation).  Draws come from
``tl.rand``'s generator (Philox4x32-10, counter = element offset), so with the
same ``seed`` the nudges are the reference's.
"""

from __future__ import annotations

import torch

from . import _native

TRITON_AVAILABLE = False  # no Triton in this build; the fused step is CUDA
BLOCK = 1024  # triton_kernels.py:48 (partial-max block of the reference)
MAX_SCRATCH = 8192  # triton_kernels.py:49


def triton_eco_step_(w_i8: torch.Tensor, m_i8: torch.Tensor, g_fp32: torch.Tensor, sw_flat: torch.Tensor,
                     sm_t: torch.Tensor, *, lr: float, beta: float, wd: float, seed: int,
                     scratch: torch.Tensor) -> str:
    """Fused in-place EcoInt8SGDM step (triton_kernels.py:127-170).  Returns ``"ok"``.

    ``sm_t`` is the persistent 0-dim fp32 momentum scale, updated in place on
    the device.  ``scratch`` needs at least 16 bytes; it is used as four
    zeroed uint32 words (the call clears them first).
    """
    _native.require_cuda(w_i8, m_i8, g_fp32, sw_flat, sm_t, scratch)
    assert w_i8.dtype == torch.int8 and w_i8.is_contiguous()
    assert m_i8.shape == w_i8.shape and m_i8.dtype == torch.int8 and m_i8.is_contiguous()
    assert g_fp32.shape == w_i8.shape and g_fp32.dtype == torch.float32
    assert sw_flat.dtype == torch.float32 and sw_flat.numel() == w_i8.shape[0]
    assert sm_t.numel() == 1 and sm_t.dtype == torch.float32
    assert scratch.numel() * scratch.element_size() >= 16 and scratch.is_contiguous()
    g = g_fp32.contiguous()
    sw = sw_flat.reshape(-1).contiguous()
    alpha = (1.0 / lr) * (1.0 - 1.0 / beta)
    rows, cols = w_i8.shape
    _native.call("eco_sgdm_step", w_i8.data_ptr(), m_i8.data_ptr(), g.data_ptr(), rows, cols, sw.data_ptr(),
                 sm_t.data_ptr(), float(lr), float(beta), float(wd), float(alpha), int(seed), scratch.data_ptr(),
                 _native.stream())
    return "ok"
