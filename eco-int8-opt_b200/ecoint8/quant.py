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


def cross_entropy_grad_i8(logits_i8: torch.Tensor, s_out, labels: torch.Tensor, count: int | None = None,
                          return_fp32: bool = False):
    """The strict loop's loss boundary in two kernels, with no host synchronisation.

    Replaces, on CUDA tensors, the reference training loop's

        logits_fp = (logits_i8.to(torch.float32) * s_out).requires_grad_()
        loss = nn.CrossEntropyLoss()(logits_fp, y)
        (g_fp,) = torch.autograd.grad(loss, logits_fp)
        g_i8, s_g = quantize_tensor_dynamic(g_fp, stochastic=True)

    (examples/i8_demo.py:56-59, quant.py:19-38).  Returns ``(loss, g_i8, s_g)``:
    ``loss`` a 0-dim fp32 device tensor (the mean over ``count`` samples of this
    process's rows), ``g_i8`` int8 ``[rows, cols]`` and ``s_g`` a device scale that
    ``I8Sequential.backward_i8`` reads in place (``float(s_g)`` reads it on the host).

    ``count``: the samples the mean runs over (default: the rows here; the global
    batch under data parallelism, where max |g| is also taken over all ranks).
    Stochastic rounding: the library's Philox stream with batch rows numbered
    globally (``ecoint8._sr.batch_rows``), or, inside ``ecoint8.sr_replay()``, one
    ``torch.rand`` draw of the logits' shape on their device -- the draw
    ``torch.rand_like`` makes in the reference.  The fp32 gradient agrees with
    PyTorch's to within a few ulp (its log-sum order is this kernel's own); given
    the gradient, the quantization is PyTorch's arithmetic bit for bit.
    ``return_fp32`` (tests): also return the fp32 gradient.
    """
    from . import _native as nat
    from . import _scale, _sr, parallel

    nat.require_cuda(logits_i8, labels)
    if logits_i8.dtype != torch.int8 or logits_i8.dim() != 2:
        raise AssertionError("logits must be a 2-D int8 tensor")
    if labels.dtype != torch.int64 or labels.dim() != 1 or labels.shape[0] != logits_i8.shape[0]:
        raise AssertionError("labels must be int64 [rows]")
    x = logits_i8 if logits_i8.stride(1) == 1 else logits_i8.contiguous()
    labels = labels.contiguous()
    rows, cols = x.shape
    ld = x.stride(0) if rows > 1 else cols
    count = rows if count is None else int(count)
    dev = x.device
    s_out = float(s_out)
    stats = torch.empty((rows, 2), dtype=torch.float32, device=dev)
    row_loss = torch.empty(rows, dtype=torch.float32, device=dev)
    amax = torch.empty(1, dtype=torch.int32, device=dev)
    nat.call("eco_ce_grad_rowstats", x.data_ptr(), rows, cols, ld, s_out, labels.data_ptr(), count,
             stats.data_ptr(), row_loss.data_ptr(), amax.data_ptr(), nat.stream())
    amax_src, bits = amax, 32
    if parallel.active():
        amax_src, bits = parallel.max_over_ranks(amax), 64
    keep = None
    if _sr.replaying():
        keep = torch.rand((rows, cols), device=dev)  # the reference's torch.rand_like(v) draw
        spec = nat.sr_spec(nat.SR_REPLAY_F32, keep)
    else:
        spec = nat.sr_spec(nat.SR_PHILOX, seed=_sr.new_key(), stream_id=0, row_base=_sr.row_base())
        if _sr.LOG is not None:
            _sr.LOG.append(("boundary", spec.seed, 0, (rows, cols), 24, spec.row_base))
    # rows padded to 16 bytes: the backward's GEMMs read g in place (TMA rows), no relayout
    ld_g = (cols + 15) // 16 * 16
    g = torch.empty((rows, ld_g), dtype=torch.int8, device=dev)[:, :cols]
    g_fp = torch.empty((rows, cols), dtype=torch.float32, device=dev) if return_fp32 else None
    scale = torch.empty(3, dtype=torch.int64, device=dev)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    nat.call("eco_ce_grad_quantize", x.data_ptr(), rows, cols, ld, s_out, labels.data_ptr(), count,
             stats.data_ptr(), amax_src.data_ptr(), bits, spec, g.data_ptr(), ld_g, nat.ptr(g_fp), scale.data_ptr(),
             row_loss.data_ptr(), loss.data_ptr(), nat.stream())
    s_g = _scale.DevScale(scale)
    return (loss, g, s_g, g_fp) if return_fp32 else (loss, g, s_g)
