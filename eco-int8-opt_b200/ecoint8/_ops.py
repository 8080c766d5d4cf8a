"""Tensor-level wrappers over the C ABI (CUDA tensors only).

Layouts: every matrix is row-major with unit column stride.  GEMM operands
must start on a 16-byte boundary with a leading dimension that is a multiple
of 16 bytes (the TMA rule); operands that are not are copied once into an
aligned buffer (``aligned``), which only happens for odd widths such as 2, 10
or 1000.
"""

from __future__ import annotations

import torch

from . import _native as nat
from ._sr import Site

_I8, _I32, _I64 = torch.int8, torch.int32, torch.int64


def _rowmajor(t: torch.Tensor) -> torch.Tensor:
    if t.dim() != 2:
        raise RuntimeError(f"expected a matrix, got shape {tuple(t.shape)}")
    return t if (t.stride(1) == 1 or t.shape[1] <= 1) and t.stride(0) >= max(t.shape[1], 1) else t.contiguous()


def aligned(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """``(buffer, ld)`` holding ``t`` with a 16-byte aligned base and leading dimension."""
    t = _rowmajor(t)
    rows, cols = t.shape
    ld = t.stride(0) if rows > 1 else max(cols, 1)
    if ld % 16 == 0 and t.data_ptr() % 16 == 0:
        return t, ld
    ld16 = (max(cols, 1) + 15) // 16 * 16
    buf = torch.empty((rows, ld16), dtype=t.dtype, device=t.device)
    nat.call("eco_copy2d_s8", t.data_ptr(), t.stride(0) if rows > 1 else cols, buf.data_ptr(), ld16, rows, cols,
             nat.stream())
    return buf, ld16


def gemm_s32(a: torch.Tensor, a_layout: int, b: torch.Tensor, b_layout: int, M: int, N: int, K: int,
             bias: torch.Tensor | None = None, amax: torch.Tensor | None = None) -> torch.Tensor:
    """``C[M,N] = A.B (+bias)`` int32; layouts as in ``eco_gemm_s8s32``; ``amax`` an int32 [1] out."""
    nat.require_cuda(a, b, bias, amax)
    a, lda = aligned(a)
    b, ldb = aligned(b)
    c = torch.empty((M, N), dtype=_I32, device=a.device)
    nat.call("eco_gemm_s8s32", a.data_ptr(), lda, a_layout, b.data_ptr(), ldb, b_layout, M, N, K, nat.ptr(bias),
             c.data_ptr(), N, nat.ptr(amax), nat.stream())
    return c


def gemm_requant(a: torch.Tensor, a_layout: int, b: torch.Tensor, b_layout: int, M: int, N: int, K: int,
                 bias: torch.Tensor | None, mult: torch.Tensor, shift: int, relu: bool, site: Site,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused GEMM + requant: ``sat8(relu?(SR((A.B + bias) * mult, shift)))``."""
    nat.require_cuda(a, b, bias, mult)
    a, lda = aligned(a)
    b, ldb = aligned(b)
    y = out if out is not None else torch.empty((M, N), dtype=_I8, device=a.device)
    nat.call("eco_gemm_s8_requant", a.data_ptr(), lda, a_layout, b.data_ptr(), ldb, b_layout, M, N, K,
             nat.ptr(bias), mult.data_ptr(), shift, int(relu), site.spec, y.data_ptr(), y.stride(0), nat.stream())
    return y


def gemm_dequant(a: torch.Tensor, a_layout: int, b: torch.Tensor, b_layout: int, M: int, N: int, K: int,
                 sa, sb, col_scale: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 ``[M, N] = fp32(A.B) * fp32(sa * sb) (* col_scale[n]) (+ bias[n])``; ``sa``/``sb`` are
    Python floats or device scales (``_scale.DevScale``)."""
    from . import _scale

    nat.require_cuda(a, b, col_scale, bias)
    a, lda = aligned(a)
    b, ldb = aligned(b)
    for t in (col_scale, bias):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != N):
            raise RuntimeError("gemm_dequant: col_scale / bias must be contiguous fp32 of N values")
    pa, va = _scale.gain_args(sa)
    pb, vb = _scale.gain_args(sb)
    y = torch.empty((M, N), dtype=torch.float32, device=a.device)
    nat.call("eco_gemm_s8_dequant", a.data_ptr(), lda, a_layout, b.data_ptr(), ldb, b_layout, M, N, K, pa, va, pb, vb,
             nat.ptr(col_scale), nat.ptr(bias), y.data_ptr(), N, nat.stream())
    return y


def quantize_dynamic(x: torch.Tensor):
    """``quantize_tensor_dynamic(x)`` (round to nearest) of a 2-D fp32 CUDA tensor with the
    scale kept on the device: returns ``(int8 tensor, _scale.DevScale)``."""
    from . import _scale

    nat.require_cuda(x)
    if x.dtype != torch.float32 or x.dim() != 2:
        raise RuntimeError("quantize_dynamic: a 2-D fp32 tensor")
    x = _rowmajor(x)
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=_I8, device=x.device)
    amax = torch.empty(1, dtype=_I32, device=x.device)
    scale = torch.empty(3, dtype=torch.int64, device=x.device)
    nat.call("eco_quantize_dynamic_f32", x.data_ptr(), rows, cols, x.stride(0) if rows > 1 else cols,
             amax.data_ptr(), q.data_ptr(), cols, scale.data_ptr(), nat.stream())
    return q, _scale.DevScale(scale)


def requant(src: torch.Tensor, mult, shift: int, site: Site, bias: torch.Tensor | None = None,
            relu: bool = False, mask: torch.Tensor | None = None,
            sumsq: torch.Tensor | None = None) -> torch.Tensor:
    """int32 [R,C] -> int8 with per-column int32 ``mult`` (tensor) or a scalar int."""
    nat.require_cuda(src, bias, mask, sumsq)
    src = _rowmajor(src)
    rows, cols = src.shape
    mult_col = mult if isinstance(mult, torch.Tensor) else None
    mult_scalar = 0 if mult_col is not None else int(mult)
    ld_mask = 0
    if mask is not None:
        mask = _rowmajor(mask)
        ld_mask = mask.stride(0) if rows > 1 else cols
    dst = torch.empty((rows, cols), dtype=_I8, device=src.device)
    nat.call("eco_requant_s32_s8", src.data_ptr(), rows, cols, src.stride(0) if rows > 1 else cols, nat.ptr(bias),
             nat.ptr(mult_col), mult_scalar, shift, int(relu), site.spec, nat.ptr(mask), ld_mask, dst.data_ptr(),
             cols, nat.ptr(sumsq), nat.stream())
    return dst


def requant_dev(src: torch.Tensor, scale, key: int, row_base: int, mask: torch.Tensor | None = None,
                sumsq: torch.Tensor | None = None) -> torch.Tensor:
    """int32 [R,C] -> int8 with the multiplier and shift of a device scale
    (``_scale.DevScale``), Philox rounding with site key ``key``."""
    nat.require_cuda(src, mask, sumsq)
    src = _rowmajor(src)
    rows, cols = src.shape
    ld_mask = 0
    if mask is not None:
        mask = _rowmajor(mask)
        ld_mask = mask.stride(0) if rows > 1 else cols
    dst = torch.empty((rows, cols), dtype=_I8, device=src.device)
    spec = nat.sr_spec(nat.SR_PHILOX, seed=key, stream_id=0, row_base=row_base)
    nat.call("eco_requant_s32_s8_dev", src.data_ptr(), rows, cols, src.stride(0) if rows > 1 else cols,
             scale.t.data_ptr(), 0, spec, nat.ptr(mask), ld_mask, dst.data_ptr(), cols, nat.ptr(sumsq), nat.stream())
    return dst


def apply_mult_shift(x: torch.Tensor, mult, mult_kind: int, shift: int, site: Site) -> torch.Tensor:
    """int64 ``apply_mult_shift`` over a contiguous [rows, cols] view of ``x``."""
    nat.require_cuda(x, mult if isinstance(mult, torch.Tensor) else None)
    x = x.contiguous()
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // max(cols, 1) if cols else 0
    bits = {torch.int8: 8, torch.int32: 32, torch.int64: 64}[x.dtype]
    out = torch.empty(x.shape, dtype=_I64, device=x.device)
    mt = mult if isinstance(mult, torch.Tensor) else None
    nat.call("eco_apply_mult_shift", x.data_ptr(), bits, rows, cols, nat.ptr(mt), mult_kind,
             0 if mt is not None else int(mult), shift, site.spec, out.data_ptr(), nat.stream())
    return out


def colsum(g: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """int64 column sums of an int8 matrix (into ``out``, a contiguous int64 vector, if given)."""
    nat.require_cuda(g)
    g = _rowmajor(g)
    rows, cols = g.shape
    if out is None:
        out = torch.empty(cols, dtype=_I64, device=g.device)
    nat.call("eco_colsum_s8", g.data_ptr(), rows, cols, g.stride(0) if rows > 1 else cols, out.data_ptr(),
             nat.stream())
    return out


def amax(x: torch.Tensor) -> torch.Tensor:
    nat.require_cuda(x)
    x = x.contiguous()
    if x.dtype == _I8:
        x = x.to(_I32)
    out = torch.empty(1, dtype=_I64, device=x.device)
    nat.call("eco_amax", x.data_ptr(), 32 if x.dtype == _I32 else 64, x.numel(), out.data_ptr(), nat.stream())
    return out


def sumsq(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    nat.require_cuda(x)
    x = x.contiguous()
    out = out if out is not None else torch.empty(1, dtype=_I64, device=x.device)
    nat.call("eco_sumsq_s8", x.data_ptr(), x.numel(), out.data_ptr(), nat.stream())
    return out


# -- host reads that do not drain the stream ------------------------------------------
class PendingRead:
    """A small device tensor on its way to the host (``read_later``)."""

    __slots__ = ("host", "event")

    def __init__(self, host: torch.Tensor, event):
        self.host, self.event = host, event

    def value(self) -> list[int]:
        self.event.synchronize()
        return self.host.tolist()


_SIDE: dict = {}  # device -> (side stream, ring of pinned slots, ring position)


def read_later(t: torch.Tensor, work=None) -> PendingRead:
    """Start copying a small device tensor to the host on a side stream that waits only
    for the work queued so far on the current stream (and for ``work``, a collective's
    handle): kernels queued after this call keep the device busy while the host waits
    in ``PendingRead.value()``."""
    if t.numel() * t.element_size() > 64:
        raise ValueError("read_later: at most 64 bytes")
    dev = t.device
    ent = _SIDE.get(dev)
    if ent is None:
        ent = _SIDE[dev] = [torch.cuda.Stream(device=dev),
                            [(torch.empty(8, dtype=_I64, pin_memory=True), torch.cuda.Event()) for _ in range(16)], 0]
    side, ring, pos = ent
    ent[2] = (pos + 1) % len(ring)
    buf, ev = ring[pos]
    ev.synchronize()  # the slot's previous read (long finished)
    host = buf.view(torch.uint8)[:t.numel() * t.element_size()].view(t.dtype).view(t.shape)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        if work is not None:
            work.wait()
        host.copy_(t, non_blocking=True)
        ev.record(side)
    t.record_stream(side)
    return PendingRead(host, ev)
