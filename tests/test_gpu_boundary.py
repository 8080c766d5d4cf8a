"""The fused loss boundary (``ecoint8.quant.cross_entropy_grad_i8``) on a B200.

It replaces the reference loop's CE gradient plus ``quantize_tensor_dynamic(g,
stochastic=True)`` (examples/i8_demo.py:56-59, quant.py:19-38).  Checks:

* the fp32 gradient against PyTorch's own cross-entropy gradient (fp32 tolerance:
  the log-sum order is the kernel's own);
* ``s_g`` equals ``calc_scale(max |g|)`` of that gradient exactly;
* the int8 gradient is exactly PyTorch's quantization of that gradient, with the
  uniforms taken from the oracle's Philox stream (Philox mode) or with the very
  ``torch.rand_like`` draw the reference makes (replay mode);
* a row shard with ``count`` = the global batch and a global row offset
  reproduces the rows of the unsplit batch bit for bit (data parallelism).
"""

import numpy as np
import pytest
import torch

from oracle import philox as oph

pytestmark = pytest.mark.gpu

SHAPES = [(300, 1000), (257, 10), (64, 2), (33, 1537), (1, 7)]


def _case(rows, cols, seed):
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, generator=gen).cuda()
    labels = torch.randint(0, cols, (rows,), generator=gen).cuda()
    return logits, labels


def _torch_grad(logits, s_out, labels, count):
    x = (logits.to(torch.float32) * s_out).requires_grad_()
    loss = torch.nn.functional.cross_entropy(x, labels, reduction="sum") / count
    (g,) = torch.autograd.grad(loss, x)
    return loss.detach(), g


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gradient_scale_and_philox_quantization(rows, cols):
    from ecoint8 import _sr
    from ecoint8.quant import EPS, calc_scale, cross_entropy_grad_i8

    logits, labels = _case(rows, cols, rows + cols)
    s_out = 0.043
    _sr.LOG = []
    loss, g_i8, s_g, g = cross_entropy_grad_i8(logits, s_out, labels, return_fp32=True)
    log, _sr.LOG = _sr.LOG, None
    loss_ref, g_ref = _torch_grad(logits, s_out, labels, rows)
    # fp32 tolerance: a few ulp of the largest gradient
    tol = 8 * torch.finfo(torch.float32).eps * g_ref.abs().max().item()
    assert (g - g_ref).abs().max().item() <= tol
    assert abs(loss.item() - loss_ref.item()) <= 1e-5 * abs(loss_ref.item()) + 1e-7
    # the dynamic scale of this gradient, in the reference's arithmetic
    assert float(s_g) == calc_scale(g.abs().max().item())
    # the quantization of this gradient with the Philox uniforms, in PyTorch's arithmetic
    (_, key, stream, shape, _, row_base) = [e for e in log if e[0] == "boundary"][0]
    r = np.arange(rows, dtype=np.uint64)[:, None] + np.uint64(row_base)
    c = np.arange(cols, dtype=np.uint64)[None, :]
    field = oph.sr_field(key, stream, r, c)
    u = torch.from_numpy(((field >> np.uint64(8)).astype(np.float32) * np.float32(2.0 ** -24))).cuda()
    v = g / (float(s_g) + EPS)
    want = torch.clamp(torch.floor(v + u), -127, 127).to(torch.int8)
    assert torch.equal(g_i8, want)


@pytest.mark.parametrize("rows,cols", SHAPES[:3])
def test_replay_consumes_the_reference_rand_like_draw(rows, cols):
    import ecoint8
    from ecoint8.quant import cross_entropy_grad_i8, quantize_symmetric

    logits, labels = _case(rows, cols, 7 * rows + cols)
    torch.manual_seed(123)
    with ecoint8.sr_replay():
        _, g_i8, s_g, g = cross_entropy_grad_i8(logits, 0.02, labels, return_fp32=True)
    torch.manual_seed(123)
    want = quantize_symmetric(g, float(s_g), stochastic=True)  # quant.py:19-28 on the same draw
    assert torch.equal(g_i8, want)


def test_row_shard_with_global_count_equals_unsplit_batch():
    """Two shards of a batch, each with count = the whole batch and its global row
    offset, give the unsplit batch's int8 rows when they share the maximum."""
    from ecoint8 import _sr
    from ecoint8.quant import cross_entropy_grad_i8

    logits, labels = _case(512, 1000, 5)
    gen = torch.Generator().manual_seed(77)
    _sr.set_generator(gen)
    try:
        _, g_all, s_all, g_fp = cross_entropy_grad_i8(logits, 0.05, labels, return_fp32=True)
        # the shard whose rows hold the maximum reproduces the global scale by itself
        g_fp = g_fp.abs().amax(1)
        half = 0 if g_fp[:256].max() >= g_fp[256:].max() else 1
        lo = 256 * half
        gen.manual_seed(77)
        with _sr.batch_rows(lo):
            _, g_part, s_part = cross_entropy_grad_i8(logits[lo:lo + 256], 0.05, labels[lo:lo + 256], count=512)
    finally:
        _sr.set_generator(None)
    assert float(s_part) == float(s_all)
    assert torch.equal(g_part, g_all[lo:lo + 256])


def test_quantization_over_many_gradient_scales():
    """The gradient's division by the Python scalar ``s_g + EPS`` is PyTorch's CUDA multiply
    by the reciprocal taken in double and rounded to fp32; for about a quarter of all scales
    that differs from the fp32 quotient.  Forty logit scales (so forty gradient maxima)
    pin it, each on the reference's own ``torch.rand_like`` draw."""
    import ecoint8
    from ecoint8.quant import cross_entropy_grad_i8, quantize_symmetric

    logits, labels = _case(96, 50, 3)
    for i in range(40):
        s_out = 0.004 * (1.0 + 0.37 * i)
        torch.manual_seed(1000 + i)
        with ecoint8.sr_replay():
            _, g_i8, s_g, g = cross_entropy_grad_i8(logits, s_out, labels, return_fp32=True)
        torch.manual_seed(1000 + i)
        want = quantize_symmetric(g, float(s_g), stochastic=True)
        assert torch.equal(g_i8, want), i
