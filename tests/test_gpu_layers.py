"""Int8Linear (layers.py:45-111) on the fused B200 path against the reference's own PyTorch
arithmetic on the same GPU (``oracle/float_layers.py``: ``torch._int_mm`` with the reference's
padding, its fp32 epilogues and dynamic quantization, op by op; pinned to the reference by
``tests/test_oracle_golden.py``).  The int8 GEMMs are exact and every fp32 operation is
PyTorch's, so the output and all three gradients must agree bit for bit.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,in_f,out_f,bias", [(64, 40, 24, True), (33, 70, 17, False), (300, 784, 256, True),
                                               (1024, 4096, 1000, True), (5, 16, 8, True)])
def test_int8_linear_equals_reference_arithmetic(n, in_f, out_f, bias):
    from ecoint8.layers import Int8Linear
    from oracle import float_layers as fl

    dev = torch.device("cuda", 0)
    torch.manual_seed(n + in_f)
    layer = Int8Linear(in_f, out_f, bias).to(dev)
    if bias:
        layer.bias.data.copy_(torch.randn(out_f, device=dev) * 0.1)
    x = (torch.randn(n, in_f, device=dev) * 2.0).requires_grad_(True)
    gy = torch.randn(n, out_f, device=dev) * 0.05
    y = layer(x)
    y.backward(gy)
    want_y, x_i8, s_x = fl.forward(x.detach(), layer.w_i8, layer.s_w, layer.bias.detach() if bias else None)
    gx, gw, gb = fl.backward(gy, x_i8, layer.w_i8, layer.s_w, s_x, bias)
    assert torch.equal(y.detach(), want_y)
    assert torch.equal(x.grad, gx)
    assert torch.equal(layer._grad_w, gw)
    if bias:
        assert torch.equal(layer.bias.grad, gb)


def test_int8_linear_trains_with_eco_optimizers():
    """A two-layer Int8Linear net learns a separable task with each fp32-state optimizer."""
    from ecoint8 import EcoAdam, EcoSGDM
    from ecoint8.layers import Int8Linear

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    X = torch.randn(512, 32, device=dev, generator=gen)
    y = (X[:, 0] + X[:, 1] > 0).long()
    for make in (lambda ls: EcoSGDM(ls, lr=0.5, momentum=0.9), lambda ls: EcoAdam(ls, lr=2e-2)):
        torch.manual_seed(1)
        l1, l2 = Int8Linear(32, 64).to(dev), Int8Linear(64, 2).to(dev)
        opt = make([l1, l2])
        for _ in range(60):
            logits = l2(torch.relu(l1(X)))
            loss = torch.nn.functional.cross_entropy(logits, y)
            loss.backward()
            opt.step()
            opt.zero_grad()
        acc = (l2(torch.relu(l1(X))).argmax(1) == y).float().mean().item()
        assert acc > 0.85, (type(opt).__name__, acc)
        assert opt.stats["mean_abs_e"] > 0.0


def test_dynamic_quantization_over_many_scales():
    """``quantize_tensor_dynamic`` divides by the Python scalar ``s + EPS``; PyTorch's CUDA
    kernel multiplies by that scalar's reciprocal taken in double and rounded to fp32, which
    differs from the fp32 quotient ``1.0f / float(s + EPS)`` for about a quarter of all
    scales.  Sixty-four tensors with spread-out maxima pin the device quantizer to it."""
    from ecoint8 import _ops
    from oracle import float_layers as fl

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(11)
    for i in range(64):
        x = torch.randn(37, 129, device=dev, generator=gen) * (10.0 ** (i / 16.0 - 2.0))
        q, s = _ops.quantize_dynamic(x)
        want_q, want_s = fl.quantize_tensor_dynamic(x)
        assert s.value() == want_s
        assert torch.equal(q, want_q), i
