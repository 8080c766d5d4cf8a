"""A training step captured as a CUDA graph (``ecoint8.graphs.StepGraph``) and replayed
makes exactly the steps the uncaptured calls make.

The same net, data and Philox generator are trained twice: once eagerly, once as one
warm-up step plus graph replays, with the learning rate changed before every step
(a cosine schedule: the replayed I8ECO step reads it from the graph's table).  Every
weight, momentum, bias accumulator, momentum scale, statistic and loss must agree
bit for bit.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

B, D, H, C = 192, 64, 128, 16
STEPS = 6


def _setup(seed=0):
    from ecoint8 import I8ECO, I8Linear, I8ReLU, I8Sequential
    from ecoint8._sr import set_generator
    from ecoint8.quant import quantize_tensor_dynamic

    dev = torch.device("cuda", 0)
    torch.manual_seed(seed)
    net = I8Sequential(I8Linear(D, H), I8ReLU(), I8Linear(H, H), I8ReLU(), I8Linear(H, C)).to(dev)
    gen = torch.Generator().manual_seed(5)
    X = torch.randn(B, D, generator=gen) * 1.5
    Y = torch.randint(0, C, (B,), generator=gen)
    x8, sx = quantize_tensor_dynamic(X)
    set_generator(torch.Generator().manual_seed(99))
    net.calibrate(x8.to(dev), sx)
    opt = I8ECO(net.int8_layers(), lr=0.3, momentum=0.9)
    return net, opt, x8.to(dev), Y.to(dev)


def _step_fn(net, opt, x8, y):
    from ecoint8.quant import cross_entropy_grad_i8

    def step():
        logits, s_out = net.forward_i8(x8)
        loss, g8, s_g = cross_entropy_grad_i8(logits, s_out, y)
        net.backward_i8(g8, s_g)
        opt.step()
        opt.zero_grad()
        return loss

    return step


def _lr(t):
    return 0.3 * (0.55 + 0.45 * math.cos(math.pi * t / STEPS))


def _state(net, opt):
    return ([l.w_i8.clone() for l in net.int8_layers()], [m.clone() for m in opt.m_i8],
            [l.b_acc.clone() for l in net.int8_layers()], list(opt.s_m), dict(opt.stats), opt.step_count)


def test_replayed_steps_equal_eager_steps():
    from ecoint8._sr import set_generator
    from ecoint8.graphs import StepGraph

    try:
        net, opt, x8, y = _setup()
        step = _step_fn(net, opt, x8, y)
        eager_losses = []
        for t in range(STEPS):
            opt.set_lr(_lr(t))
            eager_losses.append(float(step().item()))
        eager = _state(net, opt)

        net, opt, x8, y = _setup()
        g = StepGraph(_step_fn(net, opt, x8, y), warmup=1)
        opt.set_lr(_lr(0))
        losses = [float(g.capture().item())]
        for t in range(1, STEPS):
            opt.set_lr(_lr(t))
            losses.append(float(g.replay().item()))
        torch.cuda.synchronize()
        graphed = _state(net, opt)
        assert g.keys_per_step > 0
    finally:
        set_generator(None)
    assert losses == eager_losses
    for a, b in zip(graphed[0], eager[0]):
        assert torch.equal(a, b)
    for a, b in zip(graphed[1], eager[1]):
        assert torch.equal(a, b)
    for a, b in zip(graphed[2], eager[2]):
        assert torch.equal(a, b)
    assert graphed[3] == eager[3]
    assert graphed[4] == eager[4]
    assert graphed[5] == eager[5] == STEPS


def test_capture_rejects_replay_mode():
    from ecoint8 import sr_replay
    from ecoint8._sr import set_generator
    from ecoint8.graphs import StepGraph

    try:
        net, opt, x8, y = _setup()
        g = StepGraph(_step_fn(net, opt, x8, y))
        with sr_replay():
            with pytest.raises(RuntimeError, match="Philox"):
                g.capture()
    finally:
        set_generator(None)
