"""The strict int8 training path on a B200 against the reference, bit for bit.

* Replay mode: every stochastic-rounding site consumes the reference's own
  ``torch.randint`` draws (CPU generator), so the drop-in must reproduce the
  golden digests recorded from the reference (tests/golden/*.json), step by
  step, including the reference's ValueError at the blob task's last epoch.
* Philox mode: the CUDA path must equal the oracle fed the same Philox stream.
* The reference's own tests (tests/test_strict.py) rerun on CUDA tensors.
"""

import copy
import hashlib

import numpy as np
import pytest
import torch

from oracle import boundary as bnd
from oracle import strict as ost

pytestmark = pytest.mark.gpu


def digest(t) -> str:
    a = np.ascontiguousarray(t.detach().cpu().numpy() if hasattr(t, "detach") else t)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode() + str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()[:24]


def fhex(v):
    return float(v).hex()


def _blob_net():
    from ecoint8 import I8Linear, I8ReLU, I8Sequential

    torch.manual_seed(0)
    X, y = bnd.blob_data()
    net = I8Sequential(I8Linear(bnd.BLOB_D, bnd.BLOB_H), I8ReLU(), I8Linear(bnd.BLOB_H, 2)).cuda()
    return X, y, net


def test_blob_training_replay_matches_reference_every_step(golden):
    """The 32-64-2 blob task (150 epochs, cosine lr, I8ECO lr 0.5 momentum 0.9)."""
    import ecoint8
    from ecoint8 import I8ECO

    d = golden("blob_train.json")
    X, y, net = _blob_net()
    for layer, ini in zip(net.int8_layers(), d["init"]):
        assert digest(layer.w_i8) == ini["w"] and [fhex(v) for v in layer.sw] == ini["sw"]
    with ecoint8.sr_replay():
        x0, sx0 = bnd.quantize_tensor_dynamic(X, stochastic=False)
        cal, s = net.calibrate(x0.cuda(), sx0)
        assert digest(cal) == d["calib"]["logits"] and fhex(s) == d["calib"]["s"]
        x_i8 = net.quantize_input(X)[0].cuda()  # fp32 boundary on the CPU, as recorded
        assert digest(x_i8) == d["x_i8"]
        opt = I8ECO(net.int8_layers(), lr=0.5, momentum=0.9)
        err = d["error"]
        for ep, st in enumerate(d["steps"] + ([None] if err else [])):
            opt.set_lr(bnd.blob_lr(ep))
            logits, s_out = net.forward_i8(x_i8)
            loss, g_fp = bnd.ce_grad(logits.cpu(), s_out, y)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            net.backward_i8(g_i8.cuda(), s_g)
            if st is None:
                assert ep == err["epoch"]
                with pytest.raises(ValueError):
                    opt.step()
                break
            assert digest(logits) == st["logits"] and fhex(s_out) == st["s_out"], ep
            for layer, gw in zip(net.int8_layers(), st["grads"]):
                assert digest(layer._gw_i8) == gw["gw"] and fhex(layer._gw_s) == gw["gw_s"], ep
                assert digest(layer._gb_sum) == gw["gb"], ep
            opt.step()
            opt.zero_grad()
            s_m = opt.s_m
            for i, (layer, ls) in enumerate(zip(net.int8_layers(), st["layers"])):
                assert digest(layer.w_i8) == ls["w"], (ep, i)
                assert digest(opt.m_i8[i]) == ls["m"], (ep, i)
                assert digest(layer.b_acc) == ls["b"], (ep, i)
                assert fhex(s_m[i]) == ls["s_m"], (ep, i)
            assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], ep


def test_mnist_shaped_replay_matches_reference(golden):
    """784-256-128-10 at batch 128 (the MNIST-shaped config): its 5 epochs (2345 steps), every step bit-exact."""
    import ecoint8
    from ecoint8 import I8ECO, I8Linear, I8ReLU, I8Sequential

    d = golden("mnist_train.json")
    torch.manual_seed(0)
    d0, d1, d2, d3 = bnd.MNIST_SHAPE
    net = I8Sequential(I8Linear(d0, d1), I8ReLU(), I8Linear(d1, d2), I8ReLU(), I8Linear(d2, d3)).cuda()
    with ecoint8.sr_replay():
        X0, _ = bnd.mnist_batch(0)
        x0, sx0 = bnd.quantize_tensor_dynamic(X0, stochastic=False)
        net.calibrate(x0.cuda(), sx0)
        opt = I8ECO(net.int8_layers(), lr=bnd.mnist_lr(0, bnd.MNIST_GOLDEN_STEPS), momentum=0.9)
        for t, st in enumerate(d["steps"]):
            X, y = bnd.mnist_batch(t)
            opt.set_lr(bnd.mnist_lr(t, bnd.MNIST_GOLDEN_STEPS))
            x_i8 = net.quantize_input(X)[0].cuda()
            logits, s_out = net.forward_i8(x_i8)
            assert digest(logits) == st["logits"], t
            loss, g_fp = bnd.ce_grad(logits.cpu(), s_out, y)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            assert digest(g_i8) == st["g"], t
            net.backward_i8(g_i8.cuda(), s_g)
            opt.step()
            opt.zero_grad()
            s_m = opt.s_m
            for i, (layer, ls) in enumerate(zip(net.int8_layers(), st["layers"])):
                assert digest(layer.w_i8) == ls["w"] and digest(opt.m_i8[i]) == ls["m"], (t, i)
                assert digest(layer.b_acc) == ls["b"] and fhex(s_m[i]) == ls["s_m"], (t, i)
            assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], t


def test_standalone_step_replay_matches_reference(golden):
    """I8ECO.step alone (3 layers, one without bias, chunk_rows=16), three steps."""
    import ecoint8
    from ecoint8 import I8ECO, I8Linear

    d = golden("eco_step.json")
    torch.manual_seed(5)
    layers = [I8Linear(96, 64), I8Linear(64, 130, bias=False), I8Linear(130, 3)]
    for l in layers:
        l.cuda()
        l.sx = 0.02
    opt = I8ECO(layers, lr=0.05, momentum=0.9, chunk_rows=16)
    for step, st in enumerate(d):
        torch.manual_seed(100 + step)
        for l in layers:
            l._gw_i8 = torch.randint(-127, 128, l.w_i8.shape, dtype=torch.int8).cuda()
            l._gw_s = 3e-4 * (step + 1)
            l._gb_sum = torch.randint(-5000, 5000, (l.w_i8.shape[0],), dtype=torch.int64).cuda()
            l._gb_s = 2e-3
        if step == 0:
            for m in opt.m_i8:
                m.copy_(torch.randint(-127, 128, m.shape, dtype=torch.int8))
            opt.s_m = [1e-3, 5e-4, 2e-3]
        torch.manual_seed(200 + step)
        with ecoint8.sr_replay():
            opt.step()
        s_m = opt.s_m
        for i, (l, ls) in enumerate(zip(layers, st["layers"])):
            assert digest(l.w_i8) == ls["w"] and digest(opt.m_i8[i]) == ls["m"], (step, i)
            assert digest(l.b_acc) == ls["b"] and fhex(s_m[i]) == ls["s_m"], (step, i)
        assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], step


def _oracle_copy(net):
    layers = []
    for l in net.int8_layers():
        o = ost.I8Linear(l.w_i8.cpu().numpy(), list(l.sw), l.headroom, l.use_bias, l.b_acc.cpu().numpy())
        o.sx, o.sy = l.sx, l.sy
        layers.append(o)
    return layers


def test_philox_mode_equals_oracle_on_same_stream():
    """Default (Philox) mode, 4 training steps of a 20-48-16-3 net with biases; the oracle
    rebuilds every nudge from the logged keys (oracle/philox.py) and must agree exactly."""
    import ecoint8
    from ecoint8 import I8ECO, I8Linear, I8ReLU, I8Sequential, _sr

    torch.manual_seed(3)
    net = I8Sequential(I8Linear(20, 48), I8ReLU(), I8Linear(48, 16), I8ReLU(), I8Linear(16, 3)).cuda()
    X = torch.randn(96, 20)
    yl = torch.randint(0, 3, (96,))
    with ecoint8.sr_replay():
        x0, sx0 = bnd.quantize_tensor_dynamic(X)
        net.calibrate(x0.cuda(), sx0)
    ol = _oracle_copy(net)
    onet = ost.I8Sequential(ol[0], ost.I8ReLU(), ol[1], ost.I8ReLU(), ol[2])
    opt = I8ECO(net.int8_layers(), lr=0.3, momentum=0.9)
    oopt = ost.I8ECO(ol, lr=0.3, momentum=0.9)
    x_i8 = net.quantize_input(X.cuda())[0]
    from oracle import philox as oph

    for t in range(4):
        _sr.LOG = []
        logits, s_out = net.forward_i8(x_i8)
        _, g_fp = bnd.ce_grad(logits.cpu(), s_out, yl)
        g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
        net.backward_i8(g_i8.cuda(), s_g)
        opt.step()
        opt.zero_grad()
        log, _sr.LOG = _sr.LOG, None
        req = [e for e in log if e[0] not in ("i8eco_step", "none")]
        step = [e for e in log if e[0] == "i8eco_step"][0]
        draws = ost.ListDraws([oph.sr_nudge(k, s, sh, shift, rb) for (_, k, s, sh, shift, rb) in req])
        ologits, os_out = onet.forward_i8(x_i8.cpu().numpy(), draws)
        assert np.array_equal(ologits, logits.cpu().numpy()) and os_out == s_out, t
        onet.backward_i8(g_i8.numpy(), s_g, draws)
        oopt.step(philox=(step[1], {i: (sw_, sb_) for i, sw_, sb_ in step[2]}))
        oopt.zero_grad()
        s_m = opt.s_m
        for i, (l, o) in enumerate(zip(net.int8_layers(), ol)):
            assert np.array_equal(l.w_i8.cpu().numpy(), o.w_i8), (t, i)
            assert np.array_equal(opt.m_i8[i].cpu().numpy(), oopt.m_i8[i]), (t, i)
            assert np.array_equal(l.b_acc.cpu().numpy(), o.b_acc), (t, i)
            assert s_m[i] == oopt.s_m[i], (t, i)
        assert opt.stats["mean_abs_e"] == oopt.stats["mean_abs_e"], t


def test_step_at_4096_rows_equals_oracle_philox():
    """One 4096x4096 layer plus a 1000x4096 layer (config-4 / config-5 widths)."""
    from ecoint8 import I8ECO, I8Linear, _sr

    torch.manual_seed(11)
    layers = [I8Linear(4096, 4096), I8Linear(4096, 1000)]
    gen = torch.Generator().manual_seed(4)
    for l in layers:
        l.cuda()
        l.sx = 0.01
        l._gw_i8 = torch.randint(-127, 128, l.w_i8.shape, dtype=torch.int8, generator=gen).cuda()
        l._gw_s = 1e-5
        l._gb_sum = torch.randint(-10 ** 6, 10 ** 6, (l.w_i8.shape[0],), dtype=torch.int64, generator=gen).cuda()
        l._gb_s = 1e-4
    ol = []
    for l in layers:
        o = ost.I8Linear(l.w_i8.cpu().numpy(), list(l.sw), l.headroom, True, l.b_acc.cpu().numpy())
        o.sx = l.sx
        o._gw_i8, o._gw_s = l._gw_i8.cpu().numpy(), l._gw_s
        o._gb_sum, o._gb_s = l._gb_sum.cpu().numpy(), l._gb_s
        ol.append(o)
    opt = I8ECO(layers, lr=0.05, momentum=0.9)
    oopt = ost.I8ECO(ol, lr=0.05, momentum=0.9)
    for m, om in zip(opt.m_i8, oopt.m_i8):
        mm = torch.randint(-127, 128, m.shape, dtype=torch.int8, generator=gen)
        m.copy_(mm)
        om[...] = mm.numpy()
    opt.s_m = [2e-4, 3e-4]
    oopt.s_m = [2e-4, 3e-4]
    _sr.LOG = []
    opt.step()
    log, _sr.LOG = _sr.LOG, None
    step = [e for e in log if e[0] == "i8eco_step"][0]
    oopt.step(philox=(step[1], {i: (a, b) for i, a, b in step[2]}))
    s_m = opt.s_m
    for i, (l, o) in enumerate(zip(layers, ol)):
        assert np.array_equal(l.w_i8.cpu().numpy(), o.w_i8), i
        assert np.array_equal(opt.m_i8[i].cpu().numpy(), oopt.m_i8[i]), i
        assert np.array_equal(l.b_acc.cpu().numpy(), o.b_acc), i
        assert s_m[i] == oopt.s_m[i], i
    assert opt.stats["mean_abs_e"] == oopt.stats["mean_abs_e"]


# -- the reference's own tests (tests/test_strict.py:45-120), on CUDA ---------

def _toy_net():
    from ecoint8 import I8Linear, I8ReLU, I8Sequential

    return I8Sequential(I8Linear(20, 32), I8ReLU(), I8Linear(32, 2)).cuda()


def _data():
    torch.manual_seed(0)
    X = torch.randn(512, 20)
    return X.cuda(), ((X[:, :5].sum(1)) > 0).long().cuda()


def test_reference_state_is_integral():
    from ecoint8 import I8ECO
    from ecoint8.quant import quantize_tensor_dynamic

    net = _toy_net()
    X, y = _data()
    x8, sx = quantize_tensor_dynamic(X, stochastic=False)
    net.calibrate(x8, sx)
    opt = I8ECO(net.int8_layers(), lr=0.5, momentum=0.9)
    for t, p in net.named_buffers():
        assert p.dtype in {torch.int8, torch.int32, torch.int64}, f"buffer {t} is {p.dtype}"
    for m in opt.m_i8:
        assert m.dtype == torch.int8
    assert all(isinstance(s, float) for s in opt.s_m)


def test_reference_layer_matches_fp32():
    from ecoint8 import I8Linear
    from ecoint8.quant import quantize_tensor_dynamic

    torch.manual_seed(1)
    lin = I8Linear(64, 64).cuda()
    ref_w = lin.w_i8.to(torch.float32) * torch.tensor(lin.sw, device=lin.w_i8.device).unsqueeze(1)
    x = torch.randn(32, 64).cuda()
    x8, sx = quantize_tensor_dynamic(x, stochastic=False)
    lin.sx, lin.sy = None, None
    y8, sy = lin.calibrate_forward(x8, sx)
    ref = x @ ref_w.t()
    got = y8.to(torch.float32) * sy
    rel = (got - ref).abs().mean().item() / ref.abs().mean().item()
    assert rel < 0.025 * lin.headroom, f"int8 layer too far from fp32: {rel}"


def test_reference_e2e_trains():
    import torch.nn as nn

    from ecoint8 import I8ECO
    from ecoint8.quant import quantize_symmetric, quantize_tensor_dynamic

    net = _toy_net()
    X, y = _data()
    fn = nn.CrossEntropyLoss()
    x8, sx = quantize_tensor_dynamic(X, stochastic=False)
    net.calibrate(x8, sx)
    opt = I8ECO(net.int8_layers(), lr=0.5, momentum=0.9)
    for _ in range(30):
        logits, s_out = net.forward_i8(x8)
        logits_fp = (logits.to(torch.float32) * s_out).requires_grad_()
        loss = fn(logits_fp, y)
        (g_fp,) = torch.autograd.grad(loss, logits_fp)
        amax = float(g_fp.abs().max().item())
        with torch.no_grad():
            net.backward_i8(quantize_symmetric(g_fp, amax / 127.0, stochastic=True), amax / 127.0)
        opt.step()
        opt.zero_grad()
    acc = (net.forward_i8(x8)[0].argmax(1) == y).float().mean().item()
    assert acc > 0.80, f"strict int8 failed to learn: {acc}"
    for layer in net.int8_layers():
        sat = ((layer.w_i8 == 127) | (layer.w_i8 == -127)).float().mean().item()
        assert sat < 0.05, f"weights saturated at rails: {sat:.3f}"


def test_sequential_fusion_equals_unfused_modules():
    """Linear+ReLU fused in one kernel == calling the modules one by one (same draws)."""
    import ecoint8

    X, y = _data()
    torch.manual_seed(4)
    a = _toy_net()
    b = copy.deepcopy(a)
    from ecoint8.quant import quantize_tensor_dynamic

    x8, sx = quantize_tensor_dynamic(X)
    for net in (a, b):
        torch.manual_seed(5)
        with ecoint8.sr_replay():
            net.calibrate(x8, sx)
    torch.manual_seed(6)
    with ecoint8.sr_replay():
        ya, _ = a.forward_i8(x8)
    torch.manual_seed(6)
    with ecoint8.sr_replay():
        h, _ = b.blocks[0].forward_i8(x8)
        h = b.blocks[1].apply_forward(h)
        yb, _ = b.blocks[2].forward_i8(h)
    assert torch.equal(ya, yb)
    assert torch.equal(a.blocks[1].mask_cache, b.blocks[1].mask_cache)


def test_queued_backward_equals_layer_by_layer():
    """``I8Sequential.backward_i8`` in Philox mode queues the whole pass with the scales
    on the device; the same training run layer by layer (host scales: the site log
    forces it) must give identical weights, momentum, biases, s_m, stats and gradient
    scales after every step.  Widths cover the 16-aligned and the odd-width kernels."""
    from ecoint8 import I8ECO, I8Linear, I8ReLU, I8Sequential, _sr

    def run(logged):
        torch.manual_seed(5)
        net = I8Sequential(I8Linear(64, 256), I8ReLU(), I8Linear(256, 96), I8ReLU(), I8Linear(96, 10)).cuda()
        gen = torch.Generator().manual_seed(9)
        X = torch.randn(128, 64, generator=gen)
        yl = torch.randint(0, 10, (128,), generator=gen)
        x0, sx0 = bnd.quantize_tensor_dynamic(X)
        net.calibrate(x0.cuda(), sx0)
        opt = I8ECO(net.int8_layers(), lr=0.3, momentum=0.9)
        x_i8 = net.quantize_input(X.cuda())[0]
        trail = []
        for _ in range(4):
            _sr.LOG = [] if logged else None
            logits, s_out = net.forward_i8(x_i8)
            _, g_fp = bnd.ce_grad(logits.cpu(), s_out, yl)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            net.backward_i8(g_i8.cuda(), s_g)
            trail.append([fhex(l._gw_s) for l in net.int8_layers()] + [fhex(l._gb_s) for l in net.int8_layers()])
            opt.step()
            opt.zero_grad()
            _sr.LOG = None
            trail.append([digest(l.w_i8) for l in net.int8_layers()] + [digest(m) for m in opt.m_i8]
                         + [digest(l.b_acc) for l in net.int8_layers()] + [fhex(v) for v in opt.s_m]
                         + [fhex(opt.stats["mean_abs_e"])])
        return trail

    assert run(False) == run(True)


def test_checkpoint_resume_equals_uninterrupted_training():
    """torch.save((net, opt)) after two steps, load, two more steps: identical to four
    uninterrupted steps (weights, momentum, biases, s_m)."""
    import io

    from ecoint8 import I8ECO, I8Linear, I8ReLU, I8Sequential

    gen = torch.Generator().manual_seed(21)
    X = torch.randn(64, 32, generator=gen)
    yl = torch.randint(0, 4, (64,), generator=gen)

    def setup():
        torch.manual_seed(8)
        net = I8Sequential(I8Linear(32, 64), I8ReLU(), I8Linear(64, 4)).cuda()
        x0, sx0 = bnd.quantize_tensor_dynamic(X)
        net.calibrate(x0.cuda(), sx0)
        return net, I8ECO(net.int8_layers(), lr=0.3, momentum=0.9), net.quantize_input(X.cuda())[0]

    def train(net, opt, x_i8, steps):
        for _ in range(steps):
            logits, s_out = net.forward_i8(x_i8)
            _, g_fp = bnd.ce_grad(logits.cpu(), s_out, yl)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            net.backward_i8(g_i8.cuda(), s_g)
            opt.step()
            opt.zero_grad()

    net, opt, x_i8 = setup()
    train(net, opt, x_i8, 2)
    buf = io.BytesIO()
    torch.save((net, opt), buf)
    rng = torch.get_rng_state()
    train(net, opt, x_i8, 2)
    want = [l.w_i8.cpu() for l in net.int8_layers()] + [m.cpu() for m in opt.m_i8] + [
        l.b_acc.cpu() for l in net.int8_layers()]
    want_sm = list(opt.s_m)
    buf.seek(0)
    net2, opt2 = torch.load(buf, weights_only=False)
    torch.set_rng_state(rng)  # the Philox keys continue from the same CPU generator state
    train(net2, opt2, x_i8, 2)
    got = [l.w_i8.cpu() for l in net2.int8_layers()] + [m.cpu() for m in opt2.m_i8] + [
        l.b_acc.cpu() for l in net2.int8_layers()]
    assert all(torch.equal(a, b) for a, b in zip(want, got)) and list(opt2.s_m) == want_sm
