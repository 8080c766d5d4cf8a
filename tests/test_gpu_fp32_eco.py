"""EcoSGDM / EcoAdam on the fused B200 kernels against the reference's own PyTorch
arithmetic run on the same GPU (``oracle/fp32_eco.py``, the op-by-op restatement that
``tests/test_oracle_golden.py`` pins to the reference).

Replay mode consumes ``torch.rand_like`` draws like the reference, so the int8 weights,
the fp32 moments and the gradient norms must agree bit for bit; the statistic
``mean_abs_e`` is a double sum here and an fp32 mean there (relative 1e-6).  Where clipping
is active the norm decides the clip factor: the test checks the kernel's norm against
PyTorch's ``g.norm()`` (within 2 ulp) and hands the kernel's value to the oracle, so
everything downstream of it is compared exactly.  Philox mode is checked against the
oracle fed the library's Philox uniforms (``oracle/philox.py``).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(96, 160), (700, 1000), (33, 70)]  # (out, in): one layer spans 11 tiles; one has odd widths


def _layers(dev, seed):
    from ecoint8.layers import Int8Linear

    torch.manual_seed(seed)
    return [Int8Linear(i, o).to(dev) for (o, i) in SHAPES]


def _grads(layers, gen, scale=0.02):
    return [torch.randn(l.w_i8.shape, generator=gen, device=l.w_i8.device) * scale for l in layers]


def _run(kind, wd, clip, steps=3, nan_layer=None):
    from ecoint8 import eco, sr_replay
    from oracle import fp32_eco

    dev = torch.device("cuda", 0)
    layers = _layers(dev, 3)
    ref_w = [l.w_i8.clone() for l in layers]
    s_fixed = [l.s_w.clone() for l in layers]
    ref_m = [torch.zeros_like(w, dtype=torch.float32) for w in ref_w]
    ref_v = [torch.zeros_like(m) for m in ref_m]
    if kind == "sgdm":
        opt = eco.EcoSGDM(layers, lr=0.05, momentum=0.9, weight_decay=wd, grad_clip=clip)
    else:
        opt = eco.EcoAdam(layers, lr=1e-3, weight_decay=wd, grad_clip=clip)
    gen = torch.Generator(device=dev).manual_seed(17)
    for t in range(1, steps + 1):
        grads = _grads(layers, gen)
        if nan_layer is not None:
            grads[nan_layer][3, 5] = float("nan")
        for l, g in zip(layers, grads):
            l._grad_w = g
        rng = torch.cuda.get_rng_state(dev)
        with sr_replay():
            opt.step()
        norms = opt.last_norms()
        torch.cuda.set_rng_state(rng, dev)
        tot, n_e = 0.0, 0
        for i, (l, g) in enumerate(zip(layers, grads)):
            wf = ref_w[i].float() * l.s_w
            finite = bool(torch.isfinite(g).all())
            u = torch.rand_like(g) if finite else None  # the reference's draw order
            norm = None
            if finite:
                n_torch = g.norm().item()
                n_ours = norms[i]
                assert abs(n_ours - n_torch) <= 2 * float(np.spacing(np.float32(n_torch))), (n_ours, n_torch)
                norm = n_ours if clip is not None and max(n_ours, n_torch) > clip else None
            if kind == "sgdm":
                w, m, e_mean, ok, _ = fp32_eco.sgdm_layer(ref_w[i], l.s_w, s_fixed[i], ref_m[i], g, u, lr=0.05,
                                                          beta=0.9, wd=wd, grad_clip=clip, norm=norm)
            else:
                w, m, v, e_mean, ok, _ = fp32_eco.adam_layer(ref_w[i], l.s_w, s_fixed[i], ref_m[i], ref_v[i], g, u,
                                                             t=t, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=wd,
                                                             grad_clip=clip, norm=norm)
                ref_v[i] = v
            assert ok == finite
            ref_w[i], ref_m[i] = w, m
            if ok:
                tot += e_mean
                n_e += 1
        for i, l in enumerate(layers):
            assert torch.equal(l.w_i8, ref_w[i]), (kind, t, i)
            assert torch.equal(opt.m[i], ref_m[i]), (kind, t, i)
            if kind == "adam":
                assert torch.equal(opt.v[i], ref_v[i]), (kind, t, i)
        assert opt.stats["mean_abs_e"] == pytest.approx(tot / n_e, rel=1e-6)
        opt.zero_grad()


@pytest.mark.parametrize("kind", ["sgdm", "adam"])
@pytest.mark.parametrize("wd,clip", [(0.0, 1.0), (0.01, None), (0.0, 0.05), (0.01, 0.05)])
def test_replay_equals_reference_arithmetic(kind, wd, clip):
    _run(kind, wd, clip)


@pytest.mark.parametrize("kind", ["sgdm", "adam"])
def test_non_finite_gradient_leaves_the_layer(kind):
    _run(kind, 0.0, 1.0, steps=2, nan_layer=1)


def test_philox_mode_equals_oracle_on_the_library_uniforms():
    from ecoint8 import _sr, eco
    from oracle import fp32_eco
    from oracle import philox as oph

    dev = torch.device("cuda", 0)
    layers = _layers(dev, 4)
    ref_w = [l.w_i8.clone() for l in layers]
    s_fixed = [l.s_w.clone() for l in layers]
    ref_m = [torch.zeros_like(w, dtype=torch.float32) for w in ref_w]
    opt = eco.EcoSGDM(layers, lr=0.05, momentum=0.9)
    gen = torch.Generator(device=dev).manual_seed(5)
    _sr.set_generator(torch.Generator().manual_seed(44))
    try:
        for _ in range(2):
            grads = _grads(layers, gen)
            for l, g in zip(layers, grads):
                l._grad_w = g
            opt.step()
            key = opt._last_key
            norms = opt.last_norms()  # the clip factor of the 700 x 1000 layer comes from its norm
            for i, (l, g) in enumerate(zip(layers, grads)):
                rows, cols = l.w_i8.shape
                field = oph.sr_field(key, i, np.arange(rows, dtype=np.uint64)[:, None],
                                     np.arange(cols, dtype=np.uint64)[None, :])
                u = torch.from_numpy((field >> np.uint64(8)).astype(np.float32) * np.float32(2.0 ** -24)).to(dev)
                w, m, _, ok, _ = fp32_eco.sgdm_layer(ref_w[i], l.s_w, s_fixed[i], ref_m[i], g, u, lr=0.05, beta=0.9,
                                                     norm=norms[i])
                ref_w[i], ref_m[i] = w, m
                assert torch.equal(l.w_i8, w)
                assert torch.equal(opt.m[i], m)
            opt.zero_grad()
    finally:
        _sr.set_generator(None)
