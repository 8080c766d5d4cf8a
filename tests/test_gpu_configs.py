"""Parity at the benchmark configurations' own sizes (configs 3, 4 and 5), on a B200.

* Config 5 widths (I8Linear(8192, 8192) + I8ReLU + I8Linear(8192, 1000)):
  - replay mode against the reference's own run (tests/golden/wide_train.json, two
    training steps at batch 64, every SR site consuming the reference's torch.randint
    draws), digests of every tensor and the scales bit for bit;
  - Philox mode at batch 256, two training steps, against the oracle fed the logged
    keys; the same run with the backward queued on the device (device-side scales,
    the path the benchmark runs) must give the same state bit for bit.
* Config 3 (isolated GEMM + fused requant, int8 U[-127, 127], per-column ratios
  log-uniform in [1e-4, 1e-1], stochastic rounding): the fused forward kernel
  against cuBLASLt's torch._int_mm (the reference's GEMM, padded to multiples of 8 as
  ilayer.py:40-54 does) followed by the reference's requant arithmetic
  (fixedpoint.py:52-76) -- whole tensors at 4096^3 and 4097^3 in Philox and replay
  mode, row blocks at 8192^3 and 16384 x 4097 x 8192 in Philox mode.
* Config 4 (I8ECO.step over 64 layers of 4096 x 4096, w/m/g uniform, lr 0.05,
  momentum 0.9, grad_clip 1.0): one launch for all 64 layers; the first and last
  layers against the oracle with the logged key.
"""

import hashlib

import numpy as np
import pytest
import torch

from oracle import boundary as bnd
from oracle import fixedpoint as ofp
from oracle import philox as oph
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


# ----------------------------------------------------------------------------- config 5
def _wide_net():
    from ecoint8 import I8Linear, I8ReLU, I8Sequential

    return I8Sequential(I8Linear(bnd.WIDE_D, bnd.WIDE_D), I8ReLU(), I8Linear(bnd.WIDE_D, bnd.WIDE_C)).cuda()


def test_config5_width_replay_matches_reference(golden):
    import ecoint8
    from ecoint8 import I8ECO

    d = golden("wide_train.json")
    torch.manual_seed(0)
    net = _wide_net()
    assert [digest(l.w_i8) for l in net.int8_layers()] == d["init"]
    with ecoint8.sr_replay():
        X, y = bnd.wide_batch()
        x0, sx0 = bnd.quantize_tensor_dynamic(X, stochastic=False)
        cal, _ = net.calibrate(x0.cuda(), sx0)
        assert digest(cal) == d["calib"]
        assert [fhex(l.sy) for l in net.int8_layers()] == d["sy"]
        x_i8 = net.quantize_input(X)[0].cuda()
        assert digest(x_i8) == d["x_i8"]
        opt = I8ECO(net.int8_layers(), lr=0.05, momentum=0.9)
        for t, st in enumerate(d["steps"]):
            logits, s_out = net.forward_i8(x_i8)
            assert digest(logits) == st["logits"] and fhex(s_out) == st["s_out"], t
            _, g_fp = bnd.ce_grad(logits.cpu(), s_out, y)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            assert digest(g_i8) == st["g"] and fhex(s_g) == st["s_g"], t
            net.backward_i8(g_i8.cuda(), s_g)
            for layer, gw in zip(net.int8_layers(), st["grads"]):
                assert digest(layer._gw_i8) == gw["gw"] and fhex(layer._gw_s) == gw["gw_s"], t
                assert digest(layer._gb_sum) == gw["gb"], t
            opt.step()
            opt.zero_grad()
            s_m = opt.s_m
            for i, (layer, ls) in enumerate(zip(net.int8_layers(), st["layers"])):
                assert digest(layer.w_i8) == ls["w"] and digest(opt.m_i8[i]) == ls["m"], (t, i)
                assert digest(layer.b_acc) == ls["b"] and fhex(s_m[i]) == ls["s_m"], (t, i)
            assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], t


def _wide_philox_run(logged: bool, steps: int = 2, batch: int = 256):
    """Two Philox-mode training steps at config-5 widths; with ``logged`` the site log is
    kept (layer-by-layer backward, host scales), else the backward is queued."""
    import ecoint8
    from ecoint8 import I8ECO, _sr

    torch.manual_seed(12)
    net = _wide_net()
    gen = torch.Generator().manual_seed(13)
    X = torch.randn(batch, bnd.WIDE_D, generator=gen)
    yl = torch.randint(0, bnd.WIDE_C, (batch,), generator=gen)
    with ecoint8.sr_replay():
        x0, sx0 = bnd.quantize_tensor_dynamic(X)
        net.calibrate(x0.cuda(), sx0)
    init = [(l.w_i8.cpu().numpy(), list(l.sw), l.b_acc.cpu().numpy(), l.sx, l.sy) for l in net.int8_layers()]
    opt = I8ECO(net.int8_layers(), lr=0.05, momentum=0.9)
    x_i8 = net.quantize_input(X.cuda())[0]
    logs, trail = [], []
    for _ in range(steps):
        _sr.LOG = [] if logged else None
        logits, s_out = net.forward_i8(x_i8)
        _, g_fp = bnd.ce_grad(logits.cpu(), s_out, yl)
        g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
        net.backward_i8(g_i8.cuda(), s_g)
        opt.step()
        opt.zero_grad()
        logs.append((_sr.LOG, logits.cpu().numpy(), s_out, g_i8.numpy(), s_g))
        _sr.LOG = None
        trail.append(([l.w_i8.cpu().numpy() for l in net.int8_layers()], [m.cpu().numpy() for m in opt.m_i8],
                      [l.b_acc.cpu().numpy() for l in net.int8_layers()], list(opt.s_m), opt.stats["mean_abs_e"]))
    return init, x_i8.cpu().numpy(), logs, trail


def test_config5_width_philox_two_steps_equal_oracle_and_queued_backward():
    init, x_i8, logs, trail = _wide_philox_run(logged=True)
    ol = []
    for w, sw, b, sx, sy in init:
        o = ost.I8Linear(w, sw, 4.0, True, b)
        o.sx, o.sy = sx, sy
        ol.append(o)
    onet = ost.I8Sequential(ol[0], ost.I8ReLU(), ol[1])
    oopt = ost.I8ECO(ol, lr=0.05, momentum=0.9)
    for t, ((log, logits, s_out, g_i8, s_g), (ws, ms, bs, s_m, mae)) in enumerate(zip(logs, trail)):
        req = [e for e in log if e[0] not in ("i8eco_step", "none")]
        step = [e for e in log if e[0] == "i8eco_step"][0]
        draws = ost.ListDraws([oph.sr_nudge(k, s, sh, shift, rb) for (_, k, s, sh, shift, rb) in req])
        ologits, os_out = onet.forward_i8(x_i8, draws)
        assert np.array_equal(ologits, logits) and os_out == s_out, t
        onet.backward_i8(g_i8, s_g, draws)
        oopt.step(philox=(step[1], {i: (a, b) for i, a, b in step[2]}))
        oopt.zero_grad()
        for i, o in enumerate(ol):
            assert np.array_equal(ws[i], o.w_i8), (t, i)
            assert np.array_equal(ms[i], oopt.m_i8[i]), (t, i)
            assert np.array_equal(bs[i], o.b_acc), (t, i)
            assert s_m[i] == oopt.s_m[i], (t, i)
        assert mae == oopt.stats["mean_abs_e"], t
    # the queued backward (scales on the device) draws the same keys: the same state
    _, _, _, trail_q = _wide_philox_run(logged=False)
    for (ws, ms, bs, s_m, mae), (wq, mq, bq, s_mq, maeq) in zip(trail, trail_q):
        assert all(np.array_equal(a, b) for a, b in zip(ws + ms + bs, wq + mq + bq))
        assert s_m == s_mq and mae == maeq


# ----------------------------------------------------------------------------- config 3
def _ratios(n, gen):
    lo, hi = np.log(1e-4), np.log(1e-1)
    return [float(v) for v in np.exp(lo + (hi - lo) * torch.rand(n, dtype=torch.float64, generator=gen).numpy())]


def _int_mm_reference(x, w):
    """torch._int_mm (cuBLASLt) with the reference's zero padding (ilayer.py:40-54)."""
    M, K = x.shape
    N = w.shape[0]
    M8, K8, N8 = max(32, -(-M // 8) * 8), -(-K // 8) * 8, -(-N // 8) * 8
    xa = torch.nn.functional.pad(x, (0, K8 - K, 0, M8 - M))
    wa = torch.nn.functional.pad(w, (0, K8 - K, 0, N8 - N))
    return torch._int_mm(xa, wa.t())[:M, :N]


def _requant_reference(acc, bias, mults, com, nudge):
    """sat8(floor(((acc + bias) * mult + nudge) / 2^com)) in int64 (fixedpoint.py:52-82)."""
    a = (acc.to(torch.int64) + bias.to(torch.int64)).to(torch.int32).to(torch.int64)  # int32 wrap
    y = torch.div(a * mults.to(torch.int64) + nudge, 1 << com, rounding_mode="floor")
    return torch.clamp(y, -127, 127).to(torch.int8)


@pytest.mark.parametrize("M,N,K,full", [(4096, 4096, 4096, True), (4097, 4097, 4097, True),
                                        (8192, 8192, 8192, False), (16384, 4097, 8192, False)])
def test_config3_fused_forward_matches_cublas_and_reference_requant(M, N, K, full):
    from ecoint8 import _native, _ops, _sr
    from ecoint8.fixedpoint import quantize_multiplier

    gen = torch.Generator().manual_seed(M + 3 * N + 7 * K)
    x = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=gen).cuda()
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=gen).cuda()
    bias = torch.randint(-50000, 50000, (N,), dtype=torch.int32, generator=gen).cuda()
    ms = [quantize_multiplier(r) for r in _ratios(N, gen)]
    com = min(s for _, s in ms)
    mults = torch.tensor([m >> (s - com) for m, s in ms], dtype=torch.int32).cuda()
    key = 0x1234567 + M
    site = _sr.Site(_native.sr_spec(_native.SR_PHILOX, seed=key, stream_id=0), None)
    y = _ops.gemm_requant(x, 0, w, 0, M, N, K, bias, mults, com, False, site)
    acc = _int_mm_reference(x, w)
    blocks = [(0, M)] if full else [(0, 32), (M // 2 - 16, M // 2 + 16), (M - 32, M)]
    for lo, hi in blocks:
        nud = torch.from_numpy(oph.sr_nudge(key, 0, (hi - lo, N), com, row_base=lo)).cuda()
        want = _requant_reference(acc[lo:hi], bias, mults, com, nud)
        assert torch.equal(y[lo:hi], want), (M, N, K, lo)
    if full:  # replay mode: the reference's own torch.randint draw
        nud = torch.randint(0, 1 << com, (M, N), dtype=torch.int64 if com > 31 else torch.int32,
                            generator=gen).cuda()
        rsite = _sr.Site(_native.sr_spec(_native.SR_REPLAY64 if nud.dtype == torch.int64 else _native.SR_REPLAY32,
                                          nud), nud)
        y = _ops.gemm_requant(x, 0, w, 0, M, N, K, bias, mults, com, False, rsite)
        assert torch.equal(y, _requant_reference(acc, bias, mults, com, nud.to(torch.int64)))


# ----------------------------------------------------------------------------- config 4
def test_config4_step_over_64_layers_of_4096():
    from ecoint8 import I8ECO, I8Linear, _ops, _sr

    dim, n = 4096, 64
    gen = torch.Generator().manual_seed(44)
    torch.manual_seed(45)
    proto = I8Linear(dim, dim)
    layers = []
    for _ in range(n):
        l = I8Linear(1, 1)
        l.w_i8 = torch.randint(-127, 128, (dim, dim), dtype=torch.int8, generator=gen).cuda()
        l.b_acc = torch.zeros(dim, dtype=torch.int32).cuda()
        l.sw = list(proto.sw)
        l.sx = 0.01
        l._gw_i8 = torch.randint(-127, 128, (dim, dim), dtype=torch.int8, generator=gen).cuda()
        l._gw_s = 2e-4
        l._gb_sum = torch.randint(-10 ** 6, 10 ** 6, (dim,), dtype=torch.int64, generator=gen).cuda()
        l._gb_s = 1e-4
        layers.append(l)
    check = {0: None, n - 1: None}
    for i in check:
        l = layers[i]
        o = ost.I8Linear(l.w_i8.cpu().numpy(), list(l.sw), 4.0, True, l.b_acc.cpu().numpy())
        o.sx, o._gw_i8, o._gw_s = l.sx, l._gw_i8.cpu().numpy(), l._gw_s
        o._gb_sum, o._gb_s = l._gb_sum.cpu().numpy(), l._gb_s
        check[i] = o
    opt = I8ECO(layers, lr=0.05, momentum=0.9, grad_clip=1.0)
    ms = {}
    for i, m in enumerate(opt.m_i8):
        m.copy_(torch.randint(-127, 128, m.shape, dtype=torch.int8, generator=gen))
        if i in check:
            ms[i] = m.cpu().numpy()
    opt.s_m = [3e-4] * n
    _sr.LOG = []
    opt.step()
    log, _sr.LOG = _sr.LOG, None
    _, seed, streams = [e for e in log if e[0] == "i8eco_step"][0]
    streams = {i: (a, b) for i, a, b in streams}
    s_m = opt.s_m
    for i, o in check.items():
        oopt = ost.I8ECO([o], lr=0.05, momentum=0.9, grad_clip=1.0)
        oopt.m_i8[0][...] = ms[i]
        oopt.s_m = [3e-4]
        oopt.step(philox=(seed, {0: streams[i]}))
        assert np.array_equal(layers[i].w_i8.cpu().numpy(), o.w_i8), i
        assert np.array_equal(opt.m_i8[i].cpu().numpy(), oopt.m_i8[0]), i
        assert np.array_equal(layers[i].b_acc.cpu().numpy(), o.b_acc), i
        assert s_m[i] == oopt.s_m[0], i
