"""Pin the CPU oracle to the reference: every golden fixture made by running ecoint8 v0.4.9.

CPU only.  The oracle replays the reference's own draw stream (``TorchDraws``),
so a seeded oracle run must reproduce a seeded reference run bit for bit.
"""

import hashlib
import math

import numpy as np
import pytest
import torch

from oracle import boundary as bnd
from oracle import fixedpoint as ofp
from oracle import philox as oph
from oracle import strict as ost
from oracle import sgdm as osg


def digest(a) -> str:
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode() + str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()[:24]


def fhex(v):
    return float(v).hex()


def test_quantize_multiplier_and_scalars(golden):
    d = golden("fixedpoint.json")
    for r_hex, mult, shift in d["quantize_multiplier"]:
        assert ofp.quantize_multiplier(float.fromhex(r_hex)) == (mult, shift)
    for m, k, n, *exp in d["pad_mm_dims"]:
        assert list(ofp.pad_mm_dims(m, k, n)) == exp
    for a, g_hex, out_hex in d["dynamic_scale_from_int"]:
        assert fhex(ofp.dynamic_scale_from_int(a, float.fromhex(g_hex))) == out_hex
    x, y = d["to_int8_sat"]
    assert ofp.to_int8_sat(np.array(x, dtype=np.int64)).tolist() == y
    x, y = d["int_amax"]
    assert ofp.int_amax(np.array(x, dtype=np.int64)) == y


def test_apply_mult_shift_cases(golden):
    d = golden("fixedpoint.json")
    for case in d["apply_mult_shift"]:
        x = np.array(case["x"], dtype=np.int64)
        mult = case["mult"]
        if not isinstance(mult, int):
            mult = np.array(mult, dtype=np.int32)
        nudge = None if case["nudge"] is None else np.array(case["nudge"], dtype=np.int64)
        out = ofp.apply_mult_shift(x, mult, case["shift"], case["stochastic"], nudge)
        assert out.tolist() == case["out"], case["mult_kind"]
        # the draw log: one [rows, cols] draw iff stochastic and shift >= 0
        exp_draws = ([[list(x.shape), 1 << case["shift"]]]
                     if case["stochastic"] and case["shift"] >= 0 else [])
        assert case["draws"] == exp_draws


def test_int_mm_exact_like_reference_pad8_cases():
    """tests/test_strict.py:76-91 shapes: exact int GEMM, padding-free."""
    torch.manual_seed(0)
    for M, K, N in [(512, 256, 2), (2, 512, 256), (7, 13, 5), (100, 300, 2), (33, 4097, 17)]:
        a = torch.randint(-127, 127, (M, K), dtype=torch.int8)
        b = torch.randint(-127, 127, (K, N), dtype=torch.int8)
        ref = (a.to(torch.int64) @ b.to(torch.int64)).to(torch.int32)
        assert np.array_equal(ofp.int_mm(a.numpy(), b.numpy()), ref.numpy())
        if M > 16:
            assert np.array_equal(ofp.int_mm(a.numpy(), b.numpy()), torch._int_mm(a, b).numpy())


def test_gemm_requant_golden(golden):
    for c in golden("gemm_requant.json"):
        torch.manual_seed(c["seed"])
        a = torch.randint(-127, 128, (c["M"], c["K"]), dtype=torch.int8)
        b = torch.randint(-127, 128, (c["K"], c["N"]), dtype=torch.int8)
        lo = float(torch.log(torch.tensor(1e-4, dtype=torch.float64)))
        hi = float(torch.log(torch.tensor(1e-1, dtype=torch.float64)))
        ratios = [float(v) for v in torch.exp(torch.empty(c["N"], dtype=torch.float64).uniform_(lo, hi))]
        acc = ofp.int_mm(a.numpy(), b.numpy())
        assert digest(acc) == c["acc"]
        if c["stochastic"]:
            y = ost.common_shift_requant(acc, ratios, ost.TorchDraws())
        else:
            mults, com = ofp.col_mults(ratios)
            y = ofp.to_int8_sat(ofp.apply_mult_shift(acc.astype(np.int64), mults, com, False))
        assert digest(y) == c["y"]


def _blob_setup():
    torch.manual_seed(0)
    X, y = bnd.blob_data()
    l0 = ost.I8Linear.seeded(bnd.BLOB_D, bnd.BLOB_H)
    l1 = ost.I8Linear.seeded(bnd.BLOB_H, 2)
    net = ost.I8Sequential(l0, ost.I8ReLU(), l1)
    return X, y, net


def test_blob_training_bit_exact(golden):
    """The 32-64-2 blob task, all 150 epochs: every tensor and scale after every step."""
    d = golden("blob_train.json")
    X, y, net = _blob_setup()
    for layer, ini in zip(net.int8_layers(), d["init"]):
        assert digest(layer.w_i8) == ini["w"]
        assert [fhex(v) for v in layer.sw] == ini["sw"]
    draws = ost.TorchDraws()
    x0, sx0 = bnd.quantize_tensor_dynamic(X, stochastic=False)
    rec = ost.RecordingDraws(draws)
    cal, s = net.calibrate(x0.numpy(), sx0, rec)
    assert digest(cal) == d["calib"]["logits"] and fhex(s) == d["calib"]["s"]
    assert [[list(sh), dn] for sh, dn, _ in rec.log] == d["calib"]["draws"]
    sx = net.int8_layers()[0].sx
    x_i8 = torch.clamp(torch.round(X / sx), -127, 127).to(torch.int8)  # ilayer.py:210-213
    assert digest(x_i8.numpy()) == d["x_i8"]
    x_i8 = x_i8.numpy()
    opt = ost.I8ECO(net.int8_layers(), lr=0.5, momentum=0.9)
    err = d["error"]
    for ep, st in enumerate(d["steps"] + ([None] if err else [])):
        opt.set_lr(bnd.blob_lr(ep))
        rec = ost.RecordingDraws(draws)
        logits, s_out = net.forward_i8(x_i8, rec)
        loss, g_fp = bnd.ce_grad(torch.from_numpy(logits), s_out, y)
        g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
        net.backward_i8(g_i8.numpy(), s_g, rec)
        if st is None:  # the reference raised inside this step
            assert ep == err["epoch"]
            with pytest.raises(ValueError):
                opt.step(rec)
            assert [list(rec.log[-1][0]), rec.log[-1][1]] != err["last_draw"]  # failed draw not logged
            break
        assert digest(logits) == st["logits"] and fhex(s_out) == st["s_out"], ep
        assert digest(g_i8.numpy()) == st["g"] and fhex(s_g) == st["s_g"], ep
        for layer, gw in zip(net.int8_layers(), st["grads"]):
            assert digest(layer._gw_i8) == gw["gw"] and fhex(layer._gw_s) == gw["gw_s"], ep
            assert digest(layer._gb_sum) == gw["gb"], ep
        opt.step(rec)
        opt.zero_grad()
        if ep == 0:
            assert [[list(sh), dn] for sh, dn, _ in rec.log] == d["first_step_draws"]
        for i, (layer, ls) in enumerate(zip(net.int8_layers(), st["layers"])):
            assert digest(layer.w_i8) == ls["w"], (ep, i)
            assert digest(opt.m_i8[i]) == ls["m"], (ep, i)
            assert digest(layer.b_acc) == ls["b"], (ep, i)
            assert fhex(opt.s_m[i]) == ls["s_m"], (ep, i)
        assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], ep
    if err is None:
        for i, layer in enumerate(net.int8_layers()):
            assert layer.w_i8.tolist() == d["final"][f"w{i}"]


def test_mnist_shaped_training_bit_exact(golden):
    d = golden("mnist_train.json")
    torch.manual_seed(0)
    d0, d1, d2, d3 = bnd.MNIST_SHAPE
    net = ost.I8Sequential(ost.I8Linear.seeded(d0, d1), ost.I8ReLU(), ost.I8Linear.seeded(d1, d2),
                           ost.I8ReLU(), ost.I8Linear.seeded(d2, d3))
    draws = ost.TorchDraws()
    X0, _ = bnd.mnist_batch(0)
    x0, sx0 = bnd.quantize_tensor_dynamic(X0, stochastic=False)
    net.calibrate(x0.numpy(), sx0, draws)
    opt = ost.I8ECO(net.int8_layers(), lr=bnd.mnist_lr(0, bnd.MNIST_GOLDEN_STEPS), momentum=0.9)
    sx = net.int8_layers()[0].sx
    for t, st in enumerate(d["steps"][:bnd.MNIST_EPOCH_STEPS]):  # the first epoch; the GPU test runs all 5
        X, y = bnd.mnist_batch(t)
        opt.set_lr(bnd.mnist_lr(t, bnd.MNIST_GOLDEN_STEPS))
        x_i8 = torch.clamp(torch.round(X / sx), -127, 127).to(torch.int8).numpy()
        logits, s_out = net.forward_i8(x_i8, draws)
        assert digest(logits) == st["logits"], t
        loss, g_fp = bnd.ce_grad(torch.from_numpy(logits), s_out, y)
        g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
        assert digest(g_i8.numpy()) == st["g"], t
        net.backward_i8(g_i8.numpy(), s_g, draws)
        opt.step(draws)
        opt.zero_grad()
        for i, (layer, ls) in enumerate(zip(net.int8_layers(), st["layers"])):
            assert digest(layer.w_i8) == ls["w"] and digest(opt.m_i8[i]) == ls["m"], (t, i)
            assert digest(layer.b_acc) == ls["b"] and fhex(opt.s_m[i]) == ls["s_m"], (t, i)
        assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], t


def test_config5_width_first_step_bit_exact(golden):
    """Config 5's widths (I8Linear(8192, 8192) + I8ReLU + I8Linear(8192, 1000)) at batch 1024:
    the oracle reproduces the reference's calibration and first training step (every
    tensor digest and scale; the GPU test replays all three recorded steps)."""
    d = golden("wide_train.json")
    torch.manual_seed(0)
    net = ost.I8Sequential(ost.I8Linear.seeded(bnd.WIDE_D, bnd.WIDE_D), ost.I8ReLU(),
                           ost.I8Linear.seeded(bnd.WIDE_D, bnd.WIDE_C))
    assert [digest(l.w_i8) for l in net.int8_layers()] == d["init"]
    draws = ost.TorchDraws()
    X, y = bnd.wide_batch()
    x0, sx0 = bnd.quantize_tensor_dynamic(X, stochastic=False)
    cal, _ = net.calibrate(x0.numpy(), sx0, draws)
    assert digest(cal) == d["calib"]
    assert [fhex(l.sy) for l in net.int8_layers()] == d["sy"]
    sx = net.int8_layers()[0].sx
    x_i8 = torch.clamp(torch.round(X / sx), -127, 127).to(torch.int8).numpy()
    assert digest(x_i8) == d["x_i8"]
    opt = ost.I8ECO(net.int8_layers(), lr=0.05, momentum=0.9)
    st = d["steps"][0]
    logits, s_out = net.forward_i8(x_i8, draws)
    assert digest(logits) == st["logits"] and fhex(s_out) == st["s_out"]
    _, g_fp = bnd.ce_grad(torch.from_numpy(logits), s_out, y)
    g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
    assert digest(g_i8.numpy()) == st["g"] and fhex(s_g) == st["s_g"]
    net.backward_i8(g_i8.numpy(), s_g, draws)
    for layer, gw in zip(net.int8_layers(), st["grads"]):
        assert digest(layer._gw_i8) == gw["gw"] and fhex(layer._gw_s) == gw["gw_s"]
        assert digest(layer._gb_sum) == gw["gb"]
    opt.step(draws)
    for i, (layer, ls) in enumerate(zip(net.int8_layers(), st["layers"])):
        assert digest(layer.w_i8) == ls["w"] and digest(opt.m_i8[i]) == ls["m"], i
        assert digest(layer.b_acc) == ls["b"] and fhex(opt.s_m[i]) == ls["s_m"], i
    assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"]


def test_standalone_eco_step_golden(golden):
    d = golden("eco_step.json")
    torch.manual_seed(5)
    layers = [ost.I8Linear.seeded(96, 64), ost.I8Linear.seeded(64, 130, bias=False),
              ost.I8Linear.seeded(130, 3)]
    for l in layers:
        l.sx = 0.02
    opt = ost.I8ECO(layers, lr=0.05, momentum=0.9, chunk_rows=16)
    for step, st in enumerate(d):
        torch.manual_seed(100 + step)
        for l in layers:
            l._gw_i8 = torch.randint(-127, 128, l.w_i8.shape, dtype=torch.int8).numpy()
            l._gw_s = 3e-4 * (step + 1)
            l._gb_sum = torch.randint(-5000, 5000, (l.w_i8.shape[0],), dtype=torch.int64).numpy()
            l._gb_s = 2e-3
        if step == 0:
            for m in opt.m_i8:
                m[...] = torch.randint(-127, 128, m.shape, dtype=torch.int8).numpy()
            opt.s_m = [1e-3, 5e-4, 2e-3]
        torch.manual_seed(200 + step)
        rec = ost.RecordingDraws(ost.TorchDraws())
        opt.step(rec)
        assert [[list(sh), dn] for sh, dn, _ in rec.log] == st["draws"], step
        for i, (l, ls) in enumerate(zip(layers, st["layers"])):
            assert digest(l.w_i8) == ls["w"] and digest(opt.m_i8[i]) == ls["m"], (step, i)
            assert digest(l.b_acc) == ls["b"] and fhex(opt.s_m[i]) == ls["s_m"], (step, i)
        assert fhex(opt.stats["mean_abs_e"]) == st["mean_abs_e"], step


def test_single_pass_step_equals_chunked_with_same_nudges():
    """The CUDA step consumes whole-layer nudges; chunking must not change the math."""
    rng = np.random.default_rng(3)
    torch.manual_seed(9)
    layers = [ost.I8Linear.seeded(40, 70), ost.I8Linear.seeded(70, 5)]
    for l in layers:
        l.sx = 0.03
        l._gw_i8 = rng.integers(-127, 128, l.w_i8.shape).astype(np.int8)
        l._gw_s = 5e-4
        l._gb_sum = rng.integers(-900, 900, l.w_i8.shape[0])
        l._gb_s = 1e-3
    import copy

    a = ost.I8ECO(copy.deepcopy(layers), lr=0.3, chunk_rows=16)
    b = ost.I8ECO(copy.deepcopy(layers), lr=0.3, chunk_rows=16)
    for opt in (a, b):
        opt.s_m = [2e-3, 1e-3]
    for i in range(2):
        a.m_i8[i][...] = rng.integers(-127, 128, a.m_i8[i].shape).astype(np.int8)
        b.m_i8[i][...] = a.m_i8[i]
    rec = ost.RecordingDraws(ost.TorchDraws())
    a.step(rec)
    # regroup the chunked draws into whole-layer arrays in the per-layer order w, m, b
    it = iter(rec.log)
    nudges = []
    for layer in b.layers:
        out, cols = layer.w_i8.shape
        ws, ms, nb = [], [], None
        for c in range(0, out, 16):
            ws.append(next(it)[2])
            ms.append(next(it)[2])
        nb = next(it)[2]
        nudges.append((np.concatenate(ws), np.concatenate(ms), nb))
    b.step(nudges=nudges)
    for la, lb, ma, mb in zip(a.layers, b.layers, a.m_i8, b.m_i8):
        assert np.array_equal(la.w_i8, lb.w_i8) and np.array_equal(ma, mb)
        assert np.array_equal(la.b_acc, lb.b_acc)
    assert a.s_m == b.s_m and a.stats == b.stats


def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors of the Random123 distribution (kat_vectors)."""
    out = oph.philox4x32(0, 0, 0, 0, 0, 0)
    assert [int(v) for v in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    out = oph.philox4x32(0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF)
    assert [int(v) for v in out] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    out = oph.philox4x32(0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344, 0xA4093822, 0x299F31D0)
    assert [int(v) for v in out] == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_step_nudges_are_uniform_bits():
    nw, nm = oph.step_nudges(seed=1, stream=7, rows=64, cols=256, com_mm=40)
    assert nw.min() >= 0 and nw.max() < 4096 and nm.min() >= 0 and nm.max() < (1 << 40)
    assert abs(nw.mean() / 4096 - 0.5) < 0.02 and abs(nm.mean() / 2.0 ** 40 - 0.5) < 0.02
    nw2, nm2 = oph.step_nudges(seed=1, stream=7, rows=64, cols=256, com_mm=60)
    assert np.array_equal(nw, nw2) and nm2.max() < (1 << 60)


def test_sgdm_triton_interpreter_golden(golden):
    """EcoInt8SGDM's fused step (triton_kernels.py) against the reference kernels run by
    Triton's CPU interpreter: bit-exact partial maxima, scales and int8 outputs."""
    for c in golden("sgdm_triton.json"):
        w0 = np.array(c["w0"], dtype=np.int8)
        m0 = np.array(c["m0"], dtype=np.int8)
        g0 = np.array(c["g0"], dtype=np.int32).view(np.float32)
        sw = np.array(c["sw"], dtype=np.int32).view(np.float32)
        sm = np.array(c["sm"], dtype=np.int32).view(np.float32)
        res = osg.triton_step(w0, m0, g0, sw, sm, lr=c["lr"], beta=c["beta"], wd=c["wd"],
                              seed=c["seed"], division="cpu")
        assert np.array_equal(res["sg"].view(np.int32), np.int32(c["sg"]))
        assert res["partials"].view(np.int32).tolist() == c["partials"]
        assert np.array_equal(res["sm_new"].view(np.int32), np.int32(c["sm_new"]))
        assert res["w"].tolist() == c["w"]
        assert res["m"].tolist() == c["m"]


def test_fp32_eco_oracle_matches_reference_golden(golden):
    """The op-by-op PyTorch restatement of EcoSGDM / EcoAdam (oracle/fp32_eco.py) against
    the reference's own optimizers run on CPU (tests/golden/make_golden.py): bit-exact
    weights, moments, uniforms and statistics after every step."""
    import torch

    from ecoint8.layers import Int8Linear
    from oracle import fp32_eco
    from tests.golden.make_golden import digest, fp32_case_inputs

    for c in golden("fp32_eco.json"):
        layers = fp32_case_inputs(Int8Linear, [tuple(s) for s in c["shapes"]], c["steps"], c["seed"], torch)
        assert [digest(l.w_i8) for l in layers] == c["w0"]
        s_fixed = [l.s_w.clone() for l in layers]
        m = [torch.zeros_like(l.w_i8, dtype=torch.float32) for l in layers]
        v = [torch.zeros_like(mm) for mm in m]
        for t, want in enumerate(c["trace"], start=1):
            grads = [torch.randn(l.w_i8.shape) * 0.02 for l in layers]
            tot, n_e, us = 0.0, 0, []
            for i, (l, g) in enumerate(zip(layers, grads)):
                u = torch.rand(l.w_i8.shape)
                us.append(digest(u))
                if c["kind"] == "sgdm":
                    w, m[i], e_mean, ok, _ = fp32_eco.sgdm_layer(l.w_i8, l.s_w, s_fixed[i], m[i], g, u, lr=0.05,
                                                                 beta=0.9, wd=c["wd"], grad_clip=c["clip"])
                else:
                    w, m[i], v[i], e_mean, ok, _ = fp32_eco.adam_layer(l.w_i8, l.s_w, s_fixed[i], m[i], v[i], g, u,
                                                                       t=t, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8,
                                                                       wd=c["wd"], grad_clip=c["clip"])
                assert ok
                l.w_i8.copy_(w)
                tot += e_mean
                n_e += 1
            assert us == want["u"]
            assert [digest(l.w_i8) for l in layers] == want["w"]
            assert [digest(mm) for mm in m] == want["m"]
            if c["kind"] == "adam":
                assert [digest(vv) for vv in v] == want["v"]
            assert float(tot / n_e).hex() == want["mean_abs_e"]


def test_int8_linear_oracle_matches_reference_golden(golden):
    """The op-by-op PyTorch restatement of Int8LinearFunc (oracle/float_layers.py) against the
    reference's Int8Linear run through autograd on CPU: bit-exact output and gradients."""
    import torch

    from ecoint8.layers import Int8Linear
    from oracle import float_layers as fl
    from tests.golden.make_golden import digest, int8_linear_inputs

    for c in golden("int8_linear.json"):
        layer, x, gy = int8_linear_inputs(Int8Linear, c["n"], c["in"], c["out"], c["bias"], c["seed"], torch)
        assert digest(layer.w_i8) == c["w"]
        y, x_i8, s_x = fl.forward(x, layer.w_i8, layer.s_w, layer.bias.detach() if c["bias"] else None)
        gx, gw, gb = fl.backward(gy, x_i8, layer.w_i8, layer.s_w, s_x, c["bias"])
        assert digest(y) == c["y"] and digest(gx) == c["grad_x"] and digest(gw) == c["grad_w"]
        assert (digest(gb) if c["bias"] else None) == c["grad_bias"]
