"""Generate the golden fixtures by running the reference ``ecoint8`` (v0.4.9) itself.

Run in a container where the reference checkout exists (read-only is fine)::

    ECOINT8_REFERENCE=<checkout> python tests/golden/make_golden.py [--only NAME.json ...]

It imports the reference package from that path, runs the seeded workloads of
``oracle/boundary.py`` through the reference's own public API on CPU, and writes
small fixtures next to this script: digests (sha256 prefixes) of every integer
tensor after every step, the Python-float scales bit for bit (``float.hex``),
the reference's stochastic-rounding call log (shape, denominator), and a few
full arrays.  The Triton optimizer kernels run on CPU through Triton's
interpreter (``TRITON_INTERPRET=1``).  The fixtures are committed; the GPU
machines never read the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent


def digest(t) -> str:
    import numpy as np

    a = np.ascontiguousarray(t.detach().cpu().numpy() if hasattr(t, "detach") else t)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode() + str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()[:24]


def fhex(v: float) -> str:
    return float(v).hex()


class DrawLog:
    """Wraps ``_sr_nudge`` in both reference namespaces and logs (shape, denom)."""

    def __init__(self, fixedpoint_mod, iopt_mod):
        self.log = []
        self.fp, self.io = fixedpoint_mod, iopt_mod
        self.orig = fixedpoint_mod._sr_nudge

    def __enter__(self):
        orig = self.orig

        def wrapped(shape, denom, device):
            self.log.append([list(shape), int(denom)])
            return orig(shape, denom, device)

        self.fp._sr_nudge = wrapped
        self.io._sr_nudge = wrapped
        return self

    def __exit__(self, *exc):
        self.fp._sr_nudge = self.orig
        self.io._sr_nudge = self.orig


def gen_fixedpoint(ref):
    import torch

    fp = ref["fixedpoint"]
    ratios = [0.0, 1.0, 0.5, 0.75, 1e-4, 3.1e-3, 0.099, 2.0 ** -40, 123.456,
              (1 << 31) / ((1 << 31) + 0.4), 1.0 - 2.0 ** -33, 1.0 - 2.0 ** -31,
              0.999999999767, 7.0e-12, 2.5e-7]
    torch.manual_seed(7)
    ratios += [float(v) for v in torch.exp(torch.empty(40, dtype=torch.float64).uniform_(-30, 5))]
    qm = [[fhex(r), *fp.quantize_multiplier(r)] for r in ratios]
    pads = [[m, k, n, *fp.pad_mm_dims(m, k, n)] for (m, k, n) in
            [(1, 1, 1), (16, 8, 8), (17, 13, 5), (512, 256, 2), (4097, 4097, 4097), (33, 64, 1000)]]
    dyn = [[a, fhex(g), fhex(fp.dynamic_scale_from_int(a, g))] for a, g in
           [(0, 1.0), (127, 1.0), (5, 0.1), (123456, 3.3e-5), (1, 0.0), (99, 2.0 ** -30)]]
    # apply_mult_shift: det and stochastic, scalar and per-channel mults, shift sign cases
    cases = []
    torch.manual_seed(11)
    for (rows, cols, dtype, mult_kind, shift, stoch, big) in [
        (5, 7, torch.int32, "scalar", 3, False, False),
        (5, 7, torch.int32, "scalar", 0, True, False),
        (6, 9, torch.int64, "scalar", -3, True, False),
        (4, 33, torch.int32, "col", 37, True, False),
        (4, 33, torch.int32, "row", 41, True, False),
        (8, 16, torch.int64, "col", 12, False, True),
        (3, 5, torch.int64, "scalar", 62, True, True),
        (3, 5, torch.int64, "scalar", -70, False, True),
        (7, 3, torch.int32, "neg", 5, True, False),
    ]:
        hi = (1 << 62) if big else (1 << 31) - 1
        x = torch.randint(-hi, hi, (rows, cols), dtype=torch.int64).to(dtype)
        if mult_kind == "scalar":
            mult = int(torch.randint(1 << 30, 1 << 31, (1,)).item())
        elif mult_kind == "neg":
            mult = -int(torch.randint(1 << 30, 1 << 31, (1,)).item())
        elif mult_kind == "col":
            mult = torch.randint(0, 1 << 31, (cols,), dtype=torch.int32)
        else:
            mult = torch.randint(0, 1 << 31, (rows, 1), dtype=torch.int32)
        state = torch.get_rng_state()
        with DrawLog(fp, ref["iopt"]) as dl:
            out = fp.apply_mult_shift(x, mult, shift, stoch)
        torch.set_rng_state(state)  # re-draw the same nudge to store it
        nud = fp._sr_nudge(out.shape, 1 << shift, out.device) if (stoch and shift >= 0) else None
        cases.append({
            "x": x.tolist(), "dtype": str(dtype), "shift": shift, "stochastic": stoch,
            "mult": mult if isinstance(mult, int) else mult.tolist(), "mult_kind": mult_kind,
            "nudge": None if nud is None else nud.to(torch.int64).tolist(),
            "out": out.tolist(), "draws": dl.log,
        })
    sat = torch.tensor([-300, -128, -127, -1, 0, 1, 127, 128, 1 << 40], dtype=torch.int64)
    return {"quantize_multiplier": qm, "pad_mm_dims": pads, "dynamic_scale_from_int": dyn,
            "apply_mult_shift": cases, "to_int8_sat": [sat.tolist(), fp.to_int8_sat(sat).tolist()],
            "int_amax": [sat.tolist(), fp.int_amax(sat)]}


def layer_state(net, opt):
    out = []
    for i, layer in enumerate(net.int8_layers()):
        out.append({"w": digest(layer.w_i8), "b": digest(layer.b_acc), "m": digest(opt.m_i8[i]),
                    "s_m": fhex(opt.s_m[i])})
    return out


def gen_blob(ref, bnd, epochs):
    import torch

    I8Linear, I8ReLU, I8Sequential, I8ECO = (ref["I8Linear"], ref["I8ReLU"], ref["I8Sequential"],
                                             ref["I8ECO"])
    torch.manual_seed(0)
    X, y = bnd.blob_data()
    net = I8Sequential(I8Linear(bnd.BLOB_D, bnd.BLOB_H), I8ReLU(), I8Linear(bnd.BLOB_H, 2))
    init = [{"w": digest(l.w_i8), "sw": [fhex(v) for v in l.sw]} for l in net.int8_layers()]
    with torch.no_grad():
        x0, sx0 = bnd.quantize_tensor_dynamic(X, stochastic=False)
        with DrawLog(ref["fixedpoint"], ref["iopt"]) as dl_cal:
            cal_logits, cal_s = net.calibrate(x0, sx0)
        x_i8, _ = net.quantize_input(X)
    opt = I8ECO(net.int8_layers(), lr=0.5, momentum=0.9)
    steps = []
    first_log = None
    error = None
    for ep in range(epochs):
        opt.set_lr(bnd.blob_lr(ep))
        with DrawLog(ref["fixedpoint"], ref["iopt"]) as dl:
            with torch.no_grad():
                logits, s_out = net.forward_i8(x_i8)
            loss, g_fp = bnd.ce_grad(logits, s_out, y)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            with torch.no_grad():
                net.backward_i8(g_i8, s_g)
            gws = [{"gw": digest(l._gw_i8), "gw_s": fhex(l._gw_s), "gb": digest(l._gb_sum)}
                   for l in net.int8_layers()]
            try:
                opt.step()
            except ValueError as e:  # torch.randint cannot draw below 2**63 or more
                error = {"epoch": ep, "type": type(e).__name__, "msg": str(e),
                         "last_draw": dl.log[-1]}
                break
            opt.zero_grad()
        if first_log is None:
            first_log = dl.log
        steps.append({"lr": fhex(opt.lr), "logits": digest(logits), "s_out": fhex(s_out),
                      "loss": fhex(float(loss)), "g": digest(g_i8), "s_g": fhex(s_g),
                      "grads": gws, "layers": layer_state(net, opt),
                      "mean_abs_e": fhex(opt.stats["mean_abs_e"])})
    with torch.no_grad():
        acc = float((net.forward_i8(x_i8)[0].argmax(1) == y).float().mean())
    final = {f"w{i}": l.w_i8.tolist() for i, l in enumerate(net.int8_layers())}
    final.update({f"m{i}": m.tolist() for i, m in enumerate(opt.m_i8)})
    final.update({f"b{i}": l.b_acc.tolist() for i, l in enumerate(net.int8_layers())})
    return {"init": init, "calib": {"logits": digest(cal_logits), "s": fhex(cal_s),
                                    "sy": [fhex(l.sy) for l in net.int8_layers()],
                                    "draws": dl_cal.log},
            "x_i8": digest(x_i8), "steps": steps, "first_step_draws": first_log, "error": error,
            "final_acc": acc, "final": final}


def gen_mnist(ref, bnd, nsteps):
    import torch

    I8Linear, I8ReLU, I8Sequential, I8ECO = (ref["I8Linear"], ref["I8ReLU"], ref["I8Sequential"],
                                             ref["I8ECO"])
    torch.manual_seed(0)
    d0, d1, d2, d3 = bnd.MNIST_SHAPE
    net = I8Sequential(I8Linear(d0, d1), I8ReLU(), I8Linear(d1, d2), I8ReLU(), I8Linear(d2, d3))
    X0, _ = bnd.mnist_batch(0)
    with torch.no_grad():
        x0, sx0 = bnd.quantize_tensor_dynamic(X0, stochastic=False)
        net.calibrate(x0, sx0)
    opt = I8ECO(net.int8_layers(), lr=bnd.mnist_lr(0, bnd.MNIST_GOLDEN_STEPS), momentum=0.9)
    steps = []
    for t in range(nsteps):
        X, y = bnd.mnist_batch(t)
        opt.set_lr(bnd.mnist_lr(t, bnd.MNIST_GOLDEN_STEPS))
        with torch.no_grad():
            x_i8, _ = net.quantize_input(X)
            logits, s_out = net.forward_i8(x_i8)
        loss, g_fp = bnd.ce_grad(logits, s_out, y)
        g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
        with torch.no_grad():
            net.backward_i8(g_i8, s_g)
        opt.step()
        opt.zero_grad()
        steps.append({"logits": digest(logits), "g": digest(g_i8), "s_g": fhex(s_g),
                      "layers": layer_state(net, opt), "mean_abs_e": fhex(opt.stats["mean_abs_e"])})
    return {"steps": steps}


def gen_wide(ref, bnd, nsteps: int):
    """Config-5 widths: I8Linear(8192, 8192) + I8ReLU + I8Linear(8192, 1000) at batch 1024,
    Gaussian inputs quantized with the calibrated entry scale, random labels, I8ECO lr 0.05
    momentum 0.9; digests after every step."""
    import torch

    I8Linear, I8ReLU, I8Sequential, I8ECO = (ref["I8Linear"], ref["I8ReLU"], ref["I8Sequential"],
                                             ref["I8ECO"])
    torch.manual_seed(0)
    net = I8Sequential(I8Linear(bnd.WIDE_D, bnd.WIDE_D), I8ReLU(), I8Linear(bnd.WIDE_D, bnd.WIDE_C))
    init = [digest(l.w_i8) for l in net.int8_layers()]
    X, y = bnd.wide_batch()
    with torch.no_grad():
        x0, sx0 = bnd.quantize_tensor_dynamic(X, stochastic=False)
        cal, _ = net.calibrate(x0, sx0)
        x_i8, _ = net.quantize_input(X)
    opt = I8ECO(net.int8_layers(), lr=0.05, momentum=0.9)
    steps = []
    for _ in range(nsteps):
        with DrawLog(ref["fixedpoint"], ref["iopt"]) as dl:
            with torch.no_grad():
                logits, s_out = net.forward_i8(x_i8)
            loss, g_fp = bnd.ce_grad(logits, s_out, y)
            g_i8, s_g = bnd.quantize_tensor_dynamic(g_fp, stochastic=True)
            with torch.no_grad():
                net.backward_i8(g_i8, s_g)
            gws = [{"gw": digest(l._gw_i8), "gw_s": fhex(l._gw_s), "gb": digest(l._gb_sum)}
                   for l in net.int8_layers()]
            opt.step()
            opt.zero_grad()
        steps.append({"logits": digest(logits), "s_out": fhex(s_out), "g": digest(g_i8), "s_g": fhex(s_g),
                      "grads": gws, "layers": layer_state(net, opt), "mean_abs_e": fhex(opt.stats["mean_abs_e"]),
                      "draws": dl.log})
    return {"init": init, "calib": digest(cal),
            "sy": [fhex(l.sy) for l in net.int8_layers()], "x_i8": digest(x_i8), "steps": steps}


def gen_gemm_requant(ref):
    import torch

    fp = ref["fixedpoint"]
    ilayer = ref["ilayer"]
    out = []
    for (M, K, N, stoch, seed) in [(64, 48, 40, True, 1), (33, 17, 9, False, 2), (7, 13, 5, True, 3),
                                   (100, 300, 2, True, 4), (129, 65, 31, False, 5)]:
        torch.manual_seed(seed)
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8)
        b = torch.randint(-127, 128, (K, N), dtype=torch.int8)
        ratios = [float(v) for v in torch.exp(torch.empty(N, dtype=torch.float64).uniform_(
            float(torch.log(torch.tensor(1e-4, dtype=torch.float64))),
            float(torch.log(torch.tensor(1e-1, dtype=torch.float64)))))]
        acc = torch._int_mm(a, b) if M > 16 else (a.to(torch.int32) @ b.to(torch.int32))
        if stoch:
            y = ilayer._common_shift_requant(acc, ratios, stochastic=True)
        else:
            ms = [fp.quantize_multiplier(r) for r in ratios]
            com = min(s for _, s in ms)
            mults = torch.tensor([m >> (s - com) for m, s in ms], dtype=torch.int32)
            y = fp.to_int8_sat(fp.apply_mult_shift(acc.to(torch.int64), mults, com, False))
        out.append({"M": M, "K": K, "N": N, "stochastic": stoch, "seed": seed,
                    "acc": digest(acc), "y": digest(y)})
    return out


def gen_eco_step(ref):
    import torch

    I8Linear, I8ECO = ref["I8Linear"], ref["I8ECO"]
    torch.manual_seed(5)
    layers = [I8Linear(96, 64), I8Linear(64, 130, bias=False), I8Linear(130, 3)]
    for l in layers:
        l.sx = 0.02
    opt = I8ECO(layers, lr=0.05, momentum=0.9, chunk_rows=16)
    res = []
    for step in range(3):
        torch.manual_seed(100 + step)
        for l in layers:
            l._gw_i8 = torch.randint(-127, 128, l.w_i8.shape, dtype=torch.int8)
            l._gw_s = 3e-4 * (step + 1)
            l._gb_sum = torch.randint(-5000, 5000, (l.w_i8.shape[0],), dtype=torch.int64)
            l._gb_s = 2e-3
        if step == 0:
            for m in opt.m_i8:
                m.copy_(torch.randint(-127, 128, m.shape, dtype=torch.int8))
            opt.s_m = [1e-3, 5e-4, 2e-3]
        torch.manual_seed(200 + step)
        with DrawLog(ref["fixedpoint"], ref["iopt"]) as dl:
            opt.step()
        res.append({"layers": [{"w": digest(l.w_i8), "m": digest(opt.m_i8[i]), "b": digest(l.b_acc),
                                "s_m": fhex(opt.s_m[i])} for i, l in enumerate(layers)],
                    "mean_abs_e": fhex(opt.stats["mean_abs_e"]), "draws": dl.log})
    return res


def gen_sgdm_triton(ref):
    """Reference Triton optimizer kernels run by Triton's CPU interpreter.

    ``triton_eco_step_`` asserts CUDA tensors, so its four host lines
    (triton_kernels.py:156-169) are repeated here around the reference kernels.
    """
    import torch

    tk = ref["triton_kernels"]
    cases = []
    for (rows, cols, wd, seed) in [(8, 300, 0.0, 1234), (5, 1000, 0.01, 77), (33, 64, 0.0, 5)]:
        torch.manual_seed(seed)
        w = torch.randint(-127, 128, (rows, cols), dtype=torch.int8)
        m = torch.randint(-127, 128, (rows, cols), dtype=torch.int8)
        g = torch.randn(rows, cols) * 1e-2
        sw = torch.rand(rows) * 0.01 + 1e-3
        sm = torch.tensor(0.05, dtype=torch.float32)
        w0, m0, g0, sw0, sm0 = w.clone(), m.clone(), g.clone(), sw.clone(), sm.clone()
        lr, beta = 0.5, 0.9
        n = w.numel()
        grid = (n + tk.BLOCK - 1) // tk.BLOCK
        scratch = torch.zeros(tk.MAX_SCRATCH, dtype=torch.float32)
        sg_t = torch.clamp(g.abs().max(), min=1e-12) / 127.0
        alpha = (1.0 / lr) * (1.0 - 1.0 / beta)
        tk.eco_amax_kernel[(grid,)](w, m, g, sw, sm, sg_t, float(wd), float(lr), float(beta), alpha,
                                    cols, n, scratch, int(seed), tk.BLOCK)
        sm_new_t = scratch[:grid].max() / 127.0
        tk.eco_fused_kernel[(grid,)](w, m, g, sw, sm, sg_t, sm_new_t, float(wd), float(lr),
                                     float(beta), alpha, cols, n, int(seed), tk.BLOCK)
        cases.append({"rows": rows, "cols": cols, "wd": wd, "seed": seed, "lr": lr, "beta": beta,
                      "w0": w0.tolist(), "m0": m0.tolist(), "g0": g0.view(torch.int32).tolist(),
                      "sw": sw0.view(torch.int32).tolist(), "sm": sm0.view(torch.int32).item(),
                      "partials": scratch[:grid].view(torch.int32).tolist(),
                      "sg": sg_t.view(torch.int32).item(), "sm_new": sm_new_t.view(torch.int32).item(),
                      "w": w.tolist(), "m": m.tolist()})
    return cases


FP32_CASES = [  # (optimizer, layer shapes, steps, weight decay, grad clip, seed)
    ("sgdm", [(24, 40), (16, 24)], 3, 0.0, 1.0, 11),
    ("sgdm", [(24, 40), (16, 24)], 3, 0.01, 0.05, 12),  # clipping active, weight decay
    ("adam", [(24, 40), (16, 24)], 3, 0.0, 1.0, 13),
    ("adam", [(24, 40), (16, 24)], 3, 0.01, 0.05, 14),
]


def fp32_case_inputs(layer_cls, shapes, steps, seed, torch):
    """The seeded inputs of an fp32-optimizer case: layers, then per step the gradients
    (the uniforms of the stochastic rounding follow inside each step, one
    ``torch.rand_like`` per layer, from the same generator)."""
    torch.manual_seed(seed)
    layers = [layer_cls(i, o) for (o, i) in shapes]
    return layers


def gen_fp32_eco(ref):
    """EcoSGDM / EcoAdam (eco.py:50-235) on the reference's Int8Linear layers, on CPU.
    The uniforms each step draws (quant.py:25, torch.rand_like) are logged."""
    import torch

    eco, Int8Linear = ref["eco"], ref["Int8Linear"]
    cases = []
    for kind, shapes, steps, wd, clip, seed in FP32_CASES:
        layers = fp32_case_inputs(Int8Linear, shapes, steps, seed, torch)
        w0 = [l.w_i8.clone() for l in layers]
        opt = (eco.EcoSGDM(layers, lr=0.05, momentum=0.9, weight_decay=wd, grad_clip=clip) if kind == "sgdm"
               else eco.EcoAdam(layers, lr=1e-3, weight_decay=wd, grad_clip=clip))
        per_step = []
        for t in range(steps):
            for l in layers:
                l._grad_w = torch.randn(l.w_i8.shape) * 0.02
            drawn = []
            orig = torch.rand_like

            def logged(x, *a, **k):
                r = orig(x, *a, **k)
                drawn.append(digest(r))
                return r

            torch.rand_like = logged
            try:
                opt.step()
            finally:
                torch.rand_like = orig
            state = {"w": [digest(l.w_i8) for l in layers], "m": [digest(m) for m in opt.m],
                     "mean_abs_e": fhex(opt.stats["mean_abs_e"]), "u": drawn}
            if kind == "adam":
                state["v"] = [digest(v) for v in opt.v]
            per_step.append(state)
            opt.zero_grad()
        cases.append({"kind": kind, "shapes": shapes, "steps": steps, "wd": wd, "clip": clip, "seed": seed,
                      "w0": [digest(w) for w in w0], "trace": per_step})
    return cases


INT8_LINEAR_CASES = [(64, 40, 24, True, 21), (33, 70, 17, False, 22), (8, 16, 8, True, 23)]  # N, in, out, bias, seed


def int8_linear_inputs(layer_cls, n, in_f, out_f, bias, seed, torch):
    torch.manual_seed(seed)
    layer = layer_cls(in_f, out_f, bias)
    if bias:
        layer.bias.data.copy_(torch.randn(out_f) * 0.1)
    x = torch.randn(n, in_f) * 2.0
    gy = torch.randn(n, out_f) * 0.05
    return layer, x, gy


def gen_int8_linear(ref):
    """Int8Linear forward and backward through autograd (layers.py:45-111) on CPU."""
    import torch

    cases = []
    for n, in_f, out_f, bias, seed in INT8_LINEAR_CASES:
        layer, x, gy = int8_linear_inputs(ref["Int8Linear"], n, in_f, out_f, bias, seed, torch)
        x.requires_grad_(True)
        y = layer(x)
        y.backward(gy)
        cases.append({"n": n, "in": in_f, "out": out_f, "bias": bias, "seed": seed, "w": digest(layer.w_i8),
                      "y": digest(y.detach()), "grad_x": digest(x.grad), "grad_w": digest(layer._grad_w),
                      "grad_bias": digest(layer.bias.grad) if bias else None})
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ECOINT8_REFERENCE"),
                    help="the reference checkout (default: $ECOINT8_REFERENCE)")
    ap.add_argument("--epochs", type=int, default=150)
    ap.add_argument("--only", nargs="*", default=None, help="fixture file names to (re)generate")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give --reference or set ECOINT8_REFERENCE")
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(1)
    import ecoint8
    import ecoint8.fixedpoint as fixedpoint
    import ecoint8.strict.ilayer as ilayer
    import ecoint8.strict.iopt as iopt
    import ecoint8.eco as eco
    import ecoint8.layers as layers
    import ecoint8.triton_kernels as triton_kernels
    from oracle import boundary as bnd

    assert pathlib.Path(ecoint8.__file__).resolve().is_relative_to(pathlib.Path(args.reference).resolve())
    ref = {"fixedpoint": fixedpoint, "ilayer": ilayer, "iopt": iopt, "triton_kernels": triton_kernels,
           "I8Linear": ilayer.I8Linear, "I8ReLU": ilayer.I8ReLU, "I8Sequential": ilayer.I8Sequential,
           "I8ECO": iopt.I8ECO, "eco": eco, "Int8Linear": layers.Int8Linear}
    gens = {
        "fixedpoint.json": lambda: gen_fixedpoint(ref),
        "blob_train.json": lambda: gen_blob(ref, bnd, args.epochs),
        "mnist_train.json": lambda: gen_mnist(ref, bnd, bnd.MNIST_GOLDEN_STEPS),
        "gemm_requant.json": lambda: gen_gemm_requant(ref),
        "eco_step.json": lambda: gen_eco_step(ref),
        "sgdm_triton.json": lambda: gen_sgdm_triton(ref),
        "wide_train.json": lambda: gen_wide(ref, bnd, 3),
        "fp32_eco.json": lambda: gen_fp32_eco(ref),
        "int8_linear.json": lambda: gen_int8_linear(ref),
    }
    if args.only:
        torch.set_num_threads(os.cpu_count() or 1)  # the wide fixture's GEMMs (results do not depend on it)
    fixtures = {name: fn() for name, fn in gens.items() if not args.only or name in args.only}
    meta = {"reference": "valik8937/eco-int8-opt", "version": ecoint8.__version__,
            "torch": torch.__version__, "generator": "tests/golden/make_golden.py"}
    for name, obj in fixtures.items():
        obj = {"meta": meta, "data": obj}
        (HERE / name).write_text(json.dumps(obj, separators=(",", ":")))
        print(name, (HERE / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
