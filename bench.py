"""Benchmark of the strict int8 ECO training step on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1: one rank per GPU)

Headline (``value``): training steps/s of the deep strict-int8 MLP -- 8
``I8Linear(8192, 8192)`` + ``I8ReLU`` blocks and ``I8Linear(8192, 1000)`` --
at a global batch of 16384 Gaussian samples with random labels, I8ECO
(momentum 0.9).  One step = forward_i8 + the loss boundary (cross entropy and
stochastic gradient quantization, fused: ``ecoint8.quant.cross_entropy_grad_i8``)
+ backward_i8 + I8ECO.step, with no host synchronisation inside the step.  With
N GPUs the global batch (drawn once from one seed) is split across ranks
(strong scaling); every exchange is exact, so all N print the same
``weights_digest`` after the run.  Inputs are larger than L2 (no flush needed).

Also measured on rank 0 at N=1: the GEMMs in their training layouts (the int32
dX / dW GEMM is the step's dominant kernel, the roofline line), an int8 tensor
peak measured on this GPU, the standalone I8ECO step over 64 layers of
4096x4096 (config 4, HBM GB/s), the EcoInt8SGDM step at the same size, the
backward requants, and the reference's own strict step on the host cores
(``cpu_baseline``).  ``--impl reference`` times only that reference step.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import pathlib
import statistics
import struct
import subprocess
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

LAYERS = [(8192, 8192)] * 8 + [(8192, 1000)]
GLOBAL_BATCH = 16384
METRIC = "int8 train steps/s (deep MLP 8x8192^2+8192->1000, global batch 16384)"
WORKLOAD = ("config 5: deep strict-int8 MLP 8x I8Linear(8192,8192)+I8ReLU, I8Linear(8192,1000); Gaussian inputs, "
            "random labels; I8ECO lr 0.05 momentum 0.9 grad_clip 1.0")
LAYER_EQUIV = sum(a * b for a, b in LAYERS) / (8192 * 8192)  # the step's work in 8192^2-layer units


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 50 ms) while the timed region runs.  Entering waits (at
    most 3 s) for the first sample, so that sampling is under way when the region opens;
    only samples that arrive inside the region count, and when the region is shorter than
    one period the sample taken just before it stands in (``samples`` says which)."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        self.first = len(self.lines)  # samples before the timed region
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        inside = self.lines[self.first:]
        lines = inside if inside else self.lines[-1:]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm) if inside else 0,
                "sampled": "inside the timed region" if inside else "just before the (short) timed region"}


# ----------------------------------------------------------------------------- launch counter
def _step_kernels(layers, n, *rest) -> int:
    """The I8ECO step kernel, plus the bias kernel when a row shard steps every bias."""
    return 1 + int(any(layers[i].b_acc and layers[i].bias_rows > 0 for i in range(n)))


# library kernels launched per C-ABI call (an int, or a function of the call's arguments)
KERNELS_PER_CALL = {"eco_gemm_s8s32": 1, "eco_gemm_s8_requant": 1, "eco_requant_s32_s8": 1,
                    "eco_requant_s32_s8_dev": 1, "eco_scale_from_amax": 1, "eco_apply_mult_shift": 1,
                    "eco_colsum_s8": 1, "eco_amax": 2, "eco_sumsq_s8": 1, "eco_split_cols_s8": 1,
                    "eco_i8eco_step": _step_kernels, "eco_i8eco_finalize": 1, "eco_sgdm_step": 3,
                    "eco_peer_push_s8": 1, "eco_peer_push_signal_s8": 1, "eco_peer_signal": 1,
                    "eco_peer_wait": 1, "eco_peer_allreduce_i64": 1, "eco_ce_grad_rowstats": 1,
                    "eco_ce_grad_quantize": 1, "eco_copy2d_s8": 1, "eco_gemm_s8_dequant": 1,
                    "eco_quantize_dynamic_f32": 2, "eco_fp32_eco_step": 2}


class LaunchCounter:
    def __init__(self):
        from ecoint8 import _native

        self.nat = _native
        self.count = 0
        self.captured = 0  # of which recorded into a CUDA graph
        self.orig = _native.call

    def __enter__(self):
        from ecoint8 import graphs

        def counting(name, *args):
            k = KERNELS_PER_CALL.get(name, 0)
            k = k(*args) if callable(k) else k
            self.count += k
            if graphs.capturing() is not None:
                self.captured += k
            return self.orig(name, *args)

        self.nat.call = counting
        # the modules bound `call` through the module, so patching the attribute is enough
        return self

    def __exit__(self, *exc):
        self.nat.call = self.orig


# ----------------------------------------------------------------------------- model and data
def fast_layer(in_f, out_f, gen, device):
    """I8Linear with the reference's init formula (ilayer.py:96-101) evaluated on the GPU."""
    import torch

    from ecoint8 import I8Linear

    lin = I8Linear(1, 1)
    w_fp = torch.randn(out_f, in_f, generator=gen, device=device) * (2.0 / in_f) ** 0.5
    amax = w_fp.abs().amax(dim=1)
    sw = (amax / 127.0 * lin.headroom).clamp_min(1e-8)
    lin.w_i8 = torch.clamp(torch.round(w_fp / sw.unsqueeze(1)), -127, 127).to(torch.int8)
    lin.sw = [float(v) for v in sw.cpu()]
    lin.b_acc = torch.zeros(out_f, dtype=torch.int32, device=device)
    return lin


def build_mlp(device, seed=0):
    import torch

    from ecoint8 import I8ReLU, I8Sequential

    gen = torch.Generator(device=device).manual_seed(seed)
    blocks = []
    for i, (a, b) in enumerate(LAYERS):
        blocks.append(fast_layer(a, b, gen, device))
        if i + 1 < len(LAYERS):
            blocks.append(I8ReLU())
    return I8Sequential(*blocks).to(device)


def global_batch(device, rank, world):
    """This rank's rows of the global batch, drawn once from one seed on every rank
    (Gaussian inputs, labels uniform over 1000 classes), and the batch's entry scale."""
    import torch

    from ecoint8.quant import calc_scale

    gen = torch.Generator(device=device).manual_seed(100)
    x = torch.randn(GLOBAL_BATCH, LAYERS[0][0], generator=gen, device=device)
    y = torch.randint(0, LAYERS[-1][1], (GLOBAL_BATCH,), generator=gen, device=device)
    s_x = calc_scale(x.abs().max().item())  # quantize_tensor_dynamic's scale, over the global batch
    b = GLOBAL_BATCH // world
    return x[rank * b:(rank + 1) * b].clone(), y[rank * b:(rank + 1) * b].clone(), s_x


def train_step(net, opt, x_i8, y):
    from ecoint8.quant import cross_entropy_grad_i8

    logits, s_out = net.forward_i8(x_i8)
    loss, g_i8, s_g = cross_entropy_grad_i8(logits, s_out, y, count=GLOBAL_BATCH)
    net.backward_i8(g_i8, s_g)
    opt.step()
    opt.zero_grad()
    return loss


def weights_digest(net, opt, world) -> str:
    """sha256 of every layer's weights, momentum and bias accumulator and the momentum
    scales after the run (momentum rows gathered from their owners under data parallelism)."""
    from ecoint8 import parallel

    if world > 1:
        parallel.synchronize(net.int8_layers())
        parallel.gather_momentum(opt)
    h = hashlib.sha256()
    for layer, m in zip(net.int8_layers(), opt.m_i8):
        for t in (layer.w_i8, m, layer.b_acc):
            h.update(t.contiguous().cpu().numpy().tobytes())
    h.update(struct.pack(f"<{len(opt.s_m)}d", *opt.s_m))
    h.update(float(opt.stats["mean_abs_e"]).hex().encode())
    return h.hexdigest()[:24]


# ----------------------------------------------------------------------------- side measurements
def time_kernel(fn, iters=10, warmup=3):
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters / 1e3  # s per launch


def gemm_measurements(device, M=16384, N=8192, K=8192):
    """The GEMMs of an 8192-wide layer at batch 16384 in their training layouts:

    * fused forward (bias, per-column multipliers, Philox SR, ReLU): A = x [M,K], B = w [N,K];
    * int32 + max|C| dX: A = g [M,K] (K-major), B = w stored [K,N] (MN-major);
    * int32 + max|C| dW: A = g stored [K=batch, M] and B = x stored [K=batch, N] (both MN-major);
    * cuBLASLt ``torch._int_mm`` (the reference's GEMM) at the forward shape.
    """
    import torch

    from ecoint8 import _native, _ops, _sr

    gen = torch.Generator(device=device).manual_seed(1)
    x = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=device, generator=gen)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=device, generator=gen)
    bias = torch.randint(-1000, 1000, (N,), dtype=torch.int32, device=device, generator=gen)
    mult = torch.randint(1 << 20, 1 << 21, (N,), dtype=torch.int32, device=device, generator=gen)
    site = _sr.Site(_native.sr_spec(_native.SR_PHILOX, seed=7, stream_id=0), None)
    y = torch.empty((M, N), dtype=torch.int8, device=device)
    c = torch.empty((M, N), dtype=torch.int32, device=device)
    amax = torch.empty(1, dtype=torch.int32, device=device)
    t_fused = time_kernel(lambda: _ops.gemm_requant(x, 0, w, 0, M, N, K, bias, mult, 36, True, site, out=y))

    def s32(a, al, b, bl, m, n, k, out):
        _native.call("eco_gemm_s8s32", a.data_ptr(), a.stride(0), al, b.data_ptr(), b.stride(0), bl, m, n, k, None,
                     out.data_ptr(), n, amax.data_ptr(), _native.stream())

    t_fwd32 = time_kernel(lambda: s32(x, 0, w, 0, M, N, K, c))
    wt = torch.randint(-127, 128, (K, N), dtype=torch.int8, device=device, generator=gen)  # w stored [out=K, in=N]
    t_dx = time_kernel(lambda: s32(x, 0, wt, 1, M, N, K, c))
    # dW [out=N, in=K] over the batch M: A = g stored [M, N] (MN-major), B = x stored [M, K] (MN-major)
    g = torch.randint(-127, 128, (M, N), dtype=torch.int8, device=device, generator=gen)
    cw = torch.empty((N, K), dtype=torch.int32, device=device)
    t_dw = time_kernel(lambda: s32(g, 1, x, 1, N, K, M, cw))
    try:
        t_cublas = time_kernel(lambda: torch._int_mm(x, w.t()))
    except RuntimeError:  # cuBLASLt's int8 GEMM needs K and N multiples of 8
        t_cublas = None
    ops = 2.0 * M * N * K
    res = {"shape": [M, N, K], "fused_requant_tops": ops / t_fused / 1e12, "fused_ms": t_fused * 1e3,
           "s32_fwd_layout_tops": ops / t_fwd32 / 1e12,
           "s32_dx_tops": ops / t_dx / 1e12, "s32_dx_ms": t_dx * 1e3,
           "s32_dw_tops": ops / t_dw / 1e12, "s32_dw_ms": t_dw * 1e3,
           "torch_int_mm_cublas_tops": None if t_cublas is None else ops / t_cublas / 1e12}
    return res, {"fused": t_fused, "dx": t_dx, "dw": t_dw}, ops


def int8_peak(device):
    """A dense int8 tensor-core peak measured on this GPU: the best of cuBLASLt's
    ``torch._int_mm`` and this library's int32 GEMM over square and training shapes."""
    import torch

    from ecoint8 import _native

    best, where = 0.0, None
    for (M, N, K) in [(8192, 8192, 8192), (16384, 8192, 8192), (16384, 16384, 16384)]:
        gen = torch.Generator(device=device).manual_seed(2)
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=device, generator=gen)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=device, generator=gen)
        c = torch.empty((M, N), dtype=torch.int32, device=device)
        ops = 2.0 * M * N * K
        for name, fn in (("cuBLASLt torch._int_mm", lambda: torch._int_mm(a, b.t())),
                         ("gemm_s8_kernel", lambda: _native.call("eco_gemm_s8s32", a.data_ptr(), K, 0, b.data_ptr(),
                                                                  K, 0, M, N, K, None, c.data_ptr(), N, None,
                                                                  _native.stream()))):
            tops = ops / time_kernel(fn, iters=8) / 1e12
            if tops > best:
                best, where = tops, f"{name} {M}x{N}x{K}"
        del a, b, c
    return best, where


GEMM_SWEEP = [(1024, 1024, 1024), (4096, 4096, 4096), (4097, 4097, 4097), (8192, 8192, 8192),
              (16384, 8192, 8192), (16384, 16384, 16384), (16384, 4097, 8192)]


def gemm_sweep(device):
    """Config 3: the fused GEMM at M, N, K from {1024, 4096, 8192, 16384} plus non-multiple-of-16 sizes."""
    import torch

    from ecoint8 import _native, _ops, _sr

    out = []
    for (M, N, K) in GEMM_SWEEP:
        gen = torch.Generator(device=device).manual_seed(1)
        x = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=device, generator=gen)
        w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=device, generator=gen)
        mult = torch.randint(1 << 20, 1 << 21, (N,), dtype=torch.int32, device=device, generator=gen)
        site = _sr.Site(_native.sr_spec(_native.SR_PHILOX, seed=7, stream_id=0), None)
        ops = 2.0 * M * N * K
        t_f = time_kernel(lambda: _ops.gemm_requant(x, 0, w, 0, M, N, K, None, mult, 36, True, site))
        t_s = time_kernel(lambda: _ops.gemm_s32(x, 0, w, 0, M, N, K))
        try:
            t_c = time_kernel(lambda: torch._int_mm(x, w.t()))
        except RuntimeError:
            t_c = None
        out.append({"shape": [M, N, K], "fused_requant_tops": ops / t_f / 1e12, "s32_tops": ops / t_s / 1e12,
                    "torch_int_mm_cublas_tops": None if t_c is None else ops / t_c / 1e12})
    return out


def requant_measurement(device, rows=16384, cols=8192):
    """The two backward requants of one 8192-wide layer at batch 16384, as training runs
    them: dX (int32 -> int8, Philox SR, scalar multiplier, ReLU mask; 4 + 1 + 1 B per
    element) and dW (8192 x 8192, square sum for the gradient clip; 4 + 1 B)."""
    import torch

    from ecoint8 import _native, _ops, _sr

    gen = torch.Generator(device=device).manual_seed(3)
    src = torch.randint(-(1 << 24), 1 << 24, (rows, cols), dtype=torch.int32, device=device, generator=gen)
    mask = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device=device, generator=gen)
    sq = torch.empty(1, dtype=torch.int64, device=device)
    site = _sr.Site(_native.sr_spec(_native.SR_PHILOX, seed=11, stream_id=0), None)
    t = time_kernel(lambda: _ops.requant(src, 1 << 30, 38, site, mask=mask))
    w = src[:cols]
    t_w = time_kernel(lambda: _ops.requant(w, 1 << 30, 38, site, sumsq=sq))
    n = rows * cols
    return {"shape": [rows, cols], "ms": t * 1e3, "gbs": 6.0 * n / t / 1e9, "bytes_per_element": 6,
            "dw": {"shape": [cols, cols], "ms": t_w * 1e3, "gbs": 5.0 * cols * cols / t_w / 1e9,
                   "bytes_per_element": 5}}


def eco_step_measurement(device, layers=64, dim=4096, steps=5):
    """Config 4: I8ECO.step over 64 x 4096^2 int8 parameters (w, m, g uniform in [-127, 127]),
    lr 0.05, momentum 0.9, grad_clip 1.0 (the default), ECO error injection on."""
    import torch

    from ecoint8 import I8ECO, _ops

    gen = torch.Generator(device=device).manual_seed(2)
    proto = fast_layer(dim, dim, gen, device)
    lys = []
    for _ in range(layers):
        lin = fast_layer(1, 1, gen, device)
        lin.w_i8 = torch.randint(-127, 128, (dim, dim), dtype=torch.int8, device=device, generator=gen)
        lin.b_acc = torch.zeros(dim, dtype=torch.int32, device=device)
        lin.sw = list(proto.sw)
        lin.sx = 0.01
        lin._gw_i8 = torch.randint(-127, 128, (dim, dim), dtype=torch.int8, device=device, generator=gen)
        lin._gw_s = 2e-4
        lin._gw_sumsq = _ops.sumsq(lin._gw_i8)  # produced by the dW requant in training
        lin._gw_sumsq_of = lin._gw_i8
        lin._gb_sum = torch.randint(-10 ** 6, 10 ** 6, (dim,), dtype=torch.int64, device=device, generator=gen)
        lin._gb_s = 1e-4
        lys.append(lin)
    opt = I8ECO(lys, lr=0.05, momentum=0.9, grad_clip=1.0)
    for m in opt.m_i8:
        m.copy_(torch.randint(-127, 128, m.shape, dtype=torch.int8, device=device, generator=gen))
    opt.s_m = [3e-4] * layers
    t = time_kernel(opt.step, iters=steps, warmup=3)
    params = layers * dim * dim
    return {"params": params, "bytes_per_param": 5, "ms": t * 1e3, "gbs": 5.0 * params / t / 1e9,
            "lr": 0.05, "momentum": 0.9, "grad_clip": 1.0}


def fp32_eco_measurement(device, layers=16, dim=4096, steps=3):
    """EcoSGDM / EcoAdam (eco.py:50-235): the fused two-launch step over 16 x 4096^2
    parameters (int8 w, fp32 m and for Adam v, fp32 g; per-row fp32 scales).  Algorithmic
    bytes per parameter: SGDM reads w, m, g and writes w, m = 1 + 4 + 4 + 1 + 4 = 14; Adam
    adds v read and written = 22.  The kernels read g twice (the clip's norm pass, then the
    step): 18 / 26 kernel bytes."""
    import torch

    from ecoint8 import EcoAdam, EcoSGDM, Int8Linear

    out = {}
    for name, make, alg in (("sgdm", lambda ls: EcoSGDM(ls, lr=0.05, momentum=0.9), 14),
                            ("adam", lambda ls: EcoAdam(ls, lr=1e-3), 22)):
        gen = torch.Generator(device=device).manual_seed(6)
        lys = []
        for _ in range(layers):
            lin = Int8Linear(1, 1, bias=False).to(device)
            lin.w_i8 = torch.randint(-127, 128, (dim, dim), dtype=torch.int8, device=device, generator=gen)
            lin.s_w = torch.rand((dim, 1), device=device, generator=gen) * 1e-2 + 1e-3
            lys.append(lin)
        grads = [torch.randn((dim, dim), device=device, generator=gen) * 1e-3 for _ in range(layers)]
        opt = make(lys)

        def step():
            for lin, g in zip(lys, grads):
                lin._grad_w = g
            opt.step()

        t = time_kernel(step, iters=steps, warmup=2)
        params = layers * dim * dim
        out[name] = {"params": params, "ms": t * 1e3, "bytes_per_param": alg, "gbs": alg * params / t / 1e9,
                     "kernel_bytes_per_param": alg + 4}
        del lys, grads, opt
        torch.cuda.empty_cache()
    return out


def int8_linear_measurement(device, batch=16384, dim=8192, steps=3):
    """Int8Linear (layers.py:45-111) forward + backward through autograd at a config-5
    layer's shape, batch 16384 x 8192 -> 8192: the input's and the output gradient's dynamic
    quantization on the device and three int8 GEMMs with fp32 dequant epilogues
    (3 x 2 B dim^2 = 6.6e12 int ops)."""
    import torch

    from ecoint8.layers import Int8Linear

    gen = torch.Generator(device=device).manual_seed(8)
    layer = Int8Linear(dim, dim).to(device)
    x = (torch.randn(batch, dim, device=device, generator=gen) * 2.0).requires_grad_(True)
    gy = torch.randn(batch, dim, device=device, generator=gen) * 0.05

    def step():
        y = layer(x)
        y.backward(gy)
        x.grad = None

    t = time_kernel(step, iters=steps, warmup=2)
    ops = 6.0 * batch * dim * dim
    return {"shape": [batch, dim, dim], "ms": t * 1e3, "tops": ops / t / 1e12}


def boundary_measurement(device, rows=16384, classes=1000):
    """The fused loss boundary (quant.cross_entropy_grad_i8) on config 5's logits: int8
    [16384, 1000] -> loss, int8 gradient and its device scale (two launches; 1 B read twice
    and 1 B written per logit)."""
    import torch

    from ecoint8.quant import cross_entropy_grad_i8

    gen = torch.Generator(device=device).manual_seed(9)
    logits = torch.randint(-127, 128, (rows, classes), dtype=torch.int8, device=device, generator=gen)
    labels = torch.randint(0, classes, (rows,), device=device, generator=gen)
    t = time_kernel(lambda: cross_entropy_grad_i8(logits, 0.05, labels), iters=20, warmup=3)
    return {"shape": [rows, classes], "ms": t * 1e3, "gbs": 3.0 * rows * classes / t / 1e9}


def sgdm_measurement(device, layers=64, dim=4096, steps=3):
    """EcoInt8SGDM's fused step (the replacement of the reference's Triton kernels) over
    64 x 4096^2 parameters: int8 w, m, fp32 g.  Algorithmic bytes 8 per parameter (read
    w, m, g; write w, m); the step reads g and w, m again in its second pass because the
    momentum scale is the maximum over the whole layer."""
    import torch

    from ecoint8 import EcoInt8SGDM, Int8Linear

    gen = torch.Generator(device=device).manual_seed(4)
    lys = []
    for _ in range(layers):
        lin = Int8Linear(1, 1, bias=False).to(device)
        lin.w_i8 = torch.randint(-127, 128, (dim, dim), dtype=torch.int8, device=device, generator=gen)
        lin.s_w = torch.rand((dim, 1), device=device, generator=gen) * 1e-2 + 1e-3
        lin._grad_w = torch.randn((dim, dim), device=device, generator=gen) * 1e-3
        lys.append(lin)
    opt = EcoInt8SGDM(lys, lr=0.05, momentum=0.9)
    grads = [l._grad_w for l in lys]

    def step():  # the fused kernels alone, as EcoInt8SGDM.step calls them per layer
        for i, (l, g) in enumerate(zip(lys, grads)):
            opt._step_fused(i, l, g)

    t = time_kernel(step, iters=steps, warmup=2)
    params = layers * dim * dim
    return {"params": params, "ms": t * 1e3, "bytes_per_param": 8, "gbs": 8.0 * params / t / 1e9,
            "kernel_bytes_per_param": 18}


# ----------------------------------------------------------------------------- the reference on the host
def reference_layer_steps(max_samples: int, budget_s: float, batch: int = GLOBAL_BATCH):
    """The reference's own strict step (compiled from its sources into oracle/_ref) on the
    host cores: one I8Linear(8192, 8192) + I8ReLU at batch 16384 -- forward_i8,
    I8ReLU.backward_mask, backward_i8, I8ECO.step -- per sample, on all host threads.
    One untimed layer step first; then samples until ``max_samples`` or ``budget_s``.
    Returns (seconds per layer step of each timed sample, info) or None when the
    compiled reference is absent."""
    from oracle import build_ref

    ref = build_ref.load()
    if ref is None:
        return None
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)  # explicit: torchrun's OMP_NUM_THREADS=1 must not apply
    strict, quant = ref["strict"], ref["quant"]
    torch.manual_seed(0)
    lin, relu = strict.I8Linear(8192, 8192), strict.I8ReLU()
    x = torch.randn(batch, 8192)
    x0, sx0 = quant.quantize_tensor_dynamic(x)
    del x
    lin.calibrate_forward(x0, sx0)
    opt = strict.I8ECO([lin], lr=0.05, momentum=0.9)
    g = torch.randint(-127, 128, (batch, 8192), dtype=torch.int8)

    def layer_step():
        y, _ = lin.forward_i8(x0)
        relu.apply_forward(y)
        lin.backward_i8(relu.backward_mask(g), 1e-4)
        opt.step()
        opt.zero_grad()

    layer_step()  # untimed: first-touch allocations
    times, t_all = [], time.perf_counter()
    while len(times) < max(1, max_samples) and (not times or time.perf_counter() - t_all < budget_s):
        t0 = time.perf_counter()
        layer_step()
        times.append(time.perf_counter() - t0)
    info = {"threads": threads, "version": ref["version"], "torch": torch.__version__}
    return times, info


def reference_row_samples(ref) -> dict:
    """The next rows' reference code on the host cores, one bounded sample each (all host
    threads): EcoSGDM.step and EcoAdam.step on one Int8Linear(4096, 4096) (eco.py:94-131,
    182-228), Int8Linear forward + backward at batch 2048 x 8192 -> 8192 (layers.py:45-75,
    CPU torch._int_mm), and the training loop's loss boundary on config 5's logits
    [16384, 1000] (examples/i8_demo.py:56-59: cross entropy, its gradient,
    quantize_tensor_dynamic(g, stochastic=True)).  Seconds per sample and the work it did."""
    import importlib

    import torch

    eco = importlib.import_module("ecoint8.eco")
    layers = importlib.import_module("ecoint8.layers")
    quant = ref["quant"]
    out = {}
    torch.manual_seed(0)
    for name, make in (("eco_sgdm", lambda ls: eco.EcoSGDM(ls, lr=0.05, momentum=0.9)),
                       ("eco_adam", lambda ls: eco.EcoAdam(ls, lr=1e-3))):
        lin = layers.Int8Linear(4096, 4096, bias=False)
        opt = make([lin])
        g = torch.randn(4096, 4096) * 1e-3
        lin._grad_w = g.clone()
        opt.step()  # untimed: state allocation
        lin._grad_w = g.clone()
        t0 = time.perf_counter()
        opt.step()
        out[name] = {"s": time.perf_counter() - t0, "params": 4096 * 4096}
    lin = layers.Int8Linear(8192, 8192)
    x = (torch.randn(2048, 8192) * 2.0).requires_grad_(True)
    gy = torch.randn(2048, 8192) * 0.05
    lin(x).backward(gy)  # untimed
    x.grad = None
    t0 = time.perf_counter()
    lin(x).backward(gy)
    out["int8_linear"] = {"s": time.perf_counter() - t0, "int_ops": 6.0 * 2048 * 8192 * 8192}
    logits = torch.randint(-127, 128, (16384, 1000), dtype=torch.int8)
    labels = torch.randint(0, 1000, (16384,))
    t0 = time.perf_counter()
    z = (logits.to(torch.float32) * 0.05).requires_grad_(True)
    loss = torch.nn.functional.cross_entropy(z, labels)
    (gz,) = torch.autograd.grad(loss, z)
    quant.quantize_tensor_dynamic(gz, stochastic=True)
    out["loss_boundary"] = {"s": time.perf_counter() - t0, "logits": 16384 * 1000}
    return out


def row_ratios(out: dict, rows: dict) -> dict:
    """GPU rate over the reference's host rate for the rows next to the path (work per
    second each; the work unit of each row is named)."""
    r = {}
    try:
        for k, name in (("sgdm", "eco_sgdm"), ("adam", "eco_adam")):
            if name in rows:
                gpu = out["fp32_eco"][k]["params"] / (out["fp32_eco"][k]["ms"] / 1e3)
                r[name] = {"unit": "parameters/s", "ratio": gpu / (rows[name]["params"] / rows[name]["s"])}
        if "int8_linear" in rows:
            r["int8_linear"] = {"unit": "int ops/s", "ratio": out["int8_linear"]["tops"] * 1e12
                                / (rows["int8_linear"]["int_ops"] / rows["int8_linear"]["s"])}
        if "loss_boundary" in rows:
            gpu = out["loss_boundary"]["shape"][0] * out["loss_boundary"]["shape"][1] / (out["loss_boundary"]["ms"] / 1e3)
            r["loss_boundary"] = {"unit": "logits/s", "ratio": gpu / (rows["loss_boundary"]["logits"]
                                                                     / rows["loss_boundary"]["s"])}
    except (KeyError, TypeError, ZeroDivisionError):
        pass
    return r


def cpu_baseline_subprocess():
    """``cpu_baseline`` of the GPU arm: the reference arm (one untimed and one timed layer
    step of the compiled reference) in a child process, so that the reference's own
    ``ecoint8`` package never shares a process with this build's."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "OMP_NUM_THREADS")}
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, env=env, timeout=1200)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"value": None, "unit": "steps/s", "cores": None, "kind": "unavailable",
                "sample": f"reference arm failed (rc {r.returncode}): {r.stderr.strip()[-300:]}"}
    return json.loads(lines[-1])["cpu_baseline"]


def cpu_baseline_port():
    """The oracle port of the reference strict step on the host cores (used only when the
    compiled reference is absent), on a bounded sample scaled by work to the full step."""
    import numpy as np

    import torch

    from oracle import fixedpoint as ofp
    from oracle import strict as ost

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rng = np.random.default_rng(0)
    d, b, rows = 8192, 256, 256
    w = rng.integers(-127, 128, (d, d), dtype=np.int8)
    x = rng.integers(-127, 128, (b, d), dtype=np.int8)
    g = rng.integers(-127, 128, (b, d), dtype=np.int8)
    wf = w.astype(np.float64)
    sw = [1e-2 + 1e-6 * i for i in range(d)]
    draw = ost.TorchDraws()

    def mm(a, bf):
        return (a.astype(np.float64) @ bf).astype(np.int64).astype(np.int32)

    t0 = time.perf_counter()
    ost.common_shift_requant(mm(x, wf.T), [0.02 * s / 0.5 for s in sw], draw)
    dx = mm(g, wf)
    m, sh = ofp.quantize_multiplier(1e-4)
    ofp.to_int8_sat(ofp.apply_mult_shift(dx, m, sh, True, draw(dx.shape, 1 << sh)))
    t_batch = time.perf_counter() - t0
    t0 = time.perf_counter()
    dw = ofp.int_mm(g[:, :rows].T, x)
    t_dw = time.perf_counter() - t0
    t0 = time.perf_counter()
    gw = ofp.to_int8_sat(ofp.apply_mult_shift(dw, m, sh, True, draw(dw.shape, 1 << sh)))
    sub = ost.I8Linear(w[:rows].copy(), sw[:rows])
    sub.sx = 0.02
    sub._gw_i8, sub._gw_s = gw, 3e-5
    sub._gb_sum, sub._gb_s = g[:, :rows].astype(np.int64).sum(0), 3e-5
    ost.I8ECO([sub], lr=0.05).step(draw)
    t_rows = time.perf_counter() - t0
    t_full = LAYER_EQUIV * (t_batch * GLOBAL_BATCH / b + t_dw * (d / rows) * (GLOBAL_BATCH / b) + t_rows * d / rows)
    return {"value": 1.0 / t_full, "unit": "steps/s", "cores": threads, "kind": "port",
            "sample": f"numpy oracle port of one 8192x8192 layer: fwd+dX at batch {b} ({t_batch:.2f} s), dW GEMM "
                      f"{rows} rows x batch {b} ({t_dw:.2f} s), dW requant + I8ECO step on {rows} rows "
                      f"({t_rows:.2f} s); scaled by work to 9 layers x batch {GLOBAL_BATCH} (the compiled "
                      f"reference was absent)"}


def build_ref_module():
    from oracle import build_ref

    return build_ref


def run_reference_arm(args, rank):
    """``--impl reference``: the reference's own CPU strict step (rank 0 only)."""
    if rank != 0:
        return
    t_wall = time.perf_counter()
    r = reference_layer_steps(max_samples=args.steps, budget_s=60.0)
    if r is not None:
        times, info = r
        t = statistics.median(times)
        value = 1.0 / (t * LAYER_EQUIV)
        timed_steps = len(times) / LAYER_EQUIV  # training steps' worth of layer steps actually timed
        cb = {"value": value, "unit": "steps/s", "cores": info["threads"], "kind": "reference",
              "sample": f"reference ecoint8 {info['version']} (torch {info['torch']} CPU, compiled into oracle/_ref) "
                        f"strict step of one I8Linear(8192,8192)+I8ReLU at batch {GLOBAL_BATCH}: {len(times)} "
                        f"layer steps timed (of --steps {args.steps}, within a 60 s budget; one untimed first), "
                        f"median {t:.2f} s; x {LAYER_EQUIV:.3f} layer equivalents per training step"}
        ms = 1e3 * t * LAYER_EQUIV
        dtype = "int64"
        try:  # the rows next to the path, a bounded sample each
            cb["rows"] = reference_row_samples(build_ref_module().load())
        except Exception as e:  # noqa: BLE001 -- a missing row does not void the strict step's number
            cb["rows"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    else:
        cb = cpu_baseline_port()
        value, ms, timed_steps, dtype = cb["value"], 1e3 / cb["value"], None, "int64"
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s",
                      "n_gpus": args.gpus, "steps": timed_steps if timed_steps is not None else args.steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                      "vs_baseline": None, "dtype": dtype, "data": "synthetic",
                      "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH, "parallelism": "host cores",
                                 "wall_s": time.perf_counter() - t_wall},
                      "cpu_baseline": cb,
                      "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-side", action="store_true", help="skip the GEMM / step / CPU side measurements")
    ap.add_argument("--only", choices=["gemm", "gemm_sweep", "eco_step", "requant", "sgdm", "peak", "fp32_eco",
                                       "int8_linear", "boundary"],
                    help="run one side measurement alone (profiling)")
    ap.add_argument("--eco-layers", type=int, default=64, help="layers of 4096x4096 in the I8ECO step measurement")
    ap.add_argument("--sgdm-layers", type=int, default=64, help="layers of 4096x4096 in the EcoInt8SGDM measurement")
    ap.add_argument("--dw-exchange", default="peer", choices=["gather", "reduce", "peer"],
                    help="how ranks form the summed dW rows (ecoint8.parallel.init)")
    ap.add_argument("--comm-sms", type=int, default=16, help="SMs the GEMMs leave to the exchange under data parallelism")
    ap.add_argument("--push-ctas", type=int, default=32, help="CTAs per push kernel of the peer exchange")
    ap.add_argument("--trace", default=None, help="with --profile: write rank 0's chrome trace to this file")
    ap.add_argument("--no-graph", action="store_true",
                    help="issue every step from the host (default: capture the step once as a CUDA graph, "
                         "ecoint8.graphs.StepGraph, and replay it)")
    ap.add_argument("--profile", action="store_true",
                    help="after timing, run 3 steps under torch.profiler and print rank 0's GPU-time table")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank)

    sys.path.insert(0, str(REPO / "eco-int8-opt_b200"))
    import torch

    if args.only:
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        res = {"gemm": lambda: gemm_measurements(dev)[0], "gemm_sweep": lambda: gemm_sweep(dev),
               "requant": lambda: requant_measurement(dev), "fp32_eco": lambda: fp32_eco_measurement(dev),
               "int8_linear": lambda: int8_linear_measurement(dev), "boundary": lambda: boundary_measurement(dev), "sgdm": lambda: sgdm_measurement(dev, layers=args.sgdm_layers),
               "peak": lambda: int8_peak(dev),
               "eco_step": lambda: eco_step_measurement(dev, layers=args.eco_layers)}[args.only]()
        print(json.dumps({args.only: res}))
        return
    if args.gpus > 1 and world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} needs torchrun with {args.gpus} ranks (WORLD_SIZE={world})")

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    from ecoint8 import I8ECO, parallel
    from ecoint8._sr import batch_rows, set_generator
    from ecoint8.strict import iopt

    if world > 1:
        parallel.init(dw_exchange=args.dw_exchange, comm_sms=args.comm_sms, push_ctas=args.push_ctas)
    set_generator(torch.Generator().manual_seed(1234))  # identical Philox keys on every rank
    local_b = GLOBAL_BATCH // world
    net = build_mlp(device)
    x_fp, y, sx0 = global_batch(device, rank, world)
    with batch_rows(rank * local_b):
        from ecoint8.quant import quantize_symmetric

        net.calibrate(quantize_symmetric(x_fp, sx0), sx0)
        x_i8 = net.quantize_input(x_fp)[0]
        del x_fp
        opt = I8ECO(net.int8_layers(), lr=0.05, momentum=0.9)

        def barrier():
            if world > 1:
                torch.distributed.barrier()

        graph = None
        if args.no_graph:
            for _ in range(args.warmup):
                train_step(net, opt, x_i8, y)
        else:
            from ecoint8.graphs import StepGraph

            # the first warm-up step runs eagerly inside capture(); the graph then holds
            # one step's launches, counted while they are recorded
            graph = StepGraph(lambda: train_step(net, opt, x_i8, y), warmup=1)
            counter = LaunchCounter()
            with counter:
                graph.capture()
            graph_launches = counter.captured  # the launches recorded in the graph
            for _ in range(args.warmup - 1):
                graph.replay()
        step = graph.replay if graph is not None else (lambda: train_step(net, opt, x_i8, y))
        torch.cuda.synchronize()
        barrier()
        counter = LaunchCounter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk, counter:
            torch.cuda.synchronize()
            barrier()
            iopt.HOST_WAIT_S[0] = 0.0
            w0 = time.perf_counter()
            ev0.record()
            for _ in range(args.steps):
                step()
            ev1.record()
            host_wall = time.perf_counter() - w0
            host_blocked = iopt.HOST_WAIT_S[0]
            torch.cuda.synchronize()
            barrier()
        ms = ev0.elapsed_time(ev1)
        # with a graph: its recorded launches plus those issued after each replay (the weight
        # rows' pushes of the data-parallel exchange)
        launches = (graph_launches if graph is not None else 0) + counter.count // args.steps
        # e2e: the same steps through the public API with the int8 batch and labels coming
        # from pinned host memory and the loss read back every step; like a data loader,
        # the next step's batch crosses PCIe on a copy stream while this step computes
        x_host = x_i8.cpu().pin_memory()
        y_host = y.cpu().pin_memory()
        copy_stream = torch.cuda.Stream(device)
        cur = torch.cuda.current_stream(device)

        def fetch():
            with torch.cuda.stream(copy_stream):
                xb = x_host.to(device, non_blocking=True)
                yb = y_host.to(device, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
            return xb, yb, ev

        # with a graph: the batch lands in one of two staging buffers while the previous
        # step runs, and moves into the graph's input tensors at the start of its step
        stage = [(torch.empty_like(x_i8), torch.empty_like(y)) for _ in range(2)] if graph is not None else None
        used = [None, None]

        def fetch_staged(i):
            k = i % 2
            if used[k] is not None:
                copy_stream.wait_event(used[k])  # its last step has moved it into the inputs
            with torch.cuda.stream(copy_stream):
                stage[k][0].copy_(x_host, non_blocking=True)
                stage[k][1].copy_(y_host, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
            return ev

        # with a captured step, each step's loss comes back through pinned memory and is read
        # on the host one step later (as a training loop logs without stalling the device):
        # the host waits for step i - 1 while step i is queued behind it
        loss_host = torch.empty(2, dtype=torch.float32).pin_memory()
        losses = []
        pending = None

        def read(p):
            p[0].synchronize()
            losses.append(float(loss_host[p[1]]))

        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        copy_stream.wait_event(e0)  # the first batch's copy is inside the timed region too
        nxt = fetch() if graph is None else fetch_staged(0)
        for i in range(args.steps):
            if graph is None:
                xb, yb, ev = nxt
                cur.wait_event(ev)
                xb.record_stream(cur)
                yb.record_stream(cur)
                if i + 1 < args.steps:
                    nxt = fetch()
                loss = train_step(net, opt, xb, yb)
            else:
                cur.wait_event(nxt)
                x_i8.copy_(stage[i % 2][0])
                y.copy_(stage[i % 2][1])
                u = torch.cuda.Event()
                u.record(cur)
                used[i % 2] = u
                if i + 1 < args.steps:
                    nxt = fetch_staged(i + 1)
                loss = graph.replay()
            if world > 1:
                torch.distributed.all_reduce(loss)  # the mean over the global batch
            if graph is None:  # the uncaptured step: a blocking read measured faster (its host
                losses.append(float(loss.item()))  # issue, not the device, paces it)
                continue
            loss_host[i % 2].copy_(loss.reshape(()), non_blocking=True)
            done = torch.cuda.Event()
            done.record(cur)
            if pending is not None:
                read(pending)
            pending = (done, i % 2)
        e1.record()
        if pending is not None:
            read(pending)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = e0.elapsed_time(e1)
        if args.profile:
            from torch.profiler import ProfilerActivity, profile

            with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
                for _ in range(3):
                    step()
                torch.cuda.synchronize()
            if rank == 0:
                print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=70),
                      file=sys.stderr)
                if args.trace:
                    prof.export_chrome_trace(args.trace)
        digest = weights_digest(net, opt, world)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = t.tolist()
    value = args.steps / (ms / 1e3)
    e2e = args.steps / (ms_e2e / 1e3)
    if rank == 0:
        hbm, bf16, src = _peaks()
        out = {"metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "int8/int32/int64", "data": "synthetic",
               "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH, "per_gpu_batch": local_b,
                          "parallelism": f"dp{world}", "dw_exchange": args.dw_exchange if world > 1 else None,
                          "comm_sms": args.comm_sms if world > 1 else None,
                          "push_ctas": args.push_ctas if world > 1 and args.dw_exchange == "peer" else None,
                          "l2": "inputs larger than L2 (1.2 GB activations + 0.55 GB weights); no flush",
                          "data": "global batch drawn once from seed 100, rows split across ranks"},
               "e2e": {"value": e2e, "unit": "steps/s", "h2d_bytes_per_step": int(x_i8.numel() + y.numel() * 8),
                       "d2h_bytes_per_step": 4,
                       "result_read": ("each step's loss copied to pinned memory and read on the host one step later"
                                       if graph is not None else "each step's loss read with .item()")},
               "gpu_launches": launches, "cuda_graph": graph is not None, "clocks": clk.summary(),
               "host": {"issue_ms_per_step": 1e3 * (host_wall - host_blocked) / args.steps,
                        "blocked_ms_per_step": 1e3 * host_blocked / args.steps},
               "weights_digest": digest}
        if world == 1 and not args.no_side:
            gm, times, ops = gemm_measurements(device)
            out["gemm"] = gm
            peak, peak_where = int8_peak(device)
            gm["int8_peak_tops"], gm["int8_peak_source"] = peak, peak_where
            out["eco_step"] = eco_step_measurement(device)
            out["eco_step"]["frac_of_hbm"] = out["eco_step"]["gbs"] / hbm
            out["sgdm_step"] = sgdm_measurement(device)
            out["sgdm_step"]["frac_of_hbm"] = out["sgdm_step"]["gbs"] / hbm
            out["requant"] = requant_measurement(device)
            out["fp32_eco"] = fp32_eco_measurement(device)
            for k in ("sgdm", "adam"):
                out["fp32_eco"][k]["frac_of_hbm"] = out["fp32_eco"][k]["gbs"] / hbm
            out["int8_linear"] = int8_linear_measurement(device)
            out["int8_linear"]["frac_of_peak"] = out["int8_linear"]["tops"] / peak
            out["loss_boundary"] = boundary_measurement(device)
            achieved = ops / times["dx"] / 1e12
            out["roofline"] = {"bound": "tensor",
                               "kernel": ("gemm_s8_pair_kernel<0>" if os.environ.get("ECO_GEMM_PAIRS", "1") != "0"
                                          else "gemm_s8_kernel<256,0>")
                                         + " (int32 + max|C|, the dX GEMM: 16384x8192x8192, B MN-major; "
                                           "the step's dX and dW GEMMs are this kernel)",
                               "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                               "peak_source": f"measured int8 dense peak on this GPU: best of {peak_where} "
                                              f"(2 x {src} bf16 = {2 * bf16:.0f} for context)",
                               "frac": achieved / peak, "traffic": _traffic("gemm_pair_dx_16384x8192x8192.md"),
                               "dw": {"achieved": ops / times["dw"] / 1e12, "frac": ops / times["dw"] / 1e12 / peak,
                                      "shape": "8192x8192 over batch 16384, A and B MN-major"},
                               "fused_forward": {"achieved": ops / times["fused"] / 1e12,
                                                 "frac": ops / times["fused"] / 1e12 / peak}}
            out["cpu_baseline"] = cpu_baseline_subprocess()
            out["rows_vs_reference_cpu"] = row_ratios(out, out["cpu_baseline"].get("rows") or {})
        print(json.dumps(out))
    if world > 1:
        parallel.shutdown()
        torch.distributed.destroy_process_group()


def _traffic(name):
    """DRAM bytes per launch of the roofline kernel, from its committed ncu summary (or None)."""
    p = REPO / "profiles" / name
    if p.exists():
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    return None


if __name__ == "__main__":
    main()
