"""fp32 boundary of the strict path and the seeded workloads (oracle; test infrastructure only).

The strict region is entered and left through fp32 code the reference keeps in
``ecoint8/quant.py`` (entry quantization, ``quantize_tensor_dynamic`` on the
loss gradient).  These are restated with torch CPU ops so that they consume the
global torch generator exactly as the reference does (``quant.py:9-38``).

The seeded workloads (the 32-64-2 blob task, the 784-256-128-10 MNIST-shaped
task) are defined here once, so the golden generator, the oracle tests and the
GPU parity tests build identical inputs.
"""

from __future__ import annotations

import math

EPS = 1e-8  # quant.py:7


def calc_scale(amax: float, clip=None) -> float:
    """quant.py:9-16."""
    a = float(amax)
    if clip is not None:
        a = min(a, clip)
    if a < EPS:
        return 1.0
    return a / 127.0


def quantize_symmetric(x, scale, stochastic=False):
    """quant.py:19-28 (torch CPU or CUDA tensors; uses the global generator)."""
    import torch

    s = scale + EPS
    v = x / s
    if stochastic:
        q = torch.floor(v + torch.rand_like(v))
    else:
        q = torch.round(v)
    return torch.clamp(q, -127, 127).to(torch.int8)


def quantize_tensor_dynamic(x, stochastic=False):
    """quant.py:35-38."""
    amax = x.detach().abs().max().item()
    return quantize_symmetric(x, calc_scale(amax), stochastic), calc_scale(amax)


def ce_grad(logits_i8, s_out, y):
    """Loss boundary: dequantize logits, CrossEntropy, gradient (examples/i8_demo.py:56-59)."""
    import torch
    import torch.nn as nn

    logits_fp = (logits_i8.to(torch.float32) * s_out).requires_grad_()
    loss = nn.CrossEntropyLoss()(logits_fp, y)
    (g_fp,) = torch.autograd.grad(loss, logits_fp)
    return loss.detach(), g_fp


# --- seeded workloads -------------------------------------------------------

BLOB_N, BLOB_D, BLOB_H = 256, 32, 64


def blob_data():
    """2-class Gaussian blobs: means +-1 on all 32 dims, std 1; labels uniform {0,1}.

    Call right after ``torch.manual_seed(0)``; draws labels then features.
    """
    import torch

    y = torch.randint(0, 2, (BLOB_N,))
    X = torch.randn(BLOB_N, BLOB_D) + (2.0 * y.to(torch.float32) - 1.0).unsqueeze(1)
    return X, y


def blob_lr(ep: int, epochs: int = 150, lr0: float = 0.5) -> float:
    """Cosine-decayed lr (examples/i8_demo.py:30-31 form) starting at 0.5."""
    return lr0 * 0.5 * (1 + math.cos(math.pi * ep / epochs)) + 1e-4


MNIST_SHAPE = (784, 256, 128, 10)
MNIST_B = 128
MNIST_SAMPLES = 60000


def mnist_batch(index: int, batch: int = MNIST_B):
    """One batch of the MNIST-shaped synthetic set: pixel 0 w.p. 0.8 else U[0,1]; labels U{0..9}.

    Batch ``index`` is drawn from its own generator (seed 1000 + index), so any
    batch can be rebuilt without generating the 60000-sample set.
    """
    import torch

    gen = torch.Generator().manual_seed(1000 + index)
    X = torch.rand(batch, MNIST_SHAPE[0], generator=gen)
    keep = torch.rand(batch, MNIST_SHAPE[0], generator=gen) >= 0.8
    X = X * keep.to(torch.float32)
    y = torch.randint(0, 10, (batch,), generator=gen)
    return X, y


MNIST_GOLDEN_STEPS = 2345  # steps of the MNIST-shaped run pinned by the golden fixture: 5 epochs of 60000 at 128
MNIST_EPOCH_STEPS = 469  # one epoch (the CPU oracle test checks this many)

WIDE_D, WIDE_C, WIDE_B = 8192, 1000, 1024  # config-5 layer widths, the golden fixture's batch


def wide_batch():
    """Config-5-shaped inputs: Gaussian features ``[1024, 8192]`` and labels uniform over 1000
    classes, from their own generator (seed 2000)."""
    import torch

    gen = torch.Generator().manual_seed(2000)
    X = torch.randn(WIDE_B, WIDE_D, generator=gen)
    y = torch.randint(0, WIDE_C, (WIDE_B,), generator=gen)
    return X, y


def mnist_lr(step: int, total: int, lr0: float = 0.08) -> float:
    """Cosine lr over ``total`` steps (lr0 = 0.08 as in examples/mem_probe.py:83)."""
    return lr0 * 0.5 * (1 + math.cos(math.pi * step / total)) + 1e-4
