"""EcoInt8SGDM's fused optimizer step, restated in numpy fp32 (oracle; test infrastructure only).

Follows the two-pass algorithm of ``ecoint8/triton_kernels.py`` (v0.4.9):

* host: ``sg = clamp(max|g|, 1e-12) / 127`` (triton_kernels.py:156);
* pass 1, ``eco_amax_kernel`` (:67-90): per element ``_eco_elem`` (:54-65) with
  draws ``tl.rand(seed, 2i)`` / ``tl.rand(seed, 2i+1)``; block maxima of ``|m_new|``
  over blocks of 1024 elements;
* host: ``sm_new = max(partials) / 127`` (:163);
* pass 2, ``eco_fused_kernel`` (:92-119): the same element math with draws
  ``tl.rand(seed, 3i + {0, 1})`` and ``mq = clamp(floor(m_new / (sm_new + 1e-8) +
  tl.rand(seed, 3i+2)))``; stores ``w`` and ``m``; the momentum scale becomes
  ``sm_new`` (:169).

Every operation is one IEEE fp32 operation in the order written (no fused
multiply-add), which is what Triton's interpreter computes.  The two scalar
divisions by 127 follow either PyTorch's CPU kernel (``division="cpu"``: a true
division) or its CUDA kernel, which multiplies by the reciprocal (taken in double,
rounded to fp32; for 127 that equals the fp32 reciprocal) when the divisor is a CPU
scalar (``division="cuda"``).
"""

from __future__ import annotations

import numpy as np

from .philox import tl_rand

BLOCK = 1024  # triton_kernels.py:48
f32 = np.float32


def _div127(x: np.float32, division: str) -> np.float32:
    if division == "cpu":
        return f32(f32(x) / f32(127.0))
    return f32(f32(x) * f32(f32(1.0) / f32(127.0)))


def eco_elem(w, m, g, sw, sm, sg, wd, lr, beta, alpha, r_g, r_w):
    """triton_kernels.py:54-65, fp32 throughout."""
    w = w.astype(f32)
    m = m.astype(f32)
    gv = (g + (w * sw) * wd) / sg
    gq = np.minimum(np.maximum(np.floor(gv + r_g), f32(-127.0)), f32(127.0))
    g_hat = gq * sg
    one_m_beta = f32(f32(1.0) - beta)
    m_tilde = ((beta * m) * sm) + (one_m_beta * g_hat)
    th = (w * sw) - (lr * m_tilde)
    wq = np.minimum(np.maximum(np.floor((th / sw) + r_w), f32(-127.0)), f32(127.0))
    e = th - (wq * sw)
    m_new = m_tilde + (alpha * e)
    return wq.astype(np.int8), m_new.astype(f32)


def triton_step(w, m, g, sw, sm, *, lr, beta, wd, seed, division="cuda"):
    """One EcoInt8SGDM fused step on a ``[out, in]`` layer.  Returns the new state."""
    w = np.asarray(w, dtype=np.int8)
    m = np.asarray(m, dtype=np.int8)
    g = np.asarray(g, dtype=f32)
    out_f, in_f = w.shape
    n = w.size
    idx = np.arange(n, dtype=np.int64)
    wf, mf, gf = w.reshape(-1), m.reshape(-1), g.reshape(-1)
    swe = np.asarray(sw, dtype=f32)[idx // in_f]
    sm = f32(np.asarray(sm, dtype=f32).reshape(()))
    sg = _div127(f32(max(f32(np.abs(gf).max()), f32(1e-12))), division)
    alpha = (1.0 / lr) * (1.0 - 1.0 / beta)  # host double, passed as fp32
    wd_, lr_, beta_, alpha_ = f32(wd), f32(lr), f32(beta), f32(alpha)
    # int32 offsets, as in the kernels (wrap past 2**31 like Triton's int32 arithmetic)
    off = lambda k, j: ((idx * k + j) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)  # noqa: E731
    _, m_new1 = eco_elem(wf, mf, gf, swe, sm, sg, wd_, lr_, beta_, alpha_,
                         tl_rand(seed, off(2, 0)), tl_rand(seed, off(2, 1)))
    grid = (n + BLOCK - 1) // BLOCK
    a = np.abs(m_new1)
    pad = np.zeros(grid * BLOCK, dtype=f32)
    pad[:n] = a
    partials = pad.reshape(grid, BLOCK).max(axis=1).astype(f32)
    sm_new = _div127(f32(partials.max()), division)
    wq, m_new2 = eco_elem(wf, mf, gf, swe, sm, sg, wd_, lr_, beta_, alpha_,
                          tl_rand(seed, off(3, 0)), tl_rand(seed, off(3, 1)))
    smg = f32(sm_new + f32(1e-8))
    mq = np.minimum(np.maximum(np.floor((m_new2 / smg) + tl_rand(seed, off(3, 2))), f32(-127.0)),
                    f32(127.0))
    return {"w": wq.reshape(out_f, in_f), "m": mq.astype(np.int8).reshape(out_f, in_f),
            "sg": np.array(sg, dtype=f32), "sm_new": np.array(sm_new, dtype=f32),
            "partials": partials}
