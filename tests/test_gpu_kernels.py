"""Kernel parity on a B200: every C-ABI kernel against the CPU oracle, bit for bit.

Integer work, so the bar is exact equality.  Stochastic rounding is checked in
all three modes: round-half-up, replay of the reference's torch.randint draws,
and the library's Philox stream (reproduced by ``oracle/philox.py``).
"""

import math

import numpy as np
import pytest
import torch

from oracle import fixedpoint as ofp
from oracle import philox as oph

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (2, 10, 3), (17, 33, 65), (128, 128, 128), (129, 257, 255), (300, 1000, 784),
          (256, 64, 4097), (64, 2, 256), (1000, 130, 16)]


def _i8(shape, gen):
    return torch.randint(-127, 128, shape, dtype=torch.int8, generator=gen)


def _operands(M, N, K, a_layout, b_layout, gen):
    A = _i8((M, K), gen)
    B = _i8((K, N), gen)
    a_store = A if a_layout == 0 else A.t().contiguous()
    b_store = B.t().contiguous() if b_layout == 0 else B
    return A, B, a_store.cuda(), b_store.cuda()


@pytest.mark.parametrize("a_layout,b_layout", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_s32_all_layouts_exact(a_layout, b_layout):
    from ecoint8 import _ops

    gen = torch.Generator().manual_seed(10 * a_layout + b_layout)
    for M, N, K in SHAPES:
        A, B, a, b = _operands(M, N, K, a_layout, b_layout, gen)
        bias = torch.randint(-(1 << 20), 1 << 20, (N,), dtype=torch.int32, generator=gen)
        amax = torch.empty(1, dtype=torch.int32, device="cuda")
        C = _ops.gemm_s32(a, a_layout, b, b_layout, M, N, K, bias=bias.cuda(), amax=amax)
        ref = ofp.int_mm(A.numpy(), B.numpy()).astype(np.int64) + bias.numpy()
        ref = ref.astype(np.int32)
        got = C.cpu().numpy()
        assert np.array_equal(got, ref), (M, N, K, a_layout, b_layout)
        assert int(amax.item()) == int(np.abs(ref.astype(np.int64)).max()), (M, N, K)


def test_gemm_s32_matches_cublas_at_4096_and_4097():
    """Full-size C3 shapes: the int8 GEMM equals torch._int_mm (cuBLASLt) exactly."""
    from ecoint8 import _ops

    gen = torch.Generator(device="cuda").manual_seed(3)
    for M, N, K in [(4096, 4096, 4096), (4097, 4097, 4096), (1024, 8192, 1024)]:
        A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=gen)
        Bt = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=gen)
        C = _ops.gemm_s32(A, 0, Bt, 0, M, N, K)
        Mp, Kp, Np = ofp.pad_mm_dims(M, K, N)
        ref = torch._int_mm(torch.nn.functional.pad(A, (0, Kp - K, 0, Mp - M)),
                            torch.nn.functional.pad(Bt.t(), (0, Np - N, 0, Kp - K)))[:M, :N]
        assert torch.equal(C, ref), (M, N, K)


def _ratios(N, gen):
    lo, hi = math.log(1e-4), math.log(1e-1)
    return [float(v) for v in torch.exp(torch.empty(N, dtype=torch.float64).uniform_(lo, hi, generator=gen))]


@pytest.mark.parametrize("mode", ["nearest", "replay", "philox"])
@pytest.mark.parametrize("relu", [False, True])
def test_gemm_requant_fused_epilogue_exact(mode, relu):
    from ecoint8 import _native, _ops, _sr

    gen = torch.Generator().manual_seed(7)
    for M, N, K in [(64, 48, 40), (33, 17, 9), (300, 1000, 784), (129, 257, 4097), (1, 16, 16)]:
        A, B, a, b = _operands(M, N, K, 0, 0, gen)
        bias = torch.randint(-3000, 3000, (N,), dtype=torch.int32, generator=gen)
        mults, com = ofp.col_mults(_ratios(N, gen))
        acc = (ofp.int_mm(A.numpy(), B.numpy()).astype(np.int64) + bias.numpy()).astype(np.int32)
        if mode == "nearest":
            site = _sr.Site(_native.sr_spec(_native.SR_NEAREST), None)
            nud = None
            stoch = False
        elif mode == "replay":
            dt = torch.int32 if (1 << com) <= (1 << 31) else torch.int64
            nt = torch.randint(0, 1 << com, (M, N), dtype=dt, generator=gen)
            site = _sr.Site(_native.sr_spec(_native.SR_REPLAY32 if dt == torch.int32 else _native.SR_REPLAY64,
                                            nt.cuda()), nt.cuda())
            nud, stoch = nt.numpy().astype(np.int64), True
        else:
            key, rb = 0x1234_5678_9ABC + M, 5 * M
            site = _sr.Site(_native.sr_spec(_native.SR_PHILOX, seed=key, stream_id=3, row_base=rb), None)
            nud, stoch = oph.sr_nudge(key, 3, (M, N), com, row_base=rb), True
        y = _ops.gemm_requant(a, 0, b, 0, M, N, K, bias.cuda(), torch.from_numpy(mults).cuda(), com, relu, site)
        ref = ofp.to_int8_sat(ofp.apply_mult_shift(acc.astype(np.int64), mults, com, stoch, nud))
        if relu:
            ref = np.maximum(ref, 0).astype(np.int8)
        assert np.array_equal(y.cpu().numpy(), ref), (mode, M, N, K)


@pytest.mark.parametrize("mode", ["nearest", "replay", "philox"])
def test_requant_kernel_with_mask_and_square_sum(mode):
    from ecoint8 import _native, _ops, _sr

    gen = torch.Generator().manual_seed(8)
    for rows, cols in [(1, 1), (7, 13), (64, 256), (33, 1000), (257, 16)]:
        src = torch.randint(-(1 << 30), 1 << 30, (rows, cols), dtype=torch.int32, generator=gen)
        mask = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, generator=gen)
        mult = int(torch.randint(1 << 30, 1 << 31, (1,), generator=gen).item())
        shift = 37
        if mode == "nearest":
            site, nud = _sr.Site(_native.sr_spec(_native.SR_NEAREST), None), None
        elif mode == "replay":
            nt = torch.randint(0, 1 << shift, (rows, cols), dtype=torch.int64, generator=gen)
            site, nud = _sr.Site(_native.sr_spec(_native.SR_REPLAY64, nt.cuda()), None), nt.numpy()
            site.nudge = nt.cuda()
            site.spec.nudge = site.nudge.data_ptr()
        else:
            site = _sr.Site(_native.sr_spec(_native.SR_PHILOX, seed=99, stream_id=rows, row_base=0), None)
            nud = oph.sr_nudge(99, rows, (rows, cols), shift)
        sq = torch.empty(1, dtype=torch.int64, device="cuda")
        y = _ops.requant(src.cuda(), mult, shift, site, mask=mask.cuda(), sumsq=sq)
        ref = ofp.to_int8_sat(ofp.apply_mult_shift(src.numpy(), mult, shift, mode != "nearest", nud))
        ref = np.where(mask.numpy() > 0, ref, 0).astype(np.int8)
        assert np.array_equal(y.cpu().numpy(), ref), (mode, rows, cols)
        assert int(sq.item()) == int((ref.astype(np.int64) ** 2).sum())


def test_apply_mult_shift_reference_cases(golden):
    """fixedpoint.apply_mult_shift on CUDA tensors against the reference's own outputs."""
    import ecoint8
    from ecoint8 import fixedpoint as fp

    for case in golden("fixedpoint.json")["apply_mult_shift"]:
        dt = torch.int32 if "int32" in case["dtype"] else torch.int64
        x = torch.tensor(case["x"], dtype=torch.int64).to(dt).cuda()
        mult = case["mult"]
        if not isinstance(mult, int):
            mult = torch.tensor(mult, dtype=torch.int32).cuda()
        nud = case["nudge"]
        with ecoint8.sr_replay(lambda shape, denom, device: torch.tensor(nud, dtype=torch.int64)):
            out = fp.apply_mult_shift(x, mult, case["shift"], case["stochastic"])
        assert out.cpu().tolist() == case["out"], case["mult_kind"]


def test_reductions_colsum_amax_sumsq():
    from ecoint8 import _ops

    gen = torch.Generator().manual_seed(2)
    for rows, cols in [(1, 1), (5, 3), (16384, 10), (300, 8192), (16384, 1000), (7, 48), (1, 40), (2000, 4104)]:
        g = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, generator=gen)
        assert torch.equal(_ops.colsum(g.cuda()).cpu(), g.to(torch.int64).sum(0))
        # a view with 16-byte padded rows (the loss boundary's layout): 16 columns per thread
        pad = torch.zeros((rows, (cols + 15) // 16 * 16), dtype=torch.int8)
        pad[:, :cols] = g
        assert torch.equal(_ops.colsum(pad.cuda()[:, :cols]).cpu(), g.to(torch.int64).sum(0))
        assert int(_ops.sumsq(g.cuda()).item()) == int((g.to(torch.int64) ** 2).sum())
        x = torch.randint(-(1 << 31) + 1, 1 << 31, (rows, cols), dtype=torch.int64, generator=gen).to(torch.int32)
        assert int(_ops.amax(x.cuda()).item()) == int(x.to(torch.int64).abs().max())


def test_split_cols_matches_block_transpose():
    """eco_split_cols_s8 (the all-to-all send layout) equals the reshaped transpose."""
    from ecoint8 import _native

    gen = torch.Generator().manual_seed(3)
    for rows, cols, parts, ld in [(48, 48, 2, 48), (2048, 8192, 8, 8192), (7, 30, 3, 33), (5, 1000, 8, 1000)]:
        full = torch.randint(-127, 128, (rows, ld), dtype=torch.int8, generator=gen).cuda()
        src = full[:, :cols]
        dst = torch.empty((parts, rows, cols // parts), dtype=torch.int8, device="cuda")
        _native.call("eco_split_cols_s8", src.data_ptr(), ld, rows, cols, parts, dst.data_ptr(), _native.stream())
        want = src.reshape(rows, parts, cols // parts).transpose(0, 1)
        assert torch.equal(dst, want), (rows, cols, parts)


def test_copy2d_relayout_from_any_alignment():
    """eco_copy2d_s8 (the operand relayout before the GEMM's 16-byte TMA rows): rows of any
    start offset and width into a 16-byte aligned buffer, and into an unaligned one (the
    library's generic 2-D copy); bytes outside the copied columns are left alone."""
    from ecoint8 import _native

    gen = torch.Generator().manual_seed(4)
    for rows, cols, ld, off in [(1, 1, 1, 0), (3, 17, 19, 1), (5, 16, 16, 3), (64, 4097, 4097, 0), (9, 35, 40, 2),
                                (300, 1000, 1003, 1), (2, 20, 21, 3)]:
        flat = torch.randint(-127, 128, (off + rows * ld + 5,), dtype=torch.int8, generator=gen).cuda()
        src = flat[off:off + rows * ld].view(rows, ld)[:, :cols]
        for ld_dst, dst_off in [((cols + 15) // 16 * 16, 0), (cols + 3, 1)]:
            base = torch.full((dst_off + rows * ld_dst,), 55, dtype=torch.int8, device="cuda")
            dst = base[dst_off:].view(rows, ld_dst)
            _native.call("eco_copy2d_s8", src.data_ptr(), ld, dst.data_ptr(), ld_dst, rows, cols, _native.stream())
            assert torch.equal(dst[:, :cols], src), (rows, cols, ld, off, ld_dst)
            assert bool((dst[:, cols:] == 55).all()) and bool((base[:dst_off] == 55).all())


def test_peer_push_signal_and_bounded_wait_on_one_gpu():
    """The peer-exchange kernels with this GPU's own buffers as the only 'peer': both
    push modes land where the layout says, a signalled slot releases the wait, and
    a slot nobody signals times out into the sticky error flags (no hang)."""
    import ctypes

    from ecoint8 import _native

    s = _native.stream()
    gen = torch.Generator().manual_seed(4)
    for rows, cols in [(48, 40), (64, 256)]:
        src = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, generator=gen).cuda()
        dst = torch.zeros((3 * rows, cols), dtype=torch.int8, device="cuda")
        arr = (ctypes.c_void_p * 1)(dst.data_ptr())
        _native.call("eco_peer_push_s8", src.data_ptr(), cols, rows, cols, arr, 1, cols, rows, 0, 4, s)
        assert torch.equal(dst[rows:2 * rows], src) and not dst[:rows].any() and not dst[2 * rows:].any()
        dsts = [torch.zeros((2 * rows, cols // 2), dtype=torch.int8, device="cuda") for _ in range(2)]
        arr = (ctypes.c_void_p * 2)(*[d.data_ptr() for d in dsts])
        _native.call("eco_peer_push_s8", src.data_ptr(), cols, rows, cols, arr, 2, cols // 2, rows, 1, 4, s)
        for p, d in enumerate(dsts):
            assert torch.equal(d[rows:], src[:, p * cols // 2:(p + 1) * cols // 2]) and not d[:rows].any()
    flags = torch.zeros((4, 8), dtype=torch.int64, device="cuda")
    fl = (ctypes.c_void_p * 1)(flags.data_ptr())
    torch.cuda.synchronize()
    assert _native.read_device_errors() == 0
    _native.call("eco_peer_signal", fl, 1, 0, 2, 7, None, s)
    _native.call("eco_peer_wait", flags.data_ptr(), 1, 2, 7, None, 100000, s)
    torch.cuda.synchronize()
    assert int(flags[2, 0]) == 7 and _native.read_device_errors() == 0
    # epochs read from device memory when the kernels run (as a replayed CUDA graph does)
    word = torch.tensor([9], dtype=torch.int64, device="cuda")
    _native.call("eco_peer_signal", fl, 1, 0, 2, 0, word.data_ptr(), s)
    _native.call("eco_peer_wait", flags.data_ptr(), 1, 2, 0, word.data_ptr(), 100000, s)
    torch.cuda.synchronize()
    assert int(flags[2, 0]) == 9 and _native.read_device_errors() == 0
    # push and signal in one launch (every CTA fenced first); the ticket returns to zero
    src = torch.randint(-127, 128, (300, 64), dtype=torch.int8, generator=gen).cuda()
    dst = torch.zeros((300, 64), dtype=torch.int8, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    arr = (ctypes.c_void_p * 1)(dst.data_ptr())
    _native.call("eco_peer_push_signal_s8", src.data_ptr(), 64, 300, 64, arr, 1, 64, 0, 0, 7, fl, 1, 0, 1, 3, None,
                 ticket.data_ptr(), s)
    _native.call("eco_peer_wait", flags.data_ptr(), 1, 1, 3, None, 100000, s)
    torch.cuda.synchronize()
    assert torch.equal(dst, src) and int(flags[1, 0]) == 3 and int(ticket) == 0
    assert _native.read_device_errors() == 0
    _native.call("eco_peer_wait", flags.data_ptr(), 1, 3, 1, None, 100000, s)  # nothing signals slot 3
    torch.cuda.synchronize()
    assert _native.read_device_errors() == 4
    assert _native.read_device_errors() == 0  # the read clears the flags


def test_library_reports_no_device_timeouts():
    from ecoint8 import _native

    torch.cuda.synchronize()
    assert _native.read_device_errors() == 0
