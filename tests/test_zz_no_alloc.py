"""The allocation-free GEMM entry point against the regular one (GPU).

``eco_gemm_s8s32_noalloc`` exists for callers that cannot allocate device
memory -- code running under stream capture, runtimes that plan all memory
ahead, plain C hosts.  It relayouts operands that break the 16-byte TMA rule
into a buffer the library owns, where ``eco_gemm_s8s32`` needs the caller to
provide an aligned copy.  Both must give the same int32 result and max|C|.
This file is collected last so a failure here leaves every other test run.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(a, lda, a_layout, b, ldb, b_layout, M, N, K, bias):
    from ecoint8 import _native

    c = torch.empty((M, N), dtype=torch.int32, device="cuda")
    amax = torch.empty(1, dtype=torch.int32, device="cuda")
    rc = _native.load().eco_gemm_s8s32_noalloc(a, lda, a_layout, b, ldb, b_layout, M, N, K, bias, c.data_ptr(),
                                               N, amax.data_ptr(), _native.stream())
    assert rc == 0, _native.last_error()
    return c, amax


def test_noalloc_gemm_equals_regular_gemm_on_two_calls_in_a_row():
    from ecoint8 import _ops

    gen = torch.Generator(device="cuda").manual_seed(0)
    # call 1: dW-like, A = g^T with g stored [K=256, M=10] (leading dim 10 breaks the rule)
    g = torch.randint(-127, 128, (256, 10), dtype=torch.int8, device="cuda", generator=gen)
    x = torch.randint(-127, 128, (256, 96), dtype=torch.int8, device="cuda", generator=gen)
    # call 2: dX-like, A = [512, 1000] (leading dim 1000) and B a view starting 3 bytes in
    a2 = torch.randint(-127, 128, (512, 1000), dtype=torch.int8, device="cuda", generator=gen)
    big = torch.randint(-127, 128, (1000, 800), dtype=torch.int8, device="cuda", generator=gen)
    b2 = big[:, 3:787]
    bias = torch.randint(-1000, 1000, (784,), dtype=torch.int32, device="cuda", generator=gen)
    calls = [
        (g, 10, 1, x, 96, 1, 10, 96, 256, None),
        (a2, 1000, 0, b2, 800, 1, 512, 784, 1000, bias),
    ]
    for a, lda, al, b, ldb, bl, M, N, K, bi in calls:
        amax_ref = torch.empty(1, dtype=torch.int32, device="cuda")
        ref = _ops.gemm_s32(a, al, b, bl, M, N, K, bias=bi, amax=amax_ref)
        got, amax = _noalloc(a.data_ptr(), lda, al, b.data_ptr(), ldb, bl, M, N, K,
                             None if bi is None else bi.data_ptr())
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
        assert int(amax.item()) == int(amax_ref.item())


def test_noalloc_gemm_rejects_relayouts_beyond_its_buffer():
    from ecoint8 import _native

    a = torch.zeros((40000, 1000), dtype=torch.int8, device="cuda")  # 40 MB to relayout
    b = torch.zeros((40000, 16), dtype=torch.int8, device="cuda")
    c = torch.empty((1000, 16), dtype=torch.int32, device="cuda")
    rc = _native.load().eco_gemm_s8s32_noalloc(a.data_ptr(), 1000, 1, b.data_ptr(), 16, 1, 1000, 16, 40000, None,
                                               c.data_ptr(), 16, None, _native.stream())
    assert rc == -1 and "scratch" in _native.last_error()
