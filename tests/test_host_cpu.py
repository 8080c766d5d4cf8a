"""Host-side checks that need no GPU: the C ABI library, the drop-in surface, host logic."""

import pathlib
import re

import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "ecoint8_b200.h"
PKG = REPO / "eco-int8-opt_b200" / "ecoint8"


def _header_functions():
    return re.findall(r"^ECO_API\s+[\w\s\*]+?\b(eco_\w+)\s*\(", HEADER.read_text(), flags=re.M)


def test_library_loads_and_exports_every_header_symbol():
    from ecoint8 import _native

    lib = _native.load()
    names = _header_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(names) == sorted(_native.exported_symbols())
    assert lib.eco_abi_version() == 4


def test_c_abi_rejects_bad_arguments_with_a_message():
    """Argument errors come back as status codes with eco_last_error(), no device work."""
    from ecoint8 import _native

    lib = _native.load()
    rc = lib.eco_colsum_s8(None, 4, 4, 4, None, None)
    assert rc == -1 and "bad arguments" in _native.last_error()
    spec = _native.sr_spec(_native.SR_REPLAY32)
    rc = lib.eco_requant_s32_s8(1, 1, 1, 1, None, None, 1, 5, 0, spec, None, 0, 1, 1, None, None)
    assert rc == -1 and "nudge" in _native.last_error()
    spec = _native.sr_spec(_native.SR_NEAREST)
    rc = lib.eco_requant_s32_s8(1, 1, 1, 1, None, None, 1, 63, 0, spec, None, 0, 1, 1, None, None)
    assert rc == -5 and "62" in _native.last_error()
    rc = lib.eco_gemm_s8s32(16, 10, 0, 32, 16, 0, 4, 4, 4, None, 64, 4, None, None)
    assert rc == -2 and "aligned" in _native.last_error()


def test_no_cpu_path_fails_loudly():
    from ecoint8 import I8Linear, I8ECO
    from ecoint8 import fixedpoint as fp

    torch.manual_seed(0)
    lin = I8Linear(32, 16)
    lin.sx, lin.sy = 0.01, 0.05
    with pytest.raises(RuntimeError, match="CUDA"):
        lin.forward_i8(torch.zeros(4, 32, dtype=torch.int8))
    with pytest.raises(RuntimeError, match="CUDA"):
        fp.apply_mult_shift(torch.ones(3, dtype=torch.int32), 3, 2)
    lin._gw_i8 = torch.zeros(16, 32, dtype=torch.int8)
    lin._gw_s = 1e-3
    with pytest.raises(RuntimeError, match="CUDA"):
        I8ECO([lin]).step()
    from ecoint8 import EcoAdam, EcoSGDM, Int8Linear

    fl = Int8Linear(16, 8)
    fl._grad_w = torch.zeros(8, 16)
    for opt in (EcoSGDM([fl]), EcoAdam([fl])):
        with pytest.raises(RuntimeError, match="CUDA"):
            opt.step()


STRICT = ["fixedpoint.py", "strict/ilayer.py", "strict/iopt.py"]
BANNED = [".float(", "torch.float32", "torch.float(", "to(torch.float", ".double("]


def test_no_float_ops_in_strict_sources():
    """The reference's static audit (tests/test_strict.py:17-32) on the drop-in's sources."""
    for name in STRICT:
        src = (PKG / name).read_text()
        for pat in BANNED:
            assert pat not in src, f"{name} contains banned {pat!r}"


def test_public_api_matches_reference_surface():
    import ecoint8
    from ecoint8 import fixedpoint, quant
    from ecoint8.strict import I8ECO, I8Linear, I8ReLU, I8Sequential  # noqa: F401
    from ecoint8.triton_kernels import TRITON_AVAILABLE, triton_eco_step_  # noqa: F401

    for name in ["EcoInt8SGDM", "EcoSGDM", "EcoAdam", "I8ECO", "I8Linear", "I8ReLU", "I8Sequential", "Int8Linear",
                 "to_int8", "quantize_symmetric", "quantize_tensor_dynamic", "quantize_per_channel", "dequantize"]:
        assert hasattr(ecoint8, name), name
    assert ecoint8.__version__ == "0.4.9"
    for name in ["quantize_multiplier", "apply_mult_shift", "to_int8_sat", "int_amax", "pad_mm_dims",
                 "dynamic_scale_from_int", "_check_int", "_sr_nudge"]:
        assert hasattr(fixedpoint, name), name
    for name in ["calc_scale", "quantize_symmetric", "quantize_tensor_dynamic", "quantize_per_channel",
                 "dequantize", "saturation_ratio"]:
        assert hasattr(quant, name), name
    # the fp32-state optimizers construct like the reference's
    assert ecoint8.EcoSGDM([]).stats == {"skipped": 0, "mean_abs_e": 0.0}
    assert ecoint8.EcoAdam([], lr=1e-3).t == 0


def test_scalar_bookkeeping_is_the_reference_arithmetic():
    """quantize_multiplier / pad_mm_dims / dynamic_scale_from_int equal the oracle's (pinned) ones."""
    from ecoint8 import fixedpoint as fp
    from oracle import fixedpoint as ofp

    gen = torch.Generator().manual_seed(0)
    rs = torch.exp(torch.empty(5000, dtype=torch.float64).uniform_(-60, 20, generator=gen)).tolist()
    for r in rs + [0.0, 1.0, 0.5, 1 - 2 ** -40]:
        assert fp.quantize_multiplier(r) == ofp.quantize_multiplier(r)
    for m, k, n in [(1, 1, 1), (17, 13, 5), (4097, 4097, 1000)]:
        assert fp.pad_mm_dims(m, k, n) == ofp.pad_mm_dims(m, k, n)
    assert fp.dynamic_scale_from_int(0, 3.0) == 1.0


def test_state_is_integral_and_scales_are_floats():
    """tests/test_strict.py:45-56 minus the device work: buffers integral, s_m floats."""
    from ecoint8 import I8ECO, I8Linear, I8ReLU, I8Sequential

    net = I8Sequential(I8Linear(20, 32), I8ReLU(), I8Linear(32, 2))
    opt = I8ECO(net.int8_layers(), lr=0.5, momentum=0.9)
    for t, p in net.named_buffers():
        assert p.dtype in {torch.int8, torch.int32, torch.int64}, t
    assert all(m.dtype == torch.int8 for m in opt.m_i8)
    assert all(isinstance(s, float) for s in opt.s_m)
    opt.s_m[1] = 0.25
    assert opt.s_m == [1.0, 0.25]
    assert opt.memory_bytes() == 20 * 32 + 32 * 2


def test_weight_steps_track_edits_and_pickle():
    import io

    from ecoint8 import I8Linear

    lin = I8Linear(8, 4)
    v0 = lin.sw.version
    lin.sw[0] = 0.5
    lin.sw += [0.1]
    lin.sw.pop()
    assert lin.sw.version == v0 + 3 and isinstance(lin.sw, list)
    lin.sw = [1.0, 2.0, 3.0, 4.0]
    assert lin.sw == [1.0, 2.0, 3.0, 4.0] and hasattr(lin.sw, "version")
    buf = io.BytesIO()
    torch.save(lin, buf)
    buf.seek(0)
    back = torch.load(buf, weights_only=False)
    assert back.sw == [1.0, 2.0, 3.0, 4.0] and torch.equal(back.w_i8, lin.w_i8)
    # a statistics snapshot keeps the values it was taken with across later edits
    tok = back.sw.snapshot()
    assert type(back.sw).values(tok) == [1.0, 2.0, 3.0, 4.0]
    back.sw[1] = 9.0
    back.sw.append(5.0)
    assert type(back.sw).values(tok) == [1.0, 2.0, 3.0, 4.0]
    assert type(back.sw).values(back.sw.snapshot()) == [1.0, 9.0, 3.0, 4.0, 5.0]


def test_replay_sites_follow_reference_order_without_gpu():
    """Replay mode asks the draw function in the reference's order with its shapes/denominators."""
    from ecoint8 import _sr

    calls = []

    def fn(shape, denom, device):
        calls.append((tuple(shape), denom))
        return torch.zeros(tuple(shape), dtype=torch.int32)

    with _sr.replay(fn):
        s1 = _sr.draw((4, 5), 12, torch.device("cpu"), batch=True)
        s2 = _sr.draw((4, 5), -3, torch.device("cpu"), batch=True)  # left shift: no draw
    assert calls == [((4, 5), 4096)] and s1.nudge is not None and s2.nudge is None


def test_device_scale_reads_and_overflow_flags_on_host_tensors():
    """The device-scale holder turns the kernel's double bits into the reference's float, and
    an overflow flag raised by the scale kernel becomes the reference's ValueError."""
    import struct

    from ecoint8 import _scale

    bits = struct.unpack("<q", struct.pack("<d", 0.0123456789))[0]
    s = _scale.DevScale(torch.tensor([bits, 1 << 30, 40], dtype=torch.int64))
    assert float(s) == 0.0123456789 and _scale.as_float(s) == 0.0123456789 and _scale.as_float(2.5) == 2.5
    assert _scale.gain_args(0.5) == (None, 0.5) and _scale.gain_args(s)[0] == s.t.data_ptr()
    dev = torch.device("cpu")
    f = _scale.flags(dev)
    f.fill_(1)  # what the scale kernel sets for a shift beyond 62
    with pytest.raises(ValueError, match="Overflow when unpacking long long"):
        _scale.raise_flags(dev)
    assert int(f) == 0
    _scale.raise_flags(dev)  # cleared: no error
    f.fill_(2)
    with pytest.raises(AssertionError):
        _scale.raise_flags(dev)


def test_reserved_philox_site_keeps_its_place_in_the_site_log():
    """A key reserved for the dW site before the dX site is drawn stays first in the log,
    even though the dW site is built (its shift known) after the dX site."""
    from ecoint8 import _sr

    torch.manual_seed(3)
    _sr.LOG = []
    try:
        key_w = _sr.reserve_key()
        site_x = _sr.draw((8, 4), 40, torch.device("cpu"), batch=True, kind="dx")
        site_w = _sr.site_from_key(key_w, (4, 6), 37, 0, "dw")
        key_n = _sr.reserve_key()
        _sr.site_from_key(key_n, (2, 2), -1, 0, "dw")  # left shift: no draw, marked "none"
        log = _sr.LOG
    finally:
        _sr.LOG = None
    assert [e[0] for e in log] == ["dw", "dx", "none"]
    assert log[0][1] == key_w and log[0][4] == 37 and log[1][4] == 40
    assert site_w.spec.seed == key_w and site_x.spec.seed == log[1][1]
    torch.manual_seed(3)  # the keys are the CPU generator's draws, in order
    assert [_sr.new_key() for _ in range(3)] == [key_w, log[1][1], key_n]


def test_optimizer_and_layers_pickle_like_the_reference():
    """torch.save of the optimizer and of the layers (the reference's plain objects pickle);
    launch caches are rebuilt after loading."""
    import io

    from ecoint8 import I8ECO, I8Linear

    layers = [I8Linear(16, 8), I8Linear(8, 4, bias=False)]
    opt = I8ECO(layers, lr=0.25, momentum=0.8, grad_clip=None)
    opt.s_m = [0.5, 0.25]
    opt.step_count = 3
    opt._plan_cache = object()  # a launch cache that must not be pickled
    buf = io.BytesIO()
    torch.save((layers, opt), buf)
    buf.seek(0)
    layers2, opt2 = torch.load(buf, weights_only=False)
    assert opt2.s_m == [0.5, 0.25] and opt2.step_count == 3 and opt2.lr == 0.25 and opt2.beta == 0.8
    assert not hasattr(opt2, "_plan_cache") and opt2._state is None
    assert all(torch.equal(a.w_i8, b.w_i8) for a, b in zip(layers, layers2))
    assert all(torch.equal(a, b) for a, b in zip(opt.m_i8, opt2.m_i8))


def test_captured_step_pushes_weight_rows_after_each_replay(monkeypatch):
    """Under the peer exchange, a step being captured as a CUDA graph does not record its
    weight-row pushes (the graph would wait for them at every replay's end): it leaves
    them to a replay hook; an uncaptured step pushes at once."""
    from ecoint8 import graphs, parallel

    pushed = []

    class FakePeer:
        def push_weight_rows(self, bufs, lo, hi):
            pushed.append((bufs, lo, hi))

    class FakeGraph:
        def __init__(self):
            self.hooks = []

        def on_replay(self, fn):
            self.hooks.append(fn)

    bufs = object()
    monkeypatch.setattr(parallel, "_PEER", FakePeer())
    monkeypatch.setattr(parallel, "peer_bufs", lambda layer, b=None: bufs)
    parallel.gather_rows("layer", (8, 16))  # eager: pushed at once
    assert pushed == [(bufs, 8, 16)]
    g = FakeGraph()
    monkeypatch.setattr(graphs, "_ACTIVE", g)
    parallel.gather_rows("layer", (8, 16))  # captured: nothing recorded, one hook
    assert pushed == [(bufs, 8, 16)] and len(g.hooks) == 1
    monkeypatch.setattr(graphs, "_ACTIVE", None)
    for _ in range(3):  # every replay is followed by the push
        g.hooks[0]()
    assert pushed == [(bufs, 8, 16)] * 4
