"""ctypes binding of the C ABI in ``include/ecoint8_b200.h`` (``lib/libecoint8_b200.so``).

Every tensor operation of this package goes through this module.  There is no
CPU path: a CPU tensor, a missing library or a non-sm_100 device raises
``RuntimeError``.  Calls are enqueued on ``torch.cuda.current_stream()``.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

_PKG_ROOT = pathlib.Path(__file__).resolve().parent.parent
LIB_PATH = _PKG_ROOT / "lib" / "libecoint8_b200.so"

ECO_OK = 0
SR_NEAREST, SR_PHILOX, SR_REPLAY32, SR_REPLAY64, SR_REPLAY_F32, SR_PHILOX_DEV = 0, 1, 2, 3, 4, 5
FLAG_SHIFT_OVERFLOW, FLAG_BAD_RATIO, FLAG_WAIT_TIMEOUT = 1, 2, 4

c_i64, c_u64, c_i32, c_u32, c_p, c_d, c_f = (ctypes.c_int64, ctypes.c_uint64, ctypes.c_int32, ctypes.c_uint32,
                                             ctypes.c_void_p, ctypes.c_double, ctypes.c_float)


class SRSpec(ctypes.Structure):
    """``eco_sr_t``."""

    _fields_ = [("mode", c_i32), ("pad_", c_i32), ("nudge", c_p), ("nudge_ld", c_i64), ("seed", c_u64),
                ("stream", c_u64), ("row_base", c_i64)]


class I8ECOLayer(ctypes.Structure):
    """``eco_i8eco_layer_t``."""

    _fields_ = [("w", c_p), ("m", c_p), ("g", c_p), ("sw", c_p), ("rowsum", c_p), ("gsq", c_p), ("state", c_p),
                ("b_acc", c_p), ("gb_sum", c_p), ("nudge_w", c_p), ("nudge_m", c_p), ("nudge_b", c_p),
                ("rows", c_i64), ("cols", c_i64), ("row_base", c_i64), ("sw_min", c_d), ("sw_max", c_d), ("s_g", c_d),
                ("s_gb", c_d), ("sx", c_d), ("stream_w", c_u64), ("stream_b", c_u64),
                ("nudge_m_bits", c_i32), ("nudge_b_bits", c_i32), ("bias_rows", c_i64),
                ("s_g_dev", c_p), ("s_gb_dev", c_p)]


class I8ECOHyper(ctypes.Structure):
    """``eco_i8eco_hyper_t``."""

    _fields_ = [("lr", c_d), ("grad_clip", c_d), ("b_q", c_i64), ("nb_q", c_i64), ("lr_q", c_i64),
                ("a_q", c_i64), ("sr_mode", c_i32), ("finalize", c_i32), ("seed", c_u64), ("done_counter", c_p),
                ("dev", c_p)]


class Fp32Layer(ctypes.Structure):
    """``eco_fp32_layer_t``."""

    _fields_ = [("w", c_p), ("m", c_p), ("v", c_p), ("g", c_p), ("sw", c_p), ("s_fixed", c_p), ("u", c_p),
                ("rows", c_i64), ("cols", c_i64), ("stream", c_u64), ("norm_out", c_p), ("stepped_out", c_p)]


class Fp32Hyper(ctypes.Structure):
    """``eco_fp32_hyper_t``."""

    _fields_ = [("kind", c_i32), ("sr_mode", c_i32), ("lr", c_d), ("beta1", c_d), ("beta2", c_d), ("eps", c_d),
                ("weight_decay", c_d), ("grad_clip", c_d), ("bc1", c_d), ("bc2", c_d), ("seed", c_u64)]


# name -> (restype, argtypes); one line per entry point of the header
_SIGS = {
    "eco_abi_version": (c_i32, []),
    "eco_last_error": (ctypes.c_char_p, []),
    "eco_device_supported": (c_i32, [c_i32]),
    "eco_gemm_s8s32": (c_i32, [c_p, c_i64, c_i32, c_p, c_i64, c_i32, c_i64, c_i64, c_i64, c_p, c_p, c_i64, c_p,
                               c_p]),
    "eco_gemm_s8s32_noalloc": (c_i32, [c_p, c_i64, c_i32, c_p, c_i64, c_i32, c_i64, c_i64, c_i64, c_p, c_p, c_i64,
                                       c_p, c_p]),
    "eco_set_gemm_sm_limit": (c_i32, [c_i32]),
    "eco_split_cols_s8": (c_i32, [c_p, c_i64, c_i64, c_i64, c_i64, c_p, c_p]),
    "eco_scale_from_amax": (c_i32, [c_p, c_i32, c_p, c_d, c_d, c_p, c_p, c_p]),
    "eco_requant_s32_s8_dev": (c_i32, [c_p, c_i64, c_i64, c_i64, c_p, c_i32, SRSpec, c_p, c_i64, c_p, c_i64, c_p,
                                       c_p]),
    "eco_peer_push_s8": (c_i32, [c_p, c_i64, c_i64, c_i64, c_p, c_i32, c_i64, c_i64, c_i32, c_i32, c_p]),
    "eco_peer_push_signal_s8": (c_i32, [c_p, c_i64, c_i64, c_i64, c_p, c_i32, c_i64, c_i64, c_i32, c_i32, c_p, c_i32,
                                        c_i32, c_i32, c_i64, c_p, c_p, c_p]),
    "eco_peer_allreduce_i64": (c_i32, [c_p, c_i32, c_i32, c_i32, c_p, c_i32, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_i64,
                                       c_p, c_p, c_p]),
    "eco_peer_signal": (c_i32, [c_p, c_i32, c_i32, c_i32, c_i64, c_p, c_p]),
    "eco_peer_wait": (c_i32, [c_p, c_i32, c_i32, c_i64, c_p, c_i64, c_p]),
    "eco_ce_grad_rowstats": (c_i32, [c_p, c_i64, c_i64, c_i64, c_d, c_p, c_i64, c_p, c_p, c_p, c_p]),
    "eco_ce_grad_quantize": (c_i32, [c_p, c_i64, c_i64, c_i64, c_d, c_p, c_i64, c_p, c_p, c_i32, SRSpec, c_p, c_i64,
                                     c_p, c_p, c_p, c_p, c_p]),
    "eco_ipc_export": (c_i32, [c_p, c_p, ctypes.POINTER(c_i64)]),
    "eco_ipc_open": (c_i32, [c_p, ctypes.POINTER(c_p)]),
    "eco_ipc_close": (c_i32, [c_p]),
    "eco_gemm_s8_requant": (c_i32, [c_p, c_i64, c_i32, c_p, c_i64, c_i32, c_i64, c_i64, c_i64, c_p, c_p, c_i32,
                                    c_i32, SRSpec, c_p, c_i64, c_p]),
    "eco_requant_s32_s8": (c_i32, [c_p, c_i64, c_i64, c_i64, c_p, c_p, c_i64, c_i32, c_i32, SRSpec, c_p, c_i64,
                                   c_p, c_i64, c_p, c_p]),
    "eco_apply_mult_shift": (c_i32, [c_p, c_i32, c_i64, c_i64, c_p, c_i32, c_i64, c_i32, SRSpec, c_p, c_p]),
    "eco_colsum_s8": (c_i32, [c_p, c_i64, c_i64, c_i64, c_p, c_p]),
    "eco_amax": (c_i32, [c_p, c_i32, c_i64, c_p, c_p]),
    "eco_sumsq_s8": (c_i32, [c_p, c_i64, c_p, c_p]),
    "eco_read_device_errors": (c_i32, [ctypes.POINTER(c_u32)]),
    "eco_copy2d_s8": (c_i32, [c_p, c_i64, c_p, c_i64, c_i64, c_i64, c_p]),
    "eco_i8eco_step": (c_i32, [ctypes.POINTER(I8ECOLayer), c_i32, ctypes.POINTER(I8ECOHyper), c_p]),
    "eco_i8eco_finalize": (c_i32, [c_p, c_i32, c_p]),
    "eco_sgdm_step": (c_i32, [c_p, c_p, c_p, c_i64, c_i64, c_p, c_p, c_f, c_f, c_f, c_f, c_u64, c_p, c_p]),
    "eco_gemm_s8_dequant": (c_i32, [c_p, c_i64, c_i32, c_p, c_i64, c_i32, c_i64, c_i64, c_i64, c_p, c_d, c_p, c_d,
                                    c_p, c_p, c_p, c_i64, c_p]),
    "eco_quantize_dynamic_f32": (c_i32, [c_p, c_i64, c_i64, c_i64, c_p, c_p, c_i64, c_p, c_p]),
    "eco_fp32_eco_step": (c_i32, [ctypes.POINTER(Fp32Layer), c_i32, ctypes.POINTER(Fp32Hyper), c_p, c_i64, c_p]),
    "eco_fp32_eco_scratch_len": (c_i64, [ctypes.POINTER(Fp32Layer), c_i32]),
}

_lib = None
_lock = threading.Lock()
_checked_devices: set[int] = set()


def load() -> ctypes.CDLL:
    """Load the library once (RuntimeError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"ecoint8 B200 library not built ({LIB_PATH}); run `python eco-int8-opt_b200/build.py`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    return load().eco_last_error().decode(errors="replace")


def call(name: str, *args) -> None:
    rc = getattr(load(), name)(*args)
    if rc != ECO_OK:
        raise RuntimeError(f"{name} failed ({rc}): {last_error()}")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one sm_100 CUDA device; there is deliberately no CPU path."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("ecoint8 (B200 build) runs on CUDA tensors only; got a tensor on "
                               f"{t.device} (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no tensor given")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _checked_devices:
        ok = load().eco_device_supported(idx)
        if ok != 1:
            raise RuntimeError(f"ecoint8 (B200 build) needs an sm_100 GPU; device {idx} is not one")
        _checked_devices.add(idx)
    return dev


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream() -> int:
    """The current CUDA stream of the current device as a handle (no Stream object built)."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def sr_spec(mode=SR_NEAREST, nudge: torch.Tensor | None = None, seed=0, stream_id=0, row_base=0) -> SRSpec:
    """``eco_sr_t``.  A ``seed`` that is a device key (``_graphs.DevKey``, a word of a
    captured graph's table) turns a Philox site into ``ECO_SR_PHILOX_DEV``."""
    s = SRSpec()
    dev_key = getattr(seed, "ptr", None)
    if dev_key is not None:
        if mode != SR_PHILOX:
            raise ValueError("a device key needs a Philox site")
        s.mode = SR_PHILOX_DEV
        s.nudge = dev_key
        s.nudge_ld = 0
        s.seed = 0
        s.stream = stream_id & 0xFFFFFFFFFFFFFFFF
        s.row_base = row_base
        return s
    s.mode = mode
    s.nudge = ptr(nudge)
    s.nudge_ld = 0 if nudge is None else (nudge.shape[-1] if nudge.dim() else 1)
    s.seed = seed & 0xFFFFFFFFFFFFFFFF
    s.stream = stream_id & 0xFFFFFFFFFFFFFFFF
    s.row_base = row_base
    return s


def read_device_errors() -> int:
    v = c_u32(0)
    call("eco_read_device_errors", ctypes.byref(v))
    return v.value
