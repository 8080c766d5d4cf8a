"""ecoint8 for B200: the strict int8 ECO training path on sm_100a tensor cores.

Drop-in for the public API of eco-int8-opt 0.4.9.  The strict path
(``I8Linear``/``I8ReLU``/``I8Sequential``, ``I8ECO``) and ``EcoInt8SGDM`` run on
the C-ABI CUDA library ``lib/libecoint8_b200.so``; CUDA tensors only.
"""
from .eco import EcoAdam, EcoInt8SGDM, EcoSGDM
from .layers import Int8Linear, to_int8
from .quant import dequantize, quantize_per_channel, quantize_symmetric, quantize_tensor_dynamic
from .strict import I8ECO, I8Linear, I8ReLU, I8Sequential
from . import parallel
from ._sr import replay as sr_replay, set_generator as set_sr_generator

__version__ = "0.4.9"

__all__ = [
    "EcoInt8SGDM",
    "EcoSGDM",
    "EcoAdam",
    "I8ECO",
    "I8Linear",
    "I8ReLU",
    "I8Sequential",
    "Int8Linear",
    "to_int8",
    "quantize_symmetric",
    "quantize_tensor_dynamic",
    "quantize_per_channel",
    "dequantize",
    "parallel",
    "sr_replay",
    "set_sr_generator",
    "__version__",
]
