"""Strict integer-only ECO training: int8/int32/int64 only, manual forward and
backward, frozen quantization grids, on the B200 library."""
from .ilayer import I8Linear, I8ReLU, I8Sequential
from .iopt import I8ECO

__all__ = ["I8ECO", "I8Linear", "I8ReLU", "I8Sequential"]
