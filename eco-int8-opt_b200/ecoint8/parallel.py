"""Data parallelism for the strict int8 step: one process per GPU, NCCL over NVLink.

The batch is split across ranks; everything else is replicated.  The only
exchanges are the ones the single-device arithmetic needs to stay bit-exact:

* forward: none (frozen scales);
* backward, per layer: int32 dW and int64 bias column sums are summed
  (integer addition is associative, so the sum equals the single-device
  accumulator bit for bit), the dW max|acc| is taken after the sum, and the
  dX max|acc| (a global scale in the reference) is a MAX across ranks;
* calibration: the forward max|acc| is a MAX across ranks.

Stochastic rounding numbers batch rows globally (``ecoint8._sr.batch_rows``),
and every rank draws the same Philox keys, so ``n`` ranks reproduce the
single-device result on the concatenated batch exactly.  The optimizer step
is replicated (identical inputs, identical draws) and needs no exchange.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _ops

_ACTIVE = False
_GROUP = None


def init(group=None) -> None:
    """Enable the exchanges on ``group`` (default: the world group)."""
    global _ACTIVE, _GROUP
    if not dist.is_initialized():
        raise RuntimeError("ecoint8.parallel.init needs torch.distributed to be initialized")
    _ACTIVE, _GROUP = True, group


def shutdown() -> None:
    global _ACTIVE, _GROUP
    _ACTIVE, _GROUP = False, None


def active() -> bool:
    return _ACTIVE and dist.is_initialized() and dist.get_world_size(_GROUP) > 1


def allreduce_max_int(v: int, device=None) -> int:
    t = torch.tensor([int(v)], dtype=torch.int64, device=device or _device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_GROUP)
    return int(t.item())


def _device():
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")


def reduce_backward(dw_acc: torch.Tensor, gb_sum: torch.Tensor, amax: torch.Tensor, amax_fn=None):
    """Sum dW and the bias sums across ranks; return (amax_dW, amax_dX, dW, gb) with global maxima.

    ``amax`` holds this rank's [max|dW|, max|dX|] (int32).  ``amax_fn`` computes
    max|x| of a tensor (the library reduction by default).
    """
    amax_fn = amax_fn or (lambda t: _ops.amax(t))
    dist.all_reduce(dw_acc, op=dist.ReduceOp.SUM, group=_GROUP)
    dist.all_reduce(gb_sum, op=dist.ReduceOp.SUM, group=_GROUP)
    both = torch.cat([amax_fn(dw_acc).reshape(1).to(torch.int64), amax[1:2].to(torch.int64)])
    dist.all_reduce(both, op=dist.ReduceOp.MAX, group=_GROUP)
    a_dw, a_dx = both.tolist()
    return a_dw, a_dx, dw_acc, gb_sum
