"""Data parallelism for the strict int8 step: one process per GPU, NCCL over NVLink.

The batch is split across ranks.  Every exchange is exact (integer sums and
maxima), so ``n`` ranks reproduce the single-device run bit for bit:

* forward: none (frozen scales);
* backward, per layer: the int32 dW accumulator is **reduce-scattered by rows**
  (integer addition is associative) asynchronously on a dedicated NCCL group
  while the dX GEMM runs; the int64 bias column sums are summed the same way;
  the dX max|acc| (a global scale in the reference) is a MAX over a second,
  small-message group, so it never queues behind the large transfers;
* gradient finalization is deferred until the optimizer reads the gradient:
  all layers at once, one host read for every dW maximum (MAX over the row
  shards), then each rank requantizes only its rows, and the square sums for
  the gradient clip are summed on the device;
* optimizer (ZeRO-1 style): each rank steps only its rows; the row-max
  accumulators of the new momentum scale are combined with a MAX and finalized
  on the device; the updated int8 weights, int32 biases and row sums are
  all-gathered asynchronously, and a layer's next forward waits for its own.
* calibration: the forward max|acc| is a MAX across ranks.

A layer is row-sharded when its output count divides evenly by the world size
(at least 8 rows per rank); other layers all-reduce their dW and step every row
on every rank.  Stochastic rounding numbers rows globally and every rank takes
the same Philox keys, so the draws are the single-device draws.  Momentum rows
are owned by their rank: ``I8ECO.m_i8`` holds this rank's rows up to date
(``gather_momentum`` collects the rest).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _ops

_ACTIVE = False
_GROUP = None  # large transfers (dW, weights)
_SMALL = None  # scalar / small-vector collectives
_PENDING: list = []  # layers whose dW reduction is in flight
COMM_SMS = 16  # SMs the GEMMs leave free for NCCL while data parallelism is active


def init(group=None, comm_sms: int = COMM_SMS) -> None:
    """Enable the exchanges on ``group`` (default: the world).  Collective: call on every rank.

    ``comm_sms``: SMs the persistent GEMMs leave to NCCL, so the dW
    reduce-scatter and the weight all-gather overlap the GEMMs instead of
    waiting for them to finish.
    """
    global _ACTIVE, _GROUP, _SMALL
    if not dist.is_initialized():
        raise RuntimeError("ecoint8.parallel.init needs torch.distributed to be initialized")
    _GROUP = group
    ranks = list(range(dist.get_world_size())) if group is None else dist.get_process_group_ranks(group)
    _SMALL = dist.new_group(ranks=ranks)
    _ACTIVE = True
    if torch.cuda.is_available() and comm_sms > 0 and len(ranks) > 1:
        from . import _native

        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        _native.call("eco_set_gemm_sm_limit", max(1, sms - comm_sms))


def shutdown() -> None:
    global _ACTIVE, _GROUP, _SMALL
    finalize_pending()
    _ACTIVE, _GROUP, _SMALL = False, None, None
    if torch.cuda.is_available():
        from . import _native

        try:
            _native.call("eco_set_gemm_sm_limit", 0)
        except RuntimeError:
            pass


def active() -> bool:
    return _ACTIVE and dist.is_initialized() and dist.get_world_size(_GROUP) > 1


def world() -> int:
    return dist.get_world_size(_GROUP)


def rank() -> int:
    return dist.get_rank(_GROUP)


def _device():
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")


def allreduce_max_int(v: int, device=None) -> int:
    t = torch.tensor([int(v)], dtype=torch.int64, device=device or _device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_SMALL if _SMALL is not None else _GROUP)
    return int(t.item())


def shard_rows(out: int):
    """This rank's ``(lo, hi)`` rows of a layer with ``out`` rows, or None (replicated)."""
    n = world()
    if out % n or out // n < 8:
        return None
    r = rank()
    return r * out // n, (r + 1) * out // n


# -- backward ------------------------------------------------------------------
def reduce_backward(dw_acc: torch.Tensor, gb_sum: torch.Tensor, amax: torch.Tensor, amax_fn=None):
    """Blocking exchange: sum dW and the bias sums, global maxima.  Returns
    ``(amax_dW, amax_dX, dW, gb)``.  ``amax`` holds this rank's [max|dW|, max|dX|]."""
    amax_fn = amax_fn or (lambda t: _ops.amax(t))
    dist.all_reduce(dw_acc, op=dist.ReduceOp.SUM, group=_GROUP)
    dist.all_reduce(gb_sum, op=dist.ReduceOp.SUM, group=_GROUP)
    both = torch.cat([amax_fn(dw_acc).reshape(1).to(torch.int64), amax[1:2].to(torch.int64)])
    dist.all_reduce(both, op=dist.ReduceOp.MAX, group=_SMALL if _SMALL is not None else _GROUP)
    a_dw, a_dx = both.tolist()
    return a_dw, a_dx, dw_acc, gb_sum


def start_dw_reduction(layer, dw_acc: torch.Tensor, gb_sum: torch.Tensor, s_g: float) -> None:
    """Launch the asynchronous dW / bias-sum reduction of one layer's backward."""
    out = dw_acc.shape[0]
    rows = shard_rows(out)
    if rows is None:
        work = dist.all_reduce(dw_acc, op=dist.ReduceOp.SUM, group=_GROUP, async_op=True)
        red = dw_acc
    else:
        lo, hi = rows
        red = torch.empty((hi - lo, dw_acc.shape[1]), dtype=dw_acc.dtype, device=dw_acc.device)
        work = dist.reduce_scatter_tensor(red, dw_acc, op=dist.ReduceOp.SUM, group=_GROUP, async_op=True)
    layer._dw_pending = {"red": red, "full": dw_acc, "work": work, "gb": gb_sum, "rows": rows, "s_g": float(s_g)}
    _PENDING.append(layer)


def global_max_dx(amax_dx: torch.Tensor) -> int:
    t = amax_dx.reshape(1).to(torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_SMALL)
    return int(t.item())


def finalize_pending() -> None:
    """Complete every in-flight dW reduction: all layers at once (one host read)."""
    if not _PENDING:
        return
    layers = list(_PENDING)
    _PENDING.clear()
    # the bias column sums of every pending layer in one all-reduce
    gbs = [l._dw_pending["gb"] for l in layers]
    flat = torch.cat(gbs)
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=_SMALL)
    off = 0
    for l, g in zip(layers, gbs):
        l._dw_pending["gb"] = flat[off:off + g.numel()]
        off += g.numel()
    for layer in layers:
        layer._dw_pending["work"].wait()
    dev = layers[0].w_i8.device
    maxima = torch.cat([_ops.amax(l._dw_pending["red"]).reshape(1) for l in layers])
    dist.all_reduce(maxima, op=dist.ReduceOp.MAX, group=_SMALL)
    sumsq = torch.zeros(len(layers), dtype=torch.int64, device=dev)
    for i, (layer, a_dw) in enumerate(zip(layers, maxima.tolist())):
        replicated = layer._dw_pending["rows"] is None
        layer._finalize_dw(int(a_dw), sumsq[i:i + 1])
        if replicated and rank() != 0:  # every rank holds the whole layer: count it once
            sumsq[i:i + 1].zero_()
    dist.all_reduce(sumsq, op=dist.ReduceOp.SUM, group=_SMALL)
    for i, layer in enumerate(layers):
        layer._gw_sumsq = sumsq[i:i + 1]
        layer._gw_sumsq_of = layer.__dict__["_gw_i8_store"]


# -- optimizer --------------------------------------------------------------------
def combine_step_state(state: torch.Tensor) -> None:
    """MAX of the row-max accumulators and error flags (columns 1, 2) over the row shards."""
    part = state[:, 1:3].contiguous()
    dist.all_reduce(part, op=dist.ReduceOp.MAX, group=_SMALL)
    state[:, 1:3].copy_(part)


def gather_rows(layer, rowsum: torch.Tensor, rows) -> None:
    """All-gather this rank's updated rows of w, b_acc and the row sums (asynchronous)."""
    works = [dist.all_gather_into_tensor(layer.w_i8, layer.w_i8[rows[0]:rows[1]], group=_GROUP, async_op=True),
             dist.all_gather_into_tensor(rowsum, rowsum[rows[0]:rows[1]], group=_GROUP, async_op=True)]
    if layer.use_bias:
        works.append(dist.all_gather_into_tensor(layer.b_acc, layer.b_acc[rows[0]:rows[1]], group=_GROUP,
                                                 async_op=True))
    layer._gather_works = works


def wait_gathers(layer) -> None:
    works = layer.__dict__.get("_gather_works")
    if works:
        for w in works:
            w.wait()
        layer._gather_works = None


def synchronize(layers) -> None:
    """Make the current stream wait for every pending all-gather of these layers' rows
    (read weights, biases or statistics only after this, or after the next forward)."""
    for layer in layers:
        wait_gathers(layer)


def gather_momentum(opt) -> None:
    """Collective: bring every rank's momentum rows into ``opt.m_i8`` on all ranks."""
    for layer, m in zip(opt.layers, opt.m_i8):
        rows = shard_rows(m.shape[0])
        if rows is not None:
            dist.all_gather_into_tensor(m, m[rows[0]:rows[1]].clone(), group=_GROUP)
