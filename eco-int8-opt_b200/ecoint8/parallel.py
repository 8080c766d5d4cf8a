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
* optimizer (ZeRO-1 style): each rank steps only its weight rows (every rank
  steps every bias, which needs no weights); the row-max accumulators of the
  new momentum scale are combined with a MAX and finalized on the device; the
  updated int8 weights are all-gathered asynchronously, one collective per
  layer, and a layer's next forward waits for its own; the per-row |e| sums of
  all layers travel in one more all-gather.
* calibration: the forward max|acc| is a MAX across ranks.

Two ways of forming the summed dW rows (``init(dw_exchange=...)``):

* ``"reduce"``: every rank computes dW over its own batch rows and the int32
  accumulators are reduce-scattered by rows (4 bytes per dW element cross
  NVLink);
* ``"gather"``: the int8 layer inputs are all-gathered during the forward and the
  int8 dY column blocks are exchanged all-to-all in the backward, so each rank
  computes its own dW rows over the whole global batch in one GEMM (the same
  exact int32 sums; about half the bytes of the reduce-scatter, and no full-size
  int32 dW in HBM).  Needs the same batch size on every rank.
* ``"peer"``: the same data as ``"gather"``, moved by the library's own kernels
  as NVLink stores into buffers mapped on every rank (``_peer``), with flag
  barriers; the weight rows after the step travel the same way.  NCCL only
  carries the small maxima and sums.

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

from . import _native as nat
from . import _ops

_ACTIVE = False
_GROUP = None  # large transfers (dW, weights)
_SMALL = None  # scalar / small-vector collectives
_ACT = None  # activation all-gathers and dY all-to-all ("gather" exchange)
_EXCHANGE = "reduce"
_PEER = None  # _peer.Exchange of the "peer" exchange, created on first use
_PUSH_CTAS = [16]
_PENDING: list = []  # layers whose dW reduction is in flight
COMM_SMS = 16  # SMs the GEMMs leave free for NCCL while data parallelism is active


def init(group=None, comm_sms: int = COMM_SMS, dw_exchange: str = "reduce", push_ctas: int = 16) -> None:
    """Enable the exchanges on ``group`` (default: the world).  Collective: call on every rank.

    ``comm_sms``: SMs the persistent GEMMs leave to the exchange, so the dW
    reduce-scatter and the weight all-gather overlap the GEMMs instead of
    waiting for them to finish.  ``dw_exchange``: ``"reduce"``, ``"gather"`` or
    ``"peer"`` (module docstring).  ``push_ctas``: CTAs of each push kernel of
    the peer exchange.
    """
    global _ACTIVE, _GROUP, _SMALL, _ACT, _EXCHANGE
    if not dist.is_initialized():
        raise RuntimeError("ecoint8.parallel.init needs torch.distributed to be initialized")
    if dw_exchange not in ("reduce", "gather", "peer"):
        raise ValueError(f"dw_exchange must be 'reduce', 'gather' or 'peer', got {dw_exchange!r}")
    _GROUP = group
    ranks = list(range(dist.get_world_size())) if group is None else dist.get_process_group_ranks(group)
    _SMALL = dist.new_group(ranks=ranks)
    _ACT = dist.new_group(ranks=ranks) if dw_exchange == "gather" else None
    _EXCHANGE = dw_exchange
    _PUSH_CTAS[0] = int(push_ctas)
    _ACTIVE = True
    if torch.cuda.is_available() and comm_sms > 0 and len(ranks) > 1:
        from . import _native

        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        _native.call("eco_set_gemm_sm_limit", max(1, sms - comm_sms))


def shutdown() -> None:
    global _ACTIVE, _GROUP, _SMALL, _ACT, _EXCHANGE, _PEER
    finalize_pending()
    if _PEER is not None:
        _PEER.release()
    _ACTIVE, _GROUP, _SMALL, _ACT, _EXCHANGE, _PEER = False, None, None, None, "reduce", None
    if torch.cuda.is_available():
        from . import _native

        try:
            _native.call("eco_set_gemm_sm_limit", 0)
        except RuntimeError:
            pass


def active() -> bool:
    return _ACTIVE and dist.is_initialized() and dist.get_world_size(_GROUP) > 1


def exchange() -> str:
    return _EXCHANGE


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
    from . import graphs

    if graphs.capturing() is not None:
        raise RuntimeError("capturing a data-parallel step needs every layer row-sharded under the peer "
                           f"exchange (a layer of {dw_acc.shape[0]} rows does not split over {world()} ranks)")
    out = dw_acc.shape[0]
    rows = shard_rows(out)
    if rows is None:
        work = dist.all_reduce(dw_acc, op=dist.ReduceOp.SUM, group=_GROUP, async_op=True)
        red = dw_acc
    else:
        lo, hi = rows
        red = torch.empty((hi - lo, dw_acc.shape[1]), dtype=dw_acc.dtype, device=dw_acc.device)
        work = dist.reduce_scatter_tensor(red, dw_acc, op=dist.ReduceOp.SUM, group=_GROUP, async_op=True)
    layer._dw_pending = {"red": red, "full": dw_acc, "shape": tuple(dw_acc.shape), "work": work, "gb": gb_sum,
                         "rows": rows, "s_g": s_g}
    _PENDING.append(layer)


# -- "gather" exchange ---------------------------------------------------------------
def gathers_input(layer) -> bool:
    """Whether ``layer``'s forward all-gathers its input (the "gather" exchange on a row-sharded layer)."""
    return active() and _EXCHANGE == "gather" and shard_rows(layer.out_features) is not None


def gather_input(layer, x_i8: torch.Tensor) -> None:
    """Start the all-gather of a layer's int8 input over the global batch (rank-major rows)."""
    x = x_i8.contiguous()
    full = torch.empty((world() * x.shape[0], x.shape[1]), dtype=x.dtype, device=x.device)
    work = dist.all_gather_into_tensor(full, x, group=_ACT, async_op=True)
    layer._input_gather = (full, work)


def column_blocks(g_i8: torch.Tensor) -> torch.Tensor:
    """``[b, out]`` -> ``[world, b, out / world]``: column block s as one contiguous block (CUDA)."""
    n = world()
    b, out = g_i8.shape
    c = out // n
    g = _ops._rowmajor(g_i8)
    nat.require_cuda(g)
    send = torch.empty((n, b, c), dtype=g.dtype, device=g.device)
    nat.call("eco_split_cols_s8", g.data_ptr(), g.stride(0) if b > 1 else out, b, out, n, send.data_ptr(),
             nat.stream())
    return send


def exchange_blocks(send: torch.Tensor):
    """All-to-all of ``column_blocks``: block s goes to rank s.  Returns the
    ``[world * b, c]`` columns of this rank over the global batch (rows in the
    order of ``gather_input``) and the work handle."""
    n, b, c = send.shape
    recv = torch.empty_like(send)
    work = dist.all_to_all_single(recv, send, group=_ACT, async_op=True)
    return recv.view(n * b, c), work


def exchange_grad_columns(g_i8: torch.Tensor):
    """Start the all-to-all that gives each rank its dY columns over the global batch."""
    return exchange_blocks(column_blocks(g_i8))


# -- "peer" exchange --------------------------------------------------------------
def peer_bufs(layer, b: int | None = None):
    """The peer-exchange buffers of a row-sharded layer (created on its first forward,
    ``b`` = this rank's batch rows), or None when the layer does not use them."""
    global _PEER
    if not (active() and _EXCHANGE == "peer" and shard_rows(layer.out_features) is not None):
        return None
    if _PEER is None:
        if b is None:
            return None
        from . import _peer

        _PEER = _peer.Exchange(_GROUP if _GROUP is not None else dist.group.WORLD, layer.w_i8.device,
                               _PUSH_CTAS[0])
    if b is None:
        return _PEER.layers.get(id(layer))
    return _PEER.layer(layer, b)


def peer_forward(layer, x_i8: torch.Tensor) -> None:
    """Before a row-sharded layer's forward GEMM: wait for the other ranks' weight
    rows of the last step, then push this rank's input rows to every rank."""
    bufs = peer_bufs(layer, x_i8.shape[0])
    _PEER.wait_weights(bufs)
    _PEER.push_input(bufs, _ops._rowmajor(x_i8))


def start_dw_rows_peer(layer, g_i8: torch.Tensor, s_g: float) -> None:
    """Push this rank's dY column blocks, then (on the exchange's dW stream, once
    every rank's inputs and dY columns have arrived) this rank's dW rows in one
    GEMM over the global batch, their max|.| and the bias column sums."""
    bufs = peer_bufs(layer)
    ex = _PEER
    ex.push_grad_columns(bufs, _ops._rowmajor(g_i8))
    lo, hi = shard_rows(bufs.out)
    dws = ex.dw
    ex._after_current(dws)  # the dW stream forks from this point of the step (and joins in finalize_pending)
    with torch.cuda.stream(dws):
        ex.wait(bufs.slot_x, dws)
        ex.wait(bufs.slot_dy, dws)
        amax = torch.empty(1, dtype=torch.int32, device=bufs.x.t.device)
        red = _ops.gemm_s32(bufs.dy.t, 1, bufs.x.t, 1, hi - lo, bufs.in_f, bufs.x.t.shape[0], amax=amax)
        gb = bufs.gb.t  # this rank's rows here; the other ranks store theirs
        _ops.colsum(bufs.dy.t, out=gb[lo:hi])
        ex.push_bias_rows(bufs, lo, hi)
        bufs.done.record(dws)
    layer._dw_pending = {"red": red, "full": None, "shape": (bufs.out, bufs.in_f), "work": None, "gb": gb,
                         "event": bufs.done, "rows": (lo, hi), "s_g": s_g, "amax": amax, "peer": bufs}
    _PENDING.append(layer)


def start_dw_rows(layer, dy_cols: torch.Tensor, a2a, s_g: float) -> None:
    """This rank's rows of the summed dW in one GEMM over the global batch ("gather" exchange)."""
    full, xwork = layer._input_gather
    layer._input_gather = None
    a2a.wait()
    xwork.wait()
    out = layer.out_features
    lo, hi = shard_rows(out)
    K, in_f = full.shape
    amax = torch.empty(1, dtype=torch.int32, device=full.device)
    red = _ops.gemm_s32(dy_cols, 1, full, 1, hi - lo, in_f, K, amax=amax)
    gb = torch.zeros(out, dtype=torch.int64, device=red.device)
    gb[lo:hi] = _ops.colsum(dy_cols)  # the other rows arrive through the flat SUM in finalize_pending
    layer._dw_pending = {"red": red, "full": None, "shape": (out, in_f), "work": None, "gb": gb,
                         "rows": (lo, hi), "s_g": s_g, "amax": amax}
    _PENDING.append(layer)


class _Done:
    """The handle of an exchange that is already ordered on the current stream."""

    def wait(self) -> None:
        pass


def start_max(amax: torch.Tensor):
    """Start the MAX over ranks of a device maximum; ``finish_max`` reads it."""
    t = amax.reshape(1)
    if _PEER is not None:  # one kernel through the peer exchange's buffers
        return _PEER.allreduce(t, "max"), _Done()
    return t, dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_SMALL, async_op=True)


def max_over_ranks(t: torch.Tensor) -> torch.Tensor:
    """MAX over ranks of a short int32/int64 device vector, as int64, queued on the
    current stream (the peer exchange's kernel, else NCCL); the host does not wait."""
    if _PEER is not None:
        return _PEER.allreduce(t.reshape(-1), "max")
    out = t.reshape(-1).to(torch.int64)
    dist.all_reduce(out, op=dist.ReduceOp.MAX, group=_SMALL if _SMALL is not None else _GROUP)
    return out


def _small_reduce(t: torch.Tensor, op: str) -> torch.Tensor:
    """MAX / SUM over ranks of a short vector (the peer exchange's kernel, else NCCL in place)."""
    if _PEER is not None and t.numel() <= 1024:
        return _PEER.allreduce(t, op).to(t.dtype)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM, group=_SMALL)
    return t


def finish_max(handle) -> int:
    t, work = handle
    work.wait()
    return int(t.item())


def global_max_dx(amax_dx: torch.Tensor) -> int:
    return finish_max(start_max(amax_dx))


def finalize_pending() -> None:
    """Complete every in-flight dW reduction: all layers at once (one host read)."""
    if not _PENDING:
        return
    layers = list(_PENDING)
    _PENDING.clear()
    cur = torch.cuda.current_stream() if torch.cuda.is_available() else None
    for l in layers:  # dW rows formed on the peer exchange's stream
        p = l._dw_pending
        if p.get("event") is not None:
            cur.wait_event(p["event"])
            for t in (p["red"], p["amax"]):
                t.record_stream(cur)
        if p.get("peer") is not None:  # the other ranks' rows of the bias sums have arrived
            _PEER.wait_bias_rows(p["peer"], cur)
    # the bias column sums of the other pending layers in one all-reduce
    summed = [l for l in layers if l._dw_pending.get("peer") is None]
    if summed:
        gbs = [l._dw_pending["gb"] for l in summed]
        flat = torch.cat(gbs)
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=_SMALL)
        off = 0
        for l, g in zip(summed, gbs):
            l._dw_pending["gb"] = flat[off:off + g.numel()]
            off += g.numel()
    for layer in layers:
        if layer._dw_pending["work"] is not None:
            layer._dw_pending["work"].wait()
    dev = layers[0].w_i8.device
    # max|dW| of this rank's rows: the gather exchange's GEMM produced it already
    fused = [l._dw_pending.get("amax") for l in layers]
    if all(a is not None for a in fused):
        maxima = torch.cat(fused).to(torch.int64)
    else:
        maxima = torch.cat([a.to(torch.int64) if a is not None else _ops.amax(l._dw_pending["red"]).reshape(1)
                            for l, a in zip(layers, fused)])
    maxima = _small_reduce(maxima, "max")
    sumsq = torch.zeros(len(layers), dtype=torch.int64, device=dev)
    queued = [bool(l._dw_pending.get("queued")) for l in layers]
    host = None if all(queued) else maxima.tolist()  # a queued backward keeps the maxima on the device
    for i, layer in enumerate(layers):
        replicated = layer._dw_pending["rows"] is None
        if queued[i]:
            layer._finalize_dw_queued(maxima[i:i + 1], sumsq[i:i + 1])
        else:
            layer._finalize_dw(int(host[i]), sumsq[i:i + 1])
        if replicated and rank() != 0:  # every rank holds the whole layer: count it once
            sumsq[i:i + 1].zero_()
    sumsq = _small_reduce(sumsq, "sum")
    for i, layer in enumerate(layers):
        layer._gw_sumsq = sumsq[i:i + 1]
        layer._gw_sumsq_of = layer.__dict__["_gw_i8_store"]


# -- optimizer --------------------------------------------------------------------
def combine_step_state(state: torch.Tensor) -> None:
    """MAX of the row-max accumulators and error flags (columns 1, 2) over the row shards."""
    part = _small_reduce(state[:, 1:3].contiguous(), "max")
    state[:, 1:3].copy_(part.view(-1, 2))


def gather_rows(layer, rows) -> None:
    """All-gather this rank's updated weight rows (asynchronous; the biases are
    stepped in full on every rank)."""
    bufs = peer_bufs(layer)
    if bufs is not None:
        from . import graphs

        g = graphs.capturing()
        if g is not None:
            # Not recorded: a captured step joins its side streams before it ends, so a push
            # inside the graph would hold every replay until it finished.  Each replay is
            # followed by the push instead, queued behind it on the communication stream, and
            # the next replay's forward waits for it on the device -- the overlap an
            # uncaptured step gets.
            g.on_replay(lambda b=bufs, lo=rows[0], hi=rows[1]: _PEER.push_weight_rows(b, lo, hi))
            return
        _PEER.push_weight_rows(bufs, rows[0], rows[1])
        return
    layer._gather_works = [dist.all_gather_into_tensor(layer.w_i8, layer.w_i8[rows[0]:rows[1]], group=_GROUP,
                                                       async_op=True)]


def flat_buffer(shape, device) -> torch.Tensor:
    """The rank-major ``[world, k]`` int64 buffer of ``gather_flat`` (mapped on every rank
    under the peer exchange)."""
    if _PEER is not None:
        return _PEER.rowsum_buffer(shape[1])
    return torch.empty(shape, dtype=torch.int64, device=device)


class _PeerGather:
    """The handle of a peer row-sum gather: ``wait`` orders the current stream after it."""

    def wait(self) -> None:
        _PEER.wait_rowsum()


def gather_flat(flat: torch.Tensor):
    """All-gather a rank-major ``[world, k]`` buffer whose row ``rank()`` this rank filled."""
    if _PEER is not None and _PEER.rowsum is not None and flat.data_ptr() == _PEER.rowsum.t.data_ptr():
        _PEER.push_rowsum()
        return _PeerGather()
    return dist.all_gather_into_tensor(flat, flat[rank()], group=_SMALL, async_op=True)


def wait_gathers(layer) -> None:
    bufs = peer_bufs(layer) if _PEER is not None else None
    if bufs is not None:
        _PEER.wait_weights(bufs)
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
