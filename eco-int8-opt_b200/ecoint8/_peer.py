"""The "peer" exchange of data parallelism: NVLink stores into buffers that every
rank allocates and maps into the other ranks' processes (CUDA IPC handles: plain
unicast peer mappings, never an NVLink multicast object), ordered by flag barriers.

Per row-sharded layer every rank holds

* ``x``: the layer's int8 input over the global batch ``[world * b, in]``; each
  rank's forward pushes its ``b`` rows into every rank's copy;
* ``dy``: its dY columns over the global batch ``[world * b, out / world]``;
  each rank's backward pushes column block ``p`` of its dY rows to rank ``p``;
* ``w``: the weights themselves (the layer's ``w_i8`` buffer moves here); after
  the optimizer step each rank pushes its updated rows to the other ranks.

Pushes run on a communication stream with a few CTAs; each is followed by a
signal that writes an epoch into a flag slot on every rank, and consumers wait
for the slot on their own stream (``eco_peer_wait``, bounded).  The dW GEMM of
a layer runs on a third stream once the layer's inputs and dY columns of every
rank have arrived, so the dX chain never waits for the exchange.

Buffer reuse is ordered by the exchange itself: a rank only overwrites a peer's
``x``/``dy`` in the next step's forward/backward, which every rank reaches only
after the all-reduce of the dW maxima, which needs every rank's dW GEMM to have
read those buffers; the weight rows are pushed after that same all-reduce and
read by the next forward after its wait.
"""

from __future__ import annotations

import ctypes
import weakref

import torch
import torch.distributed as dist

from . import _native as nat

MAX_PEERS = 8  # ECO_MAX_PEERS of the C ABI
MAX_LAYERS = 256  # row-sharded layers per exchange
MAX_SLOTS = 4 * MAX_LAYERS + 2  # four flag slots per layer, the small all-reduces', the row sums'
RED_SLOT = MAX_SLOTS - 2
ROWSUM_SLOT = MAX_SLOTS - 1
RED_STRIDE = 1024  # longest vector of the small all-reduce
HANDLE_BYTES = 64  # ECO_IPC_HANDLE_BYTES of the C ABI


def _arr(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


class IpcMaps:
    """The peer allocations this process has mapped (one mapping per allocation: several
    exchange buffers can live in one allocation of the caching allocator)."""

    def __init__(self):
        self.opened: dict[tuple[int, bytes], int] = {}

    def open(self, rank: int, handle: bytes) -> int:
        base = self.opened.get((rank, handle))
        if base is None:
            p = ctypes.c_void_p()
            nat.call("eco_ipc_open", handle, ctypes.byref(p))
            base = self.opened[(rank, handle)] = int(p.value)
        return base

    def close_all(self) -> None:
        for base in self.opened.values():
            nat.call("eco_ipc_close", base)
        self.opened.clear()


class Shared:
    """A tensor allocated on every rank of ``group`` with the device pointers of all copies
    (the other ranks' copies mapped through CUDA IPC).  Collective: every rank creates the
    same sequence of them."""

    def __init__(self, shape, dtype, device, group, maps: IpcMaps):
        self.t = torch.empty(shape, dtype=dtype, device=device)
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        off = ctypes.c_int64()
        nat.call("eco_ipc_export", self.t.data_ptr(), handle, ctypes.byref(off))
        n, me = dist.get_world_size(group), dist.get_rank(group)
        every = [None] * n
        dist.all_gather_object(every, (handle.raw, off.value), group=group)
        self.ptrs = [self.t.data_ptr() if r == me else maps.open(r, h) + o for r, (h, o) in enumerate(every)]


class LayerBufs:
    def __init__(self, ex: "Exchange", layer, b: int):
        idx = len(ex.layers)
        if idx >= MAX_LAYERS:
            raise RuntimeError("ecoint8.parallel: too many row-sharded layers for the peer exchange")
        self.slot_x, self.slot_dy, self.slot_w, self.slot_gb = 4 * idx, 4 * idx + 1, 4 * idx + 2, 4 * idx + 3
        n, dev, g = ex.n, ex.dev, ex.group
        out, in_f = layer.w_i8.shape
        self.b, self.out, self.in_f = b, out, in_f
        self.x = Shared((n * b, in_f), torch.int8, dev, g, ex.maps)
        self.dy = Shared((n * b, out // n), torch.int8, dev, g, ex.maps)
        self.w = Shared((out, in_f), torch.int8, dev, g, ex.maps)
        self.w.t.copy_(layer.w_i8)
        layer._buffers["w_i8"] = self.w.t  # the weights live in the shared buffer from now on
        # the bias gradient's column sums over the global batch: each rank forms its rows
        # and stores them into every rank's copy
        self.gb = Shared((out,), torch.int64, dev, g, ex.maps)
        self.layer = weakref.ref(layer)
        self.x_ptrs = _arr(self.x.ptrs)
        self.dy_ptrs = _arr(self.dy.ptrs)
        self.w_peers = _arr([p for r, p in enumerate(self.w.ptrs) if r != ex.rank])
        lo = ex.rank * out // n
        self.gb_peers = _arr([p + 8 * lo for r, p in enumerate(self.gb.ptrs) if r != ex.rank])
        self.done = torch.cuda.Event()  # the layer's dW rows are formed (recorded on the dW stream)


class Exchange:
    """Flags, epochs, streams and per-layer buffers of one process."""

    def __init__(self, group, device, push_ctas: int = 16):
        self.group = group
        self.ctas = push_ctas  # CTAs per push kernel: the rest of the GPU keeps running the GEMMs
        self.n = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.n > MAX_PEERS:
            raise RuntimeError(f"the peer exchange supports up to {MAX_PEERS} ranks")
        self.dev = device
        self.maps = IpcMaps()
        self.flags = Shared((MAX_SLOTS, MAX_PEERS), torch.int64, device, group, self.maps)
        self.flags.t.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        self.flag_ptrs = _arr(self.flags.ptrs)
        self.epoch = [0] * MAX_SLOTS
        self.comm = torch.cuda.Stream(device)
        self.dw = torch.cuda.Stream(device)
        self._ev = torch.cuda.Event()  # reused: orders the communication stream after the current one
        self.tickets = torch.zeros(MAX_SLOTS, dtype=torch.int32, device=device)  # push-and-signal tickets
        self.red = Shared((2, self.n, RED_STRIDE), torch.int64, device, group, self.maps)  # small all-reduce areas
        self.red_ptrs = _arr(self.red.ptrs)
        self.layers: dict[int, LayerBufs] = {}
        self.rowsum: Shared | None = None  # the optimizer's per-row |e| sums, [world, rows] (one row per rank)

    # -- epochs -------------------------------------------------------------------
    # Every signal on a slot advances the slot's epoch; a wait waits for the current one.
    # While a StepGraph is captured the host epochs do not move: each call takes a word
    # of the graph's table, and every replay advances the epochs in the same order.
    def _next_epoch(self, slot: int):
        """(host epoch, device word or None) of a signal on ``slot``."""
        from . import graphs

        g = graphs.capturing()
        if g is not None:
            def bump(slot=slot):
                self.epoch[slot] += 1
                return self.epoch[slot]

            return 0, g.table.word(bump)
        self.epoch[slot] += 1
        return self.epoch[slot], None

    def _current_epoch(self, slot: int):
        from . import graphs

        g = graphs.capturing()
        if g is not None:
            return 0, g.table.word(lambda slot=slot: self.epoch[slot])
        return self.epoch[slot], None

    # -- flags ------------------------------------------------------------------
    def signal(self, slot: int, stream) -> None:
        e, e_dev = self._next_epoch(slot)
        nat.call("eco_peer_signal", self.flag_ptrs, self.n, self.rank, slot, e, e_dev, stream.cuda_stream)

    def wait(self, slot: int, stream) -> None:
        if self.epoch[slot] > 0:
            e, e_dev = self._current_epoch(slot)
            nat.call("eco_peer_wait", self.flags.t.data_ptr(), self.n, slot, e, e_dev, 0, stream.cuda_stream)

    def allreduce(self, src: torch.Tensor, op: str) -> torch.Tensor:
        """MAX or SUM over the ranks of a short int32/int64 vector, as int64, on the current stream."""
        n = src.numel()
        if n > RED_STRIDE or src.dtype not in (torch.int32, torch.int64):
            raise ValueError("the peer all-reduce takes at most 1024 int32/int64 values")
        src = src.contiguous()
        out = torch.empty(n, dtype=torch.int64, device=self.dev)
        e, e_dev = self._next_epoch(RED_SLOT)
        nat.call("eco_peer_allreduce_i64", src.data_ptr(), 32 if src.dtype == torch.int32 else 64, n,
                 0 if op == "max" else 1, self.red_ptrs, RED_STRIDE, self.red.t.data_ptr(), self.flag_ptrs,
                 self.flags.t.data_ptr(), self.n, self.rank, RED_SLOT, e, e_dev, out.data_ptr(), nat.stream())
        return out

    def _after_current(self, stream) -> None:
        self._ev.record(torch.cuda.current_stream(self.dev))
        stream.wait_event(self._ev)

    # -- layers -----------------------------------------------------------------
    def layer(self, layer, b: int) -> LayerBufs:
        bufs = self.layers.get(id(layer))
        if bufs is None:
            bufs = self.layers[id(layer)] = LayerBufs(self, layer, b)
        elif bufs.b != b:
            raise RuntimeError(f"the peer exchange needs a fixed per-rank batch ({bufs.b}), got {b}")
        return bufs

    def _push(self, src: int, ld: int, rows: int, cols: int, dst, n_dst: int, ld_dst: int, row0: int, split: int,
              slot: int) -> None:
        """One push kernel on the communication stream that signals ``slot`` when its stores are visible."""
        self._after_current(self.comm)
        e, e_dev = self._next_epoch(slot)
        nat.call("eco_peer_push_signal_s8", src, ld, rows, cols, dst, n_dst, ld_dst, row0, split, self.ctas,
                 self.flag_ptrs, self.n, self.rank, slot, e, e_dev, self.tickets[slot].data_ptr(),
                 self.comm.cuda_stream)
        from . import graphs

        g = graphs.capturing()
        if g is not None:
            g.join(self.comm)

    def push_input(self, bufs: LayerBufs, x: torch.Tensor) -> None:
        """This rank's input rows into every rank's ``x`` (rows rank * b ...)."""
        self._push(x.data_ptr(), x.stride(0) if x.shape[0] > 1 else x.shape[1], x.shape[0], x.shape[1], bufs.x_ptrs,
                   self.n, bufs.in_f, self.rank * bufs.b, 0, bufs.slot_x)
        x.record_stream(self.comm)

    def push_grad_columns(self, bufs: LayerBufs, g: torch.Tensor) -> None:
        """Column block p of this rank's dY rows into rank p's ``dy`` (rows rank * b ...)."""
        self._push(g.data_ptr(), g.stride(0) if g.shape[0] > 1 else g.shape[1], g.shape[0], g.shape[1],
                   bufs.dy_ptrs, self.n, bufs.out // self.n, self.rank * bufs.b, 1, bufs.slot_dy)
        g.record_stream(self.comm)

    def push_weight_rows(self, bufs: LayerBufs, lo: int, hi: int) -> None:
        """This rank's updated weight rows into the other ranks' ``w``."""
        w = bufs.w.t
        self._push(w.data_ptr() + lo * bufs.in_f, bufs.in_f, hi - lo, bufs.in_f, bufs.w_peers, self.n - 1,
                   bufs.in_f, lo, 0, bufs.slot_w)

    def push_bias_rows(self, bufs: LayerBufs, lo: int, hi: int) -> None:
        """This rank's rows of the bias column sums into the other ranks' ``gb``."""
        nbytes = 8 * (hi - lo)
        self._push(bufs.gb.t.data_ptr() + 8 * lo, nbytes, 1, nbytes, bufs.gb_peers, self.n - 1, nbytes, 0, 0,
                   bufs.slot_gb)

    def wait_bias_rows(self, bufs: LayerBufs, stream) -> None:
        self.wait(bufs.slot_gb, stream)

    def rowsum_buffer(self, rows: int) -> torch.Tensor:
        """The optimizer's ``[world, rows]`` int64 row-sum buffer, mapped on every rank
        (created on first use; collective)."""
        if self.rowsum is None:
            self.rowsum = Shared((self.n, rows), torch.int64, self.dev, self.group, self.maps)
            self.rowsum_peers = _arr([p + 8 * rows * self.rank for r, p in enumerate(self.rowsum.ptrs)
                                      if r != self.rank])
        elif self.rowsum.t.shape[1] != rows:
            raise RuntimeError("the peer exchange's row-sum buffer cannot change size")
        return self.rowsum.t

    def push_rowsum(self) -> None:
        """This rank's row of the row-sum buffer into the other ranks' copies."""
        nbytes = 8 * self.rowsum.t.shape[1]
        self._push(self.rowsum.t[self.rank].data_ptr(), nbytes, 1, nbytes, self.rowsum_peers, self.n - 1, nbytes,
                   0, 0, ROWSUM_SLOT)

    def wait_rowsum(self) -> None:
        self.wait(ROWSUM_SLOT, torch.cuda.current_stream(self.dev))

    def wait_weights(self, bufs: LayerBufs) -> None:
        self.wait(bufs.slot_w, torch.cuda.current_stream(self.dev))

    def release(self) -> None:
        """Give every layer a private copy of its weights again and unmap the peers'
        buffers.  Collective: no rank frees a buffer before every rank has unmapped it."""
        torch.cuda.synchronize(self.dev)
        for bufs in self.layers.values():
            layer = bufs.layer()
            if layer is not None and layer._buffers.get("w_i8") is bufs.w.t:
                layer._buffers["w_i8"] = bufs.w.t.clone()
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)  # every rank's kernels on the mapped buffers are done
        self.maps.close_all()
        dist.barrier(group=self.group)  # every rank has unmapped: the buffers may be freed
        self.layers.clear()
